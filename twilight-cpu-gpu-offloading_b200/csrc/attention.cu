// Sparse GQA decode attention over gathered K/V rows: split-K flash-decode
// with a log-sum-exp merge performed by the last split CTA of each segment.
//
// Reference: flash_attn_varlen_func as called by the GQA group path
// (hi/mp.py:258-279, wrapper :21-52): q [G, R, D], k/v [sum_T, 1, D],
// cu_seqlens_q = arange(G+1), cu_seqlens_k [G+1], q_len 1 (all keys visible),
// softmax scale 1/sqrt(D).  Segments generalise G (Twilight GQA groups, R
// heads each) and G*R (Quest per-query-head segments, 1 head each).
#include <math_constants.h>

#include <mutex>

#include "tw_common.cuh"

namespace tw {

constexpr int kAttnThreads = 128;   // 4 warps
constexpr int kAttnChunk = 128;     // rows per split CTA
constexpr int kAttnUnroll = 4;      // rows per warp iteration

struct AttnWorkspace {
  unsigned int* counters;  // [S]
  float* part_ml;          // [S][max_splits][R][2]  (m in log2 units, l)
  float* part_o;           // [S][max_splits][R][D]
};

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

inline int attn_max_splits(int max_seqlen_k) {
  return max(1, (max_seqlen_k + kAttnChunk - 1) / kAttnChunk);
}

inline size_t attn_ws_bytes(int S, int R, int max_splits, AttnWorkspace* ws, char* base) {
  size_t off = 0;
  const size_t c_bytes = align256((size_t)S * sizeof(unsigned int));
  const size_t ml_bytes = align256((size_t)S * max_splits * R * 2 * sizeof(float));
  const size_t o_bytes = align256((size_t)S * max_splits * R * kHeadDim * sizeof(float));
  if (ws) {
    ws->counters = reinterpret_cast<unsigned int*>(base + off);
    ws->part_ml = reinterpret_cast<float*>(base + off + c_bytes);
    ws->part_o = reinterpret_cast<float*>(base + off + c_bytes + ml_bytes);
  }
  return c_bytes + ml_bytes + o_bytes;
}

template <typename T> struct Vec4Of;
template <> struct Vec4Of<__half> {
  __device__ static void load(const __half* p, float (&f)[4]) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const __half2 a = *reinterpret_cast<const __half2*>(&raw.x);
    const __half2 b = *reinterpret_cast<const __half2*>(&raw.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    f[0] = fa.x; f[1] = fa.y; f[2] = fb.x; f[3] = fb.y;
  }
};
template <> struct Vec4Of<__nv_bfloat16> {
  __device__ static void load(const __nv_bfloat16* p, float (&f)[4]) {
    const uint2 raw = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    f[0] = fa.x; f[1] = fa.y; f[2] = fb.x; f[3] = fb.y;
  }
};

template <typename OutT>
__device__ __forceinline__ void store_out(OutT* p, float v) { *p = from_f32<OutT>(v); }

// Finalise one (segment, head) from merged (m, l, o[d]) held per thread d.
template <typename OutT>
__device__ __forceinline__ void write_final(OutT* out, float* lse, int s, int r, int R, float m,
                                            float l, float o) {
  const int d = threadIdx.x;
  const float inv = (l > 0.0f) ? 1.0f / l : 0.0f;
  store_out(out + ((int64_t)s * R + r) * kHeadDim + d, o * inv);
  if (lse && d == 0) {
    lse[(int64_t)s * R + r] = (l > 0.0f) ? (m + log2f(l)) * CUDART_LN2_F : -CUDART_INF_F;
  }
}

template <typename T, int R, typename OutT>
__global__ void __launch_bounds__(kAttnThreads)
decode_attention_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                        const int32_t* __restrict__ cu, float scale_log2, int max_splits,
                        AttnWorkspace ws, OutT* __restrict__ out, float* __restrict__ lse) {
  __shared__ float s_m[4][R];
  __shared__ float s_l[4][R];
  __shared__ float s_o[4][R][kHeadDim];
  __shared__ bool s_last;

  const int s = blockIdx.y;
  const int split = blockIdx.x;
  const int seg_begin = cu[s];
  // Rows beyond max_splits * kAttnChunk (a caller's max_seqlen_k below the real
  // segment length) are not read: the split count is clamped to the grid.
  const int seg_len = min(cu[s + 1] - seg_begin, max_splits * kAttnChunk);
  const int nsplit = (seg_len + kAttnChunk - 1) / kAttnChunk;
  if (split >= max(nsplit, 1)) return;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row_begin = seg_begin + split * kAttnChunk;
  const int row_end = min(seg_begin + seg_len, row_begin + kAttnChunk);

  float qf[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) Vec4Of<T>::load(q + ((int64_t)s * R + r) * kHeadDim + 4 * lane, qf[r]);

  float m[R], l[R], acc[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -CUDART_INF_F;
    l[r] = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;
  }

  for (int base = row_begin + warp; base < row_end; base += 4 * kAttnUnroll) {
    float kf[kAttnUnroll][4], vf[kAttnUnroll][4];
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int row = base + 4 * u;
      if (row < row_end) {
        Vec4Of<T>::load(k + (int64_t)row * kHeadDim + 4 * lane, kf[u]);
        Vec4Of<T>::load(v + (int64_t)row * kHeadDim + 4 * lane, vf[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kAttnUnroll; ++u) {
      const int row = base + 4 * u;
      if (row >= row_end) break;  // warp-uniform
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float dot = qf[r][0] * kf[u][0] + qf[r][1] * kf[u][1] + qf[r][2] * kf[u][2] +
                    qf[r][3] * kf[u][3];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
        const float sc = dot * scale_log2;
        const float m_new = fmaxf(m[r], sc);
        const float corr = exp2f(m[r] - m_new);
        const float p = exp2f(sc - m_new);
        l[r] = l[r] * corr + p;
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = acc[r][c] * corr + p * vf[u][c];
        m[r] = m_new;
      }
    }
  }

  // Merge the 4 warps of this CTA.
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (lane == 0) {
      s_m[warp][r] = m[r];
      s_l[warp][r] = l[r];
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) s_o[warp][r][4 * lane + c] = acc[r][c];
  }
  __syncthreads();
  const int d = threadIdx.x;  // 128 threads == kHeadDim
  float cm[R], cl[R], co[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float mm = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, s_m[w][r]);
    float ll = 0.0f, oo = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float wm = s_m[w][r];
      const float f = (wm == -CUDART_INF_F) ? 0.0f : exp2f(wm - mm);
      ll += s_l[w][r] * f;
      oo += s_o[w][r][d] * f;
    }
    cm[r] = mm;
    cl[r] = ll;
    co[r] = oo;
  }

  if (nsplit <= 1) {
#pragma unroll
    for (int r = 0; r < R; ++r) write_final<OutT>(out, lse, s, r, R, cm[r], cl[r], co[r]);
    return;
  }

  // Publish this split's partial, then the last split of the segment merges.
  float* pml = ws.part_ml + ((int64_t)s * max_splits + split) * R * 2;
  float* po = ws.part_o + ((int64_t)s * max_splits + split) * R * kHeadDim;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    po[r * kHeadDim + d] = co[r];
    if (d == 0) {
      pml[2 * r] = cm[r];
      pml[2 * r + 1] = cl[r];
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(&ws.counters[s], 1u);
    s_last = (prev == (unsigned int)nsplit - 1u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
#pragma unroll 1
  for (int r = 0; r < R; ++r) {
    float mm = -CUDART_INF_F;
    for (int j = 0; j < nsplit; ++j)
      mm = fmaxf(mm, __ldcg(ws.part_ml + (((int64_t)s * max_splits + j) * R + r) * 2));
    float ll = 0.0f, oo = 0.0f;
    for (int j = 0; j < nsplit; ++j) {
      const float* ml = ws.part_ml + (((int64_t)s * max_splits + j) * R + r) * 2;
      const float wm = __ldcg(ml);
      const float f = (wm == -CUDART_INF_F) ? 0.0f : exp2f(wm - mm);
      ll += __ldcg(ml + 1) * f;
      oo += __ldcg(ws.part_o + (((int64_t)s * max_splits + j) * R + r) * kHeadDim + d) * f;
    }
    write_final<OutT>(out, lse, s, r, R, mm, ll, oo);
  }
  if (threadIdx.x == 0) ws.counters[s] = 0u;
}

template <typename T, int R, typename OutT>
int launch_attention_r(const void* q, const void* k, const void* v, const int32_t* cu, int S,
                       int max_splits, float scale_log2, const AttnWorkspace& ws, void* out,
                       float* lse, cudaStream_t stream) {
  dim3 grid(max_splits, S);
  decode_attention_kernel<T, R, OutT><<<grid, kAttnThreads, 0, stream>>>(
      (const T*)q, (const T*)k, (const T*)v, cu, scale_log2, max_splits, ws, (OutT*)out, lse);
  return check_launch();
}

template <typename T, typename OutT>
int launch_attention(const void* q, const void* k, const void* v, const int32_t* cu, int S, int R,
                     int max_splits, float scale_log2, const AttnWorkspace& ws, void* out,
                     float* lse, cudaStream_t stream) {
#define TW_ATTN_CASE(RR)                                                                     \
  case RR:                                                                                   \
    return launch_attention_r<T, RR, OutT>(q, k, v, cu, S, max_splits, scale_log2, ws, out, \
                                           lse, stream);
  switch (R) {
    TW_ATTN_CASE(1)
    TW_ATTN_CASE(2)
    TW_ATTN_CASE(3)
    TW_ATTN_CASE(4)
    TW_ATTN_CASE(5)
    TW_ATTN_CASE(6)
    TW_ATTN_CASE(7)
    TW_ATTN_CASE(8)
    default:
      return TW_ERR_UNSUPPORTED;
  }
#undef TW_ATTN_CASE
}

}  // namespace tw

using namespace tw;

extern "C" size_t tw_decode_attention_workspace_size(int segments, int heads_per_segment,
                                                     int max_seqlen_k, int head_dim) {
  if (segments <= 0 || heads_per_segment <= 0 || max_seqlen_k < 0 || head_dim != kHeadDim)
    return 0;
  return attn_ws_bytes(segments, heads_per_segment, attn_max_splits(max_seqlen_k), nullptr,
                       nullptr);
}

extern "C" int tw_decode_attention(const void* q, const void* k, const void* v,
                                   const int32_t* cu_seqlens, int segments,
                                   int heads_per_segment, int max_seqlen_k, int head_dim,
                                   int dtype, float softmax_scale, void* out, int out_dtype,
                                   float* lse, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  if (!q || !k || !v || !cu_seqlens || !out || segments <= 0 || segments > 65535 ||
      heads_per_segment <= 0 || max_seqlen_k < 0 || !(softmax_scale > 0.0f))
    return TW_ERR_BAD_ARG;
  if (heads_per_segment > kMaxHeadsPerGroup) return TW_ERR_UNSUPPORTED;
  if (out_dtype != dtype && out_dtype != TW_F32) return TW_ERR_BAD_ARG;
  const int max_splits = attn_max_splits(max_seqlen_k);
  AttnWorkspace ws{};
  const size_t need = attn_ws_bytes(segments, heads_per_segment, max_splits, &ws,
                                    reinterpret_cast<char*>(workspace));
  if (max_splits > 1 && (!workspace || workspace_bytes < need)) return TW_ERR_CAPACITY;
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == TW_F16) {
    if (out_dtype == TW_F32)
      return launch_attention<__half, float>(q, k, v, cu_seqlens, segments, heads_per_segment,
                                             max_splits, scale_log2, ws, out, lse, st);
    return launch_attention<__half, __half>(q, k, v, cu_seqlens, segments, heads_per_segment,
                                            max_splits, scale_log2, ws, out, lse, st);
  }
  if (dtype == TW_BF16) {
    if (out_dtype == TW_F32)
      return launch_attention<__nv_bfloat16, float>(q, k, v, cu_seqlens, segments,
                                                    heads_per_segment, max_splits, scale_log2,
                                                    ws, out, lse, st);
    return launch_attention<__nv_bfloat16, __nv_bfloat16>(q, k, v, cu_seqlens, segments,
                                                          heads_per_segment, max_splits,
                                                          scale_log2, ws, out, lse, st);
  }
  return TW_ERR_UNSUPPORTED;
}

// ---- allocation-free variant ----------------------------------------------------
// Some callers cannot allocate device memory: a serving runtime that has
// reserved all device memory for its own arena, or a foreign-language host
// that is handed device buffers but has no CUDA allocator to call.  For them
// tw_decode_attention_noalloc keeps the split-K scratch (merge counters and
// per-split partials) in this fixed array.  Each GPU that loads the library
// holds its own copy until the process exits.  Host code must not pass the
// symbol itself to a kernel (on the host it is only a stand-in, not a device
// address); its device address comes from cudaGetSymbolAddress, looked up
// once per device on that device's first call.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TW_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::once_flag g_noalloc_once[kNoAllocMaxDevices];
void* g_noalloc_ptr[kNoAllocMaxDevices];
cudaError_t g_noalloc_err[kNoAllocMaxDevices];

// Device address of this device's scratch array (set up on first use).
int noalloc_scratch(void** ptr) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return TW_ERR_UNSUPPORTED;
  std::call_once(g_noalloc_once[dev], [dev]() {
    void* p = nullptr;
    g_noalloc_err[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_noalloc_ptr[dev] = p;
  });
  if (g_noalloc_err[dev] != cudaSuccess) {
    set_last_cuda_error(g_noalloc_err[dev]);
    return TW_ERR_CUDA;
  }
  *ptr = g_noalloc_ptr[dev];
  return TW_OK;
}
}  // namespace

extern "C" int tw_decode_attention_noalloc(const void* q, const void* k, const void* v,
                                           const int32_t* cu_seqlens, int segments,
                                           int heads_per_segment, int max_seqlen_k, int head_dim,
                                           int dtype, float softmax_scale, void* out,
                                           int out_dtype, float* lse, void* stream) {
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  if (!q || !k || !v || !cu_seqlens || !out || segments <= 0 || segments > 65535 ||
      heads_per_segment <= 0 || max_seqlen_k < 0 || !(softmax_scale > 0.0f))
    return TW_ERR_BAD_ARG;
  if (heads_per_segment > kMaxHeadsPerGroup) return TW_ERR_UNSUPPORTED;
  if (out_dtype != dtype && out_dtype != TW_F32) return TW_ERR_BAD_ARG;
  if (dtype != TW_F16 && dtype != TW_BF16) return TW_ERR_UNSUPPORTED;
  const int max_splits = attn_max_splits(max_seqlen_k);
  const size_t need = attn_ws_bytes(segments, heads_per_segment, max_splits, nullptr, nullptr);
  if (max_splits > 1 && need > (size_t)TW_NOALLOC_SCRATCH_BYTES) return TW_ERR_CAPACITY;
  cudaStream_t st = (cudaStream_t)stream;
  AttnWorkspace ws{};
  if (max_splits > 1) {
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != TW_OK) return rc;
    attn_ws_bytes(segments, heads_per_segment, max_splits, &ws, reinterpret_cast<char*>(scratch));
    // The array keeps the previous call's contents: the merge counters must
    // start at zero.
    cudaError_t err = cudaMemsetAsync(ws.counters, 0, (size_t)segments * sizeof(unsigned int), st);
    if (err != cudaSuccess) {
      set_last_cuda_error(err);
      return TW_ERR_CUDA;
    }
  }
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  if (dtype == TW_F16) {
    if (out_dtype == TW_F32)
      return launch_attention<__half, float>(q, k, v, cu_seqlens, segments, heads_per_segment,
                                             max_splits, scale_log2, ws, out, lse, st);
    return launch_attention<__half, __half>(q, k, v, cu_seqlens, segments, heads_per_segment,
                                            max_splits, scale_log2, ws, out, lse, st);
  }
  if (out_dtype == TW_F32)
    return launch_attention<__nv_bfloat16, float>(q, k, v, cu_seqlens, segments,
                                                  heads_per_segment, max_splits, scale_log2, ws,
                                                  out, lse, st);
  return launch_attention<__nv_bfloat16, __nv_bfloat16>(q, k, v, cu_seqlens, segments,
                                                        heads_per_segment, max_splits, scale_log2,
                                                        ws, out, lse, st);
}
