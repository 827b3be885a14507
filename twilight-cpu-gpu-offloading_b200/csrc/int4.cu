// Twilight INT4 stage: group-wise affine INT4 quantiser and the INT4 QK estimate.
//
// Reference: affine_int4_pack / affine_int4_dequantize
// (hi/twilight_offload_cache.py:25-47), fused_affine_int4_qk
// (hi/twilight_fused_qk.py:13-55), logits /= sqrt(D) (hi/twilight_offload_cache.py:1261).
#include "append.cuh"
#include "select_math.cuh"

namespace tw {

// Warp per row.  keys rows: entry e, row t at keys + (e*key_entry_stride + t)*D.
template <typename T>
__global__ void int4_pack_kernel(const T* __restrict__ keys, int64_t key_entry_stride,
                                 int64_t n_tokens, int group_size, int scale_div,
                                 uint8_t* __restrict__ packed, T* __restrict__ scale,
                                 T* __restrict__ minimum, int64_t out_entry_stride,
                                 int64_t out_row_offset) {
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int64_t t = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5);
  const int e = blockIdx.y;
  if (t >= n_tokens) return;
  const T* row = keys + (e * key_entry_stride + t) * kHeadDim;
  T raw[4];
  const uint2 v = *reinterpret_cast<const uint2*>(row + 4 * lane);
  memcpy(raw, &v, sizeof(v));
  const int ngroups = kHeadDim / group_size;
  const int64_t orow = e * out_entry_stride + out_row_offset + t;
  const int grp = (4 * lane) / group_size;
  const uint16_t bytes = quantize_lane<T>(raw, group_size, scale_div, scale + orow * ngroups + grp,
                                          minimum + orow * ngroups + grp);
  reinterpret_cast<uint16_t*>(packed + orow * (kHeadDim / 2))[lane] = bytes;
}

// INT4 QK estimate.  4 lanes per candidate token, lane j covers channels
// 32j .. 32j+31 (16 code bytes, one uint4 load); the arithmetic is
// int4_dot32 (select_math.cuh), then (a0+a1)+(a2+a3) over the lanes.
template <typename T, typename QT>
__global__ void __launch_bounds__(256)
int4_qk_kernel(const QT* __restrict__ q, const uint8_t* __restrict__ packed,
               const T* __restrict__ scale, const T* __restrict__ minimum,
               int64_t entry_stride, const int32_t* __restrict__ pages, int R, int b0,
               int block, int sink, int group_size, float inv_sqrt_d,
               float* __restrict__ logits, int tokens_per_cta) {
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.y;  // g*R + r
  const int g = row / R;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  const int sub = lane & 3;
  const int tok = lane >> 2;
  const int n_cand = b0 * block;
  float qr[32];
  const QT* qrow = q + (int64_t)row * kHeadDim + 32 * sub;
#pragma unroll
  for (int i = 0; i < 32; ++i) qr[i] = to_f32(qrow[i]);
  const int ngroups = kHeadDim / group_size;
  const int grp = (32 * sub) / group_size;
  const int32_t* prow = pages + (int64_t)row * b0;
  const int64_t ebase = (int64_t)g * entry_stride;
  const int cta_begin = blockIdx.x * tokens_per_cta;
  const int cta_end = min(n_cand, cta_begin + tokens_per_cta);
  for (int base = cta_begin + warp * 8; base < cta_end; base += warps * 8) {
    const int n = base + tok;
    const bool valid = n < cta_end;
    float acc = 0.0f;
    if (valid) {
      const int page = prow[n / block];
      const int64_t pos = (int64_t)sink + (int64_t)page * block + (n % block);
      const int64_t tr = ebase + pos;
      const uint4 c = __ldg(reinterpret_cast<const uint4*>(packed + tr * (kHeadDim / 2)) + sub);
      acc = int4_dot32<T>(c, scale[tr * ngroups + grp], to_f32(minimum[tr * ngroups + grp]),
                       qr);
    }
    const float logit = int4_logit(acc, inv_sqrt_d);
    if (valid && sub == 0) logits[(int64_t)row * n_cand + n] = logit;
  }
}

// New-token append: one CTA (128 threads) per group (append_token_row).
template <typename T>
__global__ void append_token_kernel(AppendArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  append_token_row<T>(a, blockIdx.x, threadIdx.x);
}

bool valid_group_size(int gs) { return gs == 32 || gs == 64 || gs == 128; }

}  // namespace tw

using namespace tw;

int tw_int4_pack_mode(const void* keys, int64_t key_entry_stride, int n_entries, int64_t n_tokens,
                      int head_dim, int group_size, int dtype, uint8_t* packed, void* scale,
                      void* minimum, int64_t out_entry_stride, int64_t out_row_offset,
                      int scale_div, void* stream) {
  if (head_dim != kHeadDim || !valid_group_size(group_size)) return TW_ERR_UNSUPPORTED;
  if (!keys || !packed || !scale || !minimum || n_entries < 0 || n_tokens < 0 ||
      n_entries > 65535 || (scale_div != kScaleReciprocal && scale_div != kScaleDivide))
    return TW_ERR_BAD_ARG;
  if (n_entries == 0 || n_tokens == 0) return TW_OK;
  constexpr int kThreads = 256;
  const int64_t blocks = (n_tokens + (kThreads / 32) - 1) / (kThreads / 32);
  if (blocks > 0x7fffffff) return TW_ERR_BAD_ARG;
  dim3 grid((unsigned)blocks, n_entries);
  TW_DISPATCH_KV_DTYPE(dtype, T, {
    int4_pack_kernel<T><<<grid, kThreads, 0, (cudaStream_t)stream>>>(
        (const T*)keys, key_entry_stride, n_tokens, group_size, scale_div, packed, (T*)scale,
        (T*)minimum, out_entry_stride, out_row_offset);
    return check_launch();
  });
}

extern "C" int tw_int4_pack(const void* keys, int64_t key_entry_stride, int n_entries,
                            int64_t n_tokens, int head_dim, int group_size, int dtype,
                            uint8_t* packed, void* scale, void* minimum,
                            int64_t out_entry_stride, int64_t out_row_offset, void* stream) {
  return tw_int4_pack_mode(keys, key_entry_stride, n_entries, n_tokens, head_dim, group_size,
                           dtype, packed, scale, minimum, out_entry_stride, out_row_offset,
                           kScaleReciprocal, stream);
}

// Same as tw_int4_pack with an explicit rounding mode of the `/ 15` step:
// 0 = multiply by the fp32 reciprocal (torch on CUDA), 1 = IEEE divide (torch on CPU).
extern "C" int tw_int4_pack_ex(const void* keys, int64_t key_entry_stride, int n_entries,
                               int64_t n_tokens, int head_dim, int group_size, int dtype,
                               uint8_t* packed, void* scale, void* minimum,
                               int64_t out_entry_stride, int64_t out_row_offset, int scale_div,
                               void* stream) {
  return tw_int4_pack_mode(keys, key_entry_stride, n_entries, n_tokens, head_dim, group_size,
                           dtype, packed, scale, minimum, out_entry_stride, out_row_offset,
                           scale_div, stream);
}

// q in fp32 (q_dtype TW_F32) or in the K dtype (converted exactly on load).
int launch_int4_qk(const void* q, int q_dtype, const uint8_t* packed, const void* scale,
                   const void* minimum, int64_t entry_stride_tokens, const int32_t* pages,
                   int groups, int R, int b0_pages, int block_size, int sink, int group_size,
                   int dtype, float* logits, cudaStream_t stream) {
  const int n_cand = b0_pages * block_size;
  constexpr int kThreads = 256;
  constexpr int kTokensPerCta = 256;
  dim3 grid((n_cand + kTokensPerCta - 1) / kTokensPerCta, groups * R);
  const float inv = inv_sqrt_head_dim(kHeadDim);
  if (q_dtype != TW_F32 && q_dtype != dtype) return TW_ERR_BAD_ARG;
  TW_DISPATCH_KV_DTYPE(dtype, T, {
    if (q_dtype == TW_F32)
      return launch_pdl(int4_qk_kernel<T, float>, grid, dim3(kThreads), 0, stream,
                        (const float*)q, packed, (const T*)scale, (const T*)minimum,
                        entry_stride_tokens, pages, R, b0_pages, block_size, sink, group_size, inv,
                        logits, kTokensPerCta);
    return launch_pdl(int4_qk_kernel<T, T>, grid, dim3(kThreads), 0, stream, (const T*)q, packed,
                      (const T*)scale, (const T*)minimum, entry_stride_tokens, pages, R, b0_pages,
                      block_size, sink, group_size, inv, logits, kTokensPerCta);
  });
}

extern "C" int tw_int4_qk(const float* q, const uint8_t* packed, const void* scale,
                          const void* minimum, int64_t entry_stride_tokens, const int32_t* pages,
                          int groups, int heads_per_group, int b0_pages, int block_size,
                          int sink, int head_dim, int group_size, int dtype, float* logits,
                          void* stream) {
  if (head_dim != kHeadDim || !valid_group_size(group_size)) return TW_ERR_UNSUPPORTED;
  if (!q || !packed || !scale || !minimum || !pages || !logits || groups <= 0 ||
      heads_per_group <= 0 || b0_pages < 0 || block_size <= 0 || sink < 0 ||
      (int64_t)groups * heads_per_group > 65535)
    return TW_ERR_BAD_ARG;
  if (b0_pages == 0) return TW_OK;
  return launch_int4_qk(q, TW_F32, packed, scale, minimum, entry_stride_tokens, pages, groups,
                        heads_per_group, b0_pages, block_size, sink, group_size, dtype, logits,
                        (cudaStream_t)stream);
}

extern "C" int tw_append_token(void* slab_k, void* slab_v, const uint64_t* entry_dirs,
                               int64_t n_entries, int64_t max_len, int first_entry,
                               int groups, int64_t position, const void* cur_k, const void* cur_v,
                               int head_dim, int dtype, int sink, int block_size, void* page_min,
                               void* page_max, int64_t meta_entry_stride, uint8_t* packed,
                               void* scale, void* minimum, int group_size, void* stream) {
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  const int st = check_append_args(slab_k, slab_v, entry_dirs, n_entries, max_len, first_entry,
                                   groups, position, cur_k, cur_v, sink, block_size, page_min,
                                   page_max, packed, scale, minimum, group_size);
  if (st != TW_OK) return st;
  const AppendArgs a = make_append_args(slab_k, slab_v, entry_dirs, n_entries, max_len,
                                        first_entry, position, cur_k, cur_v, sink, block_size,
                                        page_min, page_max, meta_entry_stride, packed, scale,
                                        minimum, group_size);
  TW_DISPATCH_KV_DTYPE(dtype, T, {
    return launch_pdl(append_token_kernel<T>, dim3(groups), dim3(kHeadDim), 0,
                      (cudaStream_t)stream, a);
  });
}
