// Decode-layer front end: the q / k / v projections of one token (a GEMV per
// head, batch 1) and rotary position embedding, in one kernel, writing q as
// [n_q_heads][D] (= [G][R][D] for GQA groups) and k, v as [n_kv_heads][D]:
// the inputs of the sparse decode layer-step.
//
// Reference: LlamaAttention_fast_forward's layer-batched projection
// (hi/mp.py:90-237: grouped q/k/v projections, then apply_rotary_pos_emb on
// the concatenated query / key heads) and its CUDA-graph replay
// (hi/twilight_projection_graph.py:12-41).  The rotary step follows the
// Llama formula out = x * cos + rotate_half(x) * sin with
// rotate_half(x) = cat(-x[D/2:], x[:D/2]), each product and the sum rounded to
// the model dtype, as elementwise ops in that dtype compute them.
//
// Layout: one CTA per rotary channel pair (c, c + 64) of one head, so the
// rotation needs no exchange between CTAs.  The CTA's 8 warps split the
// hidden dimension: thread t reads 16-byte vectors t, t + 256, ... of both
// weight rows and of the hidden vector (all its loads issued before its
// arithmetic), accumulates in fp32, and the 8 warp sums are added in warp
// order through shared memory (a fixed order: the result does not depend on
// scheduling).  Thread 0 rounds both dot products to the model dtype, like the
// projection's output, and writes the rotated channels.  (n_q + 2 n_kv) * 64
// pairs make 3072 small CTAs for Llama-3-8B, several resident per SM, so the
// hardware balances them over the 148 SMs.  The kernel is bound by the weight
// bytes read from HBM ((n_q + 2 n_kv) * D * hidden * 2 bytes per token).
#include "tw_common.cuh"

namespace tw {

constexpr int kFrontThreads = 256;   // 8 warps per channel pair
constexpr int kFrontHalf = kHeadDim / 2;
constexpr int kFrontMaxHidden = 16384;
constexpr int kFrontBatch = 2;       // 16-byte vectors of each row in flight per thread

template <typename T>
__global__ void __launch_bounds__(kFrontThreads, 6)
qkv_rope_kernel(const T* __restrict__ hidden, const T* __restrict__ w_q,
                const T* __restrict__ w_k, const T* __restrict__ w_v, int hidden_size,
                int n_q, int n_kv, const T* __restrict__ cos, const T* __restrict__ sin,
                T* __restrict__ q_out, T* __restrict__ k_out, T* __restrict__ v_out) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float s_part[kFrontThreads / 32][2];
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int pair = blockIdx.x;
  const int head = pair / kFrontHalf;  // q heads, then k heads, then v heads
  const int c = pair % kFrontHalf;     // channels c and c + 64
  const T* w;
  T* dst;
  bool rotate;
  if (head < n_q) {
    w = w_q + (int64_t)head * kHeadDim * hidden_size;
    dst = q_out + (int64_t)head * kHeadDim;
    rotate = true;
  } else if (head < n_q + n_kv) {
    w = w_k + (int64_t)(head - n_q) * kHeadDim * hidden_size;
    dst = k_out + (int64_t)(head - n_q) * kHeadDim;
    rotate = true;
  } else {
    w = w_v + (int64_t)(head - n_q - n_kv) * kHeadDim * hidden_size;
    dst = v_out + (int64_t)(head - n_q - n_kv) * kHeadDim;
    rotate = false;
  }
  const int vecs = hidden_size / 8;  // 16-byte vectors per weight row
  const uint4* wa = reinterpret_cast<const uint4*>(w + (int64_t)c * hidden_size);
  const uint4* wb = reinterpret_cast<const uint4*>(w + (int64_t)(c + kFrontHalf) * hidden_size);
  const uint4* hv = reinterpret_cast<const uint4*>(hidden);
  float acc_a = 0.0f, acc_b = 0.0f;
  for (int base = tid; base < vecs; base += kFrontThreads * kFrontBatch) {
    uint4 ra[kFrontBatch], rb[kFrontBatch], rh[kFrontBatch];
#pragma unroll
    for (int u = 0; u < kFrontBatch; ++u) {
      const int i = base + kFrontThreads * u;
      const bool in = i < vecs;
      ra[u] = in ? __ldcs(wa + i) : make_uint4(0u, 0u, 0u, 0u);
      rb[u] = in ? __ldcs(wb + i) : make_uint4(0u, 0u, 0u, 0u);
      rh[u] = in ? __ldg(hv + i) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kFrontBatch; ++u) {
      float fa[8], fb[8], fh[8];
      unpack8<T>(ra[u], fa);
      unpack8<T>(rb[u], fb);
      unpack8<T>(rh[u], fh);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc_a = fmaf(fa[j], fh[j], acc_a);
        acc_b = fmaf(fb[j], fh[j], acc_b);
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    acc_a += __shfl_xor_sync(0xffffffffu, acc_a, off);
    acc_b += __shfl_xor_sync(0xffffffffu, acc_b, off);
  }
  if (lane == 0) {
    s_part[warp][0] = acc_a;
    s_part[warp][1] = acc_b;
  }
  __syncthreads();
  if (tid != 0) return;
  float sa = 0.0f, sb = 0.0f;
#pragma unroll
  for (int k = 0; k < kFrontThreads / 32; ++k) {
    sa += s_part[k][0];
    sb += s_part[k][1];
  }
  const T xa = from_f32<T>(sa);  // channel c
  const T xb = from_f32<T>(sb);  // channel c + 64
  if (!rotate) {
    dst[c] = xa;
    dst[c + kFrontHalf] = xb;
    return;
  }
  // rotate_half: channel c pairs with -x[c + 64], channel c + 64 with x[c]
  const float fa = to_f32(xa), fb = to_f32(xb);
  const int d1 = c + kFrontHalf;
  const float a1 = to_f32(from_f32<T>(__fmul_rn(fa, to_f32(cos[c]))));
  const float a2 = to_f32(from_f32<T>(__fmul_rn(-fb, to_f32(sin[c]))));
  const float b1 = to_f32(from_f32<T>(__fmul_rn(fb, to_f32(cos[d1]))));
  const float b2 = to_f32(from_f32<T>(__fmul_rn(fa, to_f32(sin[d1]))));
  dst[c] = from_f32<T>(__fadd_rn(a1, a2));
  dst[d1] = from_f32<T>(__fadd_rn(b1, b2));
}

}  // namespace tw

using namespace tw;

extern "C" int tw_qkv_rope(const void* hidden, const void* w_q, const void* w_k, const void* w_v,
                           int hidden_size, int n_q_heads, int n_kv_heads, int head_dim,
                           const void* cos, const void* sin, int dtype, void* q_out, void* k_out,
                           void* v_out, void* stream) {
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  if (dtype != TW_F16 && dtype != TW_BF16) return TW_ERR_UNSUPPORTED;
  if (!hidden || !w_q || !w_k || !w_v || !cos || !sin || !q_out || !k_out || !v_out ||
      n_q_heads <= 0 || n_kv_heads <= 0 || hidden_size <= 0 || hidden_size % 256 != 0 ||
      hidden_size > kFrontMaxHidden || (int64_t)(n_q_heads + 2 * n_kv_heads) * kFrontHalf > (1 << 30))
    return TW_ERR_BAD_ARG;
  if ((((uintptr_t)hidden | (uintptr_t)w_q | (uintptr_t)w_k | (uintptr_t)w_v) & 15) != 0)
    return TW_ERR_BAD_ARG;
  const int pairs = (n_q_heads + 2 * n_kv_heads) * kFrontHalf;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == TW_F16)
    return launch_pdl(qkv_rope_kernel<__half>, dim3(pairs), dim3(kFrontThreads), 0, st,
                      (const __half*)hidden, (const __half*)w_q, (const __half*)w_k,
                      (const __half*)w_v, hidden_size, n_q_heads, n_kv_heads,
                      (const __half*)cos, (const __half*)sin, (__half*)q_out, (__half*)k_out,
                      (__half*)v_out);
  return launch_pdl(qkv_rope_kernel<__nv_bfloat16>, dim3(pairs), dim3(kFrontThreads), 0, st,
                    (const __nv_bfloat16*)hidden, (const __nv_bfloat16*)w_q,
                    (const __nv_bfloat16*)w_k, (const __nv_bfloat16*)w_v, hidden_size, n_q_heads,
                    n_kv_heads, (const __nv_bfloat16*)cos, (const __nv_bfloat16*)sin,
                    (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out);
}
