// Per-element arithmetic of the selection stage, shared by the per-stage
// kernels (quest.cu, int4.cu) and the fused whole-layer selection
// (topp_union.cu) so that both compute bit-identical scores and logits.
#pragma once

#include "tw_common.cuh"

namespace tw {

// Quest upper-bound score of page p for R query heads (warp-wide).  Lane l
// holds channels l, l+32, l+64, l+96; per head the products are added in that
// order (mul and add separately rounded), then reduced by shfl-down 1..16,
// the order of hi/twilight_fused_quest.py:13-46.  The result is valid in lane 0.
template <typename T, int R>
__device__ __forceinline__ void quest_page_score(const float (&qr)[R][4], const T* __restrict__ gmin,
                                                 const T* __restrict__ gmax, int64_t p, int lane,
                                                 float (&out)[R]) {
  float lo[4], hi[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    lo[c] = to_f32(gmin[p * kHeadDim + lane + 32 * c]);
    hi[c] = to_f32(gmax[p * kHeadDim + lane + 32 * c]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float e = qr[r][c] > 0.0f ? hi[c] : lo[c];
      acc = __fadd_rn(acc, __fmul_rn(e, qr[r][c]));
    }
#pragma unroll
    for (int off = 1; off < 32; off <<= 1)
      acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
    out[r] = acc;
  }
}

// quest_page_score with 8 threads per page.  Thread j (0..7) of the page's
// 8-thread group holds the partial sums of lanes l = 4j .. 4j+3 of the warp
// layout above (the same products added in the same order: channels l, l+32,
// l+64, l+96), then combines them in the same tree: the lane offsets 1 and 2
// inside the thread, the lane offsets 4, 8, 16 as group offsets 1, 2, 4.
// Bit-identical to quest_page_score, with 8-byte loads (4 channels) and a
// quarter of its shuffles.  q: the R query rows as fp32 [R][D] in shared
// memory.  valid = false: no loads, the result is unused.  The result is
// valid in thread j = 0; all 32 lanes of the warp must call this together.
template <typename T, int R>
__device__ __forceinline__ void quest_page_score8(const float* __restrict__ q,
                                                  const T* __restrict__ gmin,
                                                  const T* __restrict__ gmax, int64_t p, int j,
                                                  bool valid, float (&out)[R]) {
  float lo[4][4], hi[4][4];  // [c][i]: channel 32 c + 4 j + i
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint2 a = make_uint2(0u, 0u), b = make_uint2(0u, 0u);
    if (valid) {
      a = *reinterpret_cast<const uint2*>(gmin + p * kHeadDim + 32 * c + 4 * j);
      b = *reinterpret_cast<const uint2*>(gmax + p * kHeadDim + 32 * c + 4 * j);
    }
    const T* ta = reinterpret_cast<const T*>(&a);
    const T* tb = reinterpret_cast<const T*>(&b);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      lo[c][i] = to_f32(ta[i]);
      hi[c][i] = to_f32(tb[i]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float part[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float4 qv = *reinterpret_cast<const float4*>(q + r * kHeadDim + 32 * c + 4 * j);
      const float qq[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        part[i] = __fadd_rn(part[i], __fmul_rn(qq[i] > 0.0f ? hi[c][i] : lo[c][i], qq[i]));
    }
    float v = __fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3]));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 8));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 8));
    v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 8));
    out[r] = v;
  }
}

// quest_page_score for one head with 4 threads per page.  Thread j (0..3) of
// the page's 4-thread group holds the partial sums of lanes l = 8j .. 8j+7 of
// the warp layout above (the same products added in the same order: channels
// l, l+32, l+64, l+96), combines them as the tree's lane offsets 1, 2 and 4
// inside the thread, then the lane offsets 8 and 16 as group offsets 1 and 2.
// Bit-identical to quest_page_score, with 16-byte loads (8 channels).  q: the
// query row as fp32 [D] in shared memory.  valid = false: no loads, the
// result is unused.  The result is valid in thread j = 0; all 32 lanes of the
// warp must call this together (the groups are 4 consecutive lanes).
template <typename T>
__device__ __forceinline__ float quest_page_score4(const float* __restrict__ q,
                                                   const T* __restrict__ gmin,
                                                   const T* __restrict__ gmax, int64_t p, int j,
                                                   bool valid) {
  uint4 lo[4], hi[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    lo[c] = make_uint4(0u, 0u, 0u, 0u);
    hi[c] = lo[c];
    if (valid) {
      lo[c] = *reinterpret_cast<const uint4*>(gmin + p * kHeadDim + 32 * c + 8 * j);
      hi[c] = *reinterpret_cast<const uint4*>(gmax + p * kHeadDim + 32 * c + 8 * j);
    }
  }
  float part[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) part[i] = 0.0f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const T* tl = reinterpret_cast<const T*>(&lo[c]);
    const T* th = reinterpret_cast<const T*>(&hi[c]);
    const float4 q0 = *reinterpret_cast<const float4*>(q + 32 * c + 8 * j);
    const float4 q1 = *reinterpret_cast<const float4*>(q + 32 * c + 8 * j + 4);
    const float qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int i = 0; i < 8; ++i)
      part[i] = __fadd_rn(part[i], __fmul_rn(qq[i] > 0.0f ? to_f32(th[i]) : to_f32(tl[i]), qq[i]));
  }
  float v = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), __fadd_rn(part[2], part[3])),
                      __fadd_rn(__fadd_rn(part[4], part[5]), __fadd_rn(part[6], part[7])));
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 1, 4));
  v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 4));
  return v;
}

// INT4 estimate of 32 channels of one candidate (lane j of a 4-lane group
// covers channels 32j .. 32j+31, one uint4 of 16 code bytes): per channel
// k = code * s + m, the value of the reference's separately rounded mul and
// add (code * s is exact in fp32: a 4-bit integer times a value of at most 11
// significant bits, so one rounding of code * s + m equals the two), then
// acc[c % 4] = fma(k, q, acc[c % 4]) over the lane's channels c = 0..31 in
// order (fused multiply-adds, as torch.matmul's fp32 GEMV of
// hi/twilight_offload_cache.py:1257 accumulates on CUDA), and the lane's sum is
// (acc0 + acc1) + (acc2 + acc3).  Four interleaved accumulators keep four
// independent FMA chains per lane.
//
// The dequantisation is one mixed-precision fused multiply-add per channel
// (sm_100: fma.rn.f32.f16 / .bf16, the 16-bit operands exact in fp32, one
// rounding).  Two codes become a pair of 16-bit values exactly: a byte permute
// writes 0x64 (fp16) or 0x43 (bf16) above each code, the value 1024 + v or
// 128 + v, and one packed subtraction of 1024 or 128 leaves v.  s is the scale
// in the K dtype, m the minimum widened to fp32.
template <typename T> __device__ __forceinline__ uint32_t code_pair(uint32_t bytes, uint32_t sel);
template <> __device__ __forceinline__ uint32_t code_pair<__half>(uint32_t bytes, uint32_t sel) {
  const uint32_t x = __byte_perm(bytes, 0x64646464u, sel);  // fp16 1024 + v
  __half2 h = *reinterpret_cast<const __half2*>(&x);
  h = __hsub2(h, __half2(__ushort_as_half(0x6400u), __ushort_as_half(0x6400u)));
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t code_pair<__nv_bfloat16>(uint32_t bytes, uint32_t sel) {
  const uint32_t x = __byte_perm(bytes, 0x43434343u, sel);  // bf16 128 + v
  __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&x);
  h = __hsub2(h, __nv_bfloat162(__ushort_as_bfloat16(0x4300u), __ushort_as_bfloat16(0x4300u)));
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <typename T> __device__ __forceinline__ float fma_mixed(uint16_t a, uint16_t b, float c);
template <> __device__ __forceinline__ float fma_mixed<__half>(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
template <> __device__ __forceinline__ float fma_mixed<__nv_bfloat16>(uint16_t a, uint16_t b, float c) {
  float d;
  asm("fma.rn.f32.bf16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
template <typename T> __device__ __forceinline__ uint16_t bits16(T x);
template <> __device__ __forceinline__ uint16_t bits16<__half>(__half x) { return __half_as_ushort(x); }
template <> __device__ __forceinline__ uint16_t bits16<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat16_as_ushort(x);
}

template <typename T>
__device__ __forceinline__ float int4_dot32(const uint4& codes, T s, float m,
                                                  const float (&qr)[32]) {
  const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
  const uint16_t sb = bits16<T>(s);
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t lo = words[w] & 0x0f0f0f0fu;         // byte b: channel 8w + 2b
    const uint32_t hi = (words[w] >> 4) & 0x0f0f0f0fu;  // byte b: channel 8w + 2b + 1
    // pairs: (8w, 8w+2), (8w+4, 8w+6), (8w+1, 8w+3), (8w+5, 8w+7)
    const uint32_t p0 = code_pair<T>(lo, 0x5140u), p1 = code_pair<T>(lo, 0x5342u);
    const uint32_t p2 = code_pair<T>(hi, 0x5140u), p3 = code_pair<T>(hi, 0x5342u);
    const int i = 8 * w;
    acc[0] = __fmaf_rn(fma_mixed<T>((uint16_t)p0, sb, m), qr[i + 0], acc[0]);
    acc[1] = __fmaf_rn(fma_mixed<T>((uint16_t)p2, sb, m), qr[i + 1], acc[1]);
    acc[2] = __fmaf_rn(fma_mixed<T>((uint16_t)(p0 >> 16), sb, m), qr[i + 2], acc[2]);
    acc[3] = __fmaf_rn(fma_mixed<T>((uint16_t)(p2 >> 16), sb, m), qr[i + 3], acc[3]);
    acc[0] = __fmaf_rn(fma_mixed<T>((uint16_t)p1, sb, m), qr[i + 4], acc[0]);
    acc[1] = __fmaf_rn(fma_mixed<T>((uint16_t)p3, sb, m), qr[i + 5], acc[1]);
    acc[2] = __fmaf_rn(fma_mixed<T>((uint16_t)(p1 >> 16), sb, m), qr[i + 6], acc[2]);
    acc[3] = __fmaf_rn(fma_mixed<T>((uint16_t)(p3 >> 16), sb, m), qr[i + 7], acc[3]);
  }
  return __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
}

// int4_dot32 with the lane's 32 query channels read from shared memory
// (q: 16-byte aligned) instead of registers; the same operations in the same
// order, so the same result bit for bit.
template <typename T>
__device__ __forceinline__ float int4_dot32_s(const uint4& codes, T s, float m,
                                              const float* __restrict__ q) {
  const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
  const uint16_t sb = bits16<T>(s);
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const float4 qa = *reinterpret_cast<const float4*>(q + 8 * w);
    const float4 qb = *reinterpret_cast<const float4*>(q + 8 * w + 4);
    const uint32_t lo = words[w] & 0x0f0f0f0fu;
    const uint32_t hi = (words[w] >> 4) & 0x0f0f0f0fu;
    const uint32_t p0 = code_pair<T>(lo, 0x5140u), p1 = code_pair<T>(lo, 0x5342u);
    const uint32_t p2 = code_pair<T>(hi, 0x5140u), p3 = code_pair<T>(hi, 0x5342u);
    acc[0] = __fmaf_rn(fma_mixed<T>((uint16_t)p0, sb, m), qa.x, acc[0]);
    acc[1] = __fmaf_rn(fma_mixed<T>((uint16_t)p2, sb, m), qa.y, acc[1]);
    acc[2] = __fmaf_rn(fma_mixed<T>((uint16_t)(p0 >> 16), sb, m), qa.z, acc[2]);
    acc[3] = __fmaf_rn(fma_mixed<T>((uint16_t)(p2 >> 16), sb, m), qa.w, acc[3]);
    acc[0] = __fmaf_rn(fma_mixed<T>((uint16_t)p1, sb, m), qb.x, acc[0]);
    acc[1] = __fmaf_rn(fma_mixed<T>((uint16_t)p3, sb, m), qb.y, acc[1]);
    acc[2] = __fmaf_rn(fma_mixed<T>((uint16_t)(p1 >> 16), sb, m), qb.z, acc[2]);
    acc[3] = __fmaf_rn(fma_mixed<T>((uint16_t)(p3 >> 16), sb, m), qb.w, acc[3]);
  }
  return __fadd_rn(__fadd_rn(acc[0], acc[1]), __fadd_rn(acc[2], acc[3]));
}

// Sum of the 4 lanes' partial dot products ((a0 + a1) + (a2 + a3), in lane
// 0 of the group) times 1/sqrt(D): the candidate's estimated logit.
__device__ __forceinline__ float int4_logit(float acc, float inv_sqrt_d) {
  acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
  acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 2));
  return __fmul_rn(acc, inv_sqrt_d);
}

// 1/sqrt(D) as torch on CUDA applies `logits /= math.sqrt(D)`: the double
// divisor is narrowed to fp32 and its fp32 reciprocal multiplies.
inline float inv_sqrt_head_dim(int head_dim) {
  const float d = (float)sqrt((double)head_dim);
  return 1.0f / d;
}

}  // namespace tw
