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

// quest_page_score for two pages at once (both pages' loads issued first).
template <typename T, int R>
__device__ __forceinline__ void quest_page_score2(const float (&qr)[R][4], const T* __restrict__ gmin,
                                                  const T* __restrict__ gmax, int64_t p, int64_t p2,
                                                  int lane, float (&out)[R], float (&out2)[R]) {
  float lo[4], hi[4], lo2[4], hi2[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    lo[c] = to_f32(gmin[p * kHeadDim + lane + 32 * c]);
    hi[c] = to_f32(gmax[p * kHeadDim + lane + 32 * c]);
    lo2[c] = to_f32(gmin[p2 * kHeadDim + lane + 32 * c]);
    hi2[c] = to_f32(gmax[p2 * kHeadDim + lane + 32 * c]);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float acc = 0.0f, acc2 = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      acc = __fadd_rn(acc, __fmul_rn(qr[r][c] > 0.0f ? hi[c] : lo[c], qr[r][c]));
      acc2 = __fadd_rn(acc2, __fmul_rn(qr[r][c] > 0.0f ? hi2[c] : lo2[c], qr[r][c]));
    }
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
      acc2 = __fadd_rn(acc2, __shfl_down_sync(0xffffffffu, acc2, off));
    }
    out[r] = acc;
    out2[r] = acc2;
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

// INT4 estimate of 32 channels of one candidate (lane j of a 4-lane group
// covers channels 32j .. 32j+31, one uint4 of 16 code bytes): per channel
// k = code * s + m (the values of separately rounded mul and add, as the
// reference dequantises), then acc[c % 4] = fma(k, q, acc[c % 4]) over the
// lane's channels c = 0..31 in order (fused multiply-adds, as torch.matmul's
// fp32 GEMV of hi/twilight_offload_cache.py:1257 accumulates on CUDA), and the
// lane's sum is (acc0 + acc1) + (acc2 + acc3).  Four interleaved accumulators
// keep four independent FMA chains per lane.  s and m are fp16 / bf16 values.
// A code v in 0..15 as float, exactly: the bits 0x4B0000vv are the float
// 2^23 + v, from which 2^23 is subtracted (exact).  One byte permute puts
// byte b of `nibbles` (one code per byte) under the exponent 0x4B.
__device__ __forceinline__ float nibble_float(uint32_t nibbles, int b) {
  return __fsub_rn(__int_as_float(__byte_perm(nibbles, 0x4B000000u, 0x7440u | (uint32_t)b)),
                   8388608.0f);
}

__device__ __forceinline__ float int4_dot32(const uint4& codes, float s, float m,
                                            const float (&qr)[32]) {
  const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const uint32_t lo = words[w] & 0x0f0f0f0fu;         // even channels, one per byte
    const uint32_t hi = (words[w] >> 4) & 0x0f0f0f0fu;  // odd channels
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = 8 * w + 2 * b;  // channels i (even) and i + 1 (odd)
      // code * s is exact in fp32 (a 4-bit integer times a value of at most
      // 11 significant bits), so the fused multiply-add rounds exactly as the
      // separately rounded code * s + m does.
      const float k0 = __fmaf_rn(nibble_float(lo, b), s, m);
      acc[i & 3] = __fmaf_rn(k0, qr[i], acc[i & 3]);
      const float k1 = __fmaf_rn(nibble_float(hi, b), s, m);
      acc[(i + 1) & 3] = __fmaf_rn(k1, qr[i + 1], acc[(i + 1) & 3]);
    }
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
