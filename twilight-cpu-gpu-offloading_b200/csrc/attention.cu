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

constexpr int kAttnThreads = 256;   // 8 warps
constexpr int kAttnChunk = 128;     // rows per split CTA (16 per warp)
constexpr int kVecPerRow = 16;      // 16-byte vectors per 128-dim fp16/bf16 row
constexpr int kMergeChunk = 128;    // splits whose weights the merge stages at once

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
  const size_t c_bytes = align256((size_t)S * sizeof(unsigned int));
  const size_t ml_bytes = align256((size_t)S * max_splits * R * 2 * sizeof(float));
  const size_t o_bytes = align256((size_t)S * max_splits * R * kHeadDim * sizeof(float));
  if (ws) {
    ws->counters = reinterpret_cast<unsigned int*>(base);
    ws->part_ml = reinterpret_cast<float*>(base + c_bytes);
    ws->part_o = reinterpret_cast<float*>(base + c_bytes + ml_bytes);
  }
  return c_bytes + ml_bytes + o_bytes;
}

// Rows already gathered into device memory: segment s = rows [cu[s], cu[s+1]).
struct FlatRows {
  const uint4* k;
  const uint4* v;
  const int32_t* cu;
  __device__ __forceinline__ void keep(int, int, int64_t, int, const uint4&, const uint4&) const {}
  __device__ __forceinline__ int length(int s) const { return cu[s + 1] - cu[s]; }
  __device__ __forceinline__ void count(int, int, int) const {}
  __device__ __forceinline__ bool locate(int s, int i, const uint4*& kp, const uint4*& vp,
                                         int64_t&, int&, int&) const {
    const int64_t r = (int64_t)cu[s] + i;
    kp = k + r * kVecPerRow;
    vp = v + r * kVecPerRow;
    return true;
  }
};

// Rows read in place from the (mapped host) slab, or per entry through an
// entry directory (row-0 addresses; resident entries point into device memory):
// segment g = the group's sorted union positions, then its current token.
struct UnionRows {
  const uint4* slab_k;
  const uint4* slab_v;
  const unsigned long long* dirs;  // [2][n_entries] or null
  int64_t n_entries;
  int64_t max_len;
  int first_entry;
  int64_t old_length;
  const int32_t* union_pos;
  int64_t pos_stride;
  const int32_t* union_count;
  const uint4* cur_k;
  const uint4* cur_v;
  int32_t* error_flag;
  // previous-token row reuse (row_map null: every row from the slab, none kept)
  unsigned long long* row_map;
  int64_t map_stride;
  unsigned prev_tag;
  unsigned next_tag;
  const uint4* prev_k;
  const uint4* prev_v;
  int64_t prev_rows;
  uint4* next_k;
  uint4* next_v;
  int64_t rows_stride;
  int32_t* row_counts;
  // protected rows staged by the selection launch (stage.stage_k null: none)
  ProtectedStage stage;
  // Adds this warp's hit / miss row counts to group s (lane 0 of the warp).
  __device__ __forceinline__ void count(int s, int hits, int misses) const {
    if (!row_counts) return;
    hits = __reduce_add_sync(0xffffffffu, hits);
    misses = __reduce_add_sync(0xffffffffu, misses);
    if ((threadIdx.x & 31) == 0 && (hits | misses)) {
      atomicAdd(&row_counts[2 * s], hits);
      atomicAdd(&row_counts[2 * s + 1], misses);
    }
  }
  __device__ __forceinline__ int length(int s) const { return union_count[s] + 1; }
  // Row i (position pos) of group s is kept for the next step: its vectors go
  // to next_k / next_v and lane 0 of the half-warp records it in the row map
  // (after the whole half-warp has read the entry in locate).
  __device__ __forceinline__ void keep(int s, int i, int64_t pos, int l16, const uint4& kv,
                                       const uint4& vv) const {
    if (!row_map || i >= rows_stride) return;
    const int64_t row = (int64_t)s * rows_stride + i;
    next_k[row * kVecPerRow + l16] = kv;
    next_v[row * kVecPerRow + l16] = vv;
    if (l16 == 0)
      row_map[(int64_t)s * map_stride + pos] =
          ((unsigned long long)next_tag << 32) | (unsigned long long)row;
  }
  // The previous step's row holding position pos of group s, or -1.  Lane 0
  // of the half-warp reads the entry and broadcasts it to the other 15.
  __device__ __forceinline__ int64_t previous_row(int s, int64_t pos) const {
    const unsigned half_mask = 0xffffu << (threadIdx.x & 16);
    unsigned long long e = 0;
    if ((threadIdx.x & 15) == 0) e = row_map[(int64_t)s * map_stride + pos];
    e = __shfl_sync(half_mask, e, 0, 16);
    const int64_t row = (int64_t)(e & 0xffffffffull);
    return (prev_tag != 0 && (unsigned)(e >> 32) == prev_tag && row < prev_rows) ? row : -1;
  }
  // hits / misses count the history rows (not the current token) read from the
  // previous rows / from the slab; only lane 0 of each half-warp counts.
  __device__ __forceinline__ bool locate(int s, int i, const uint4*& kp, const uint4*& vp,
                                         int64_t& pos, int& hits, int& misses) const {
    if (i >= union_count[s]) {
      kp = cur_k + (int64_t)s * kVecPerRow;
      vp = cur_v + (int64_t)s * kVecPerRow;
      pos = old_length;
      return true;
    }
    pos = union_pos[(int64_t)s * pos_stride + i];
    if (pos < 0 || pos >= old_length) {
      if (error_flag) atomicExch(error_flag, TW_ERR_INVALID_INDEX);
      return false;
    }
    if (stage.stage_k) {
      const int64_t j = stage_index(stage, pos);
      if (j >= 0) {
        kp = stage.stage_k + ((int64_t)s * stage.stage_rows + j) * kVecPerRow;
        vp = stage.stage_v + ((int64_t)s * stage.stage_rows + j) * kVecPerRow;
        misses += (threadIdx.x & 15) == 0;  // read over the host link by the staging
        return true;
      }
    }
    if (row_map) {
      const int64_t j = previous_row(s, pos);
      if (j >= 0) {
        kp = prev_k + j * kVecPerRow;
        vp = prev_v + j * kVecPerRow;
        hits += (threadIdx.x & 15) == 0;
        return true;
      }
    }
    misses += (threadIdx.x & 15) == 0;
    const int64_t e = (int64_t)first_entry + s;
    if (dirs) {
      kp = reinterpret_cast<const uint4*>(dirs[e]) + pos * kVecPerRow;
      vp = reinterpret_cast<const uint4*>(dirs[n_entries + e]) + pos * kVecPerRow;
    } else {
      kp = slab_k + (e * max_len + pos) * kVecPerRow;
      vp = slab_v + (e * max_len + pos) * kVecPerRow;
    }
    return true;
  }
};

template <typename OutT>
__device__ __forceinline__ void write_final(OutT* out, float* lse, int s, int r, int R, int d,
                                            float m, float l, float o) {
  const float inv = (l > 0.0f) ? 1.0f / l : 0.0f;
  out[((int64_t)s * R + r) * kHeadDim + d] = from_f32<OutT>(o * inv);
  if (lse && d == 0)
    lse[(int64_t)s * R + r] = (l > 0.0f) ? (m + log2f(l)) * CUDART_LN2_F : -CUDART_INF_F;
}

__device__ __forceinline__ float weight(float m, float M) {
  return (m == -CUDART_INF_F) ? 0.0f : exp2f(m - M);
}

// One split CTA: 8 warps x 16 rows.  A half-warp owns a row per step (16 lanes
// x 8 channels, one 16-byte load each of K and V); every lane keeps its 8
// channels of q and of the output accumulator for all R heads.  Scores of a
// block of rows are computed first (4-step shuffle reduction inside the
// half-warp), then one online-softmax update per block.  The 8 warps are
// combined in shared memory; with several splits the last split CTA of the
// segment merges all partials in parallel (threads over (head, float4 column,
// split subset)).
template <typename T, int R, typename OutT, typename Rows>
__global__ void __launch_bounds__(kAttnThreads)
attention_kernel(Rows rows, const T* __restrict__ q, float scale_log2, int max_splits,
                 AttnWorkspace ws, OutT* __restrict__ out, float* __restrict__ lse) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int kWarps = kAttnThreads / 32;
  constexpr int kRowsPerWarp = kAttnChunk / kWarps;
  constexpr int kRowsPerHalf = (R <= 4) ? 8 : 4;
  constexpr int kIters = kRowsPerWarp / (2 * kRowsPerHalf);
  __shared__ float s_m[kWarps][R];
  __shared__ float s_l[kWarps][R];
  __shared__ float s_o[kWarps][R][kHeadDim];
  __shared__ float s_M[R], s_L[R];
  __shared__ float s_wt[kMergeChunk][R];
  __shared__ bool s_last;

  const int s = blockIdx.y;
  const int split = blockIdx.x;
  // Rows beyond max_splits * kAttnChunk (a caller's max_seqlen_k below the real
  // segment length) are not read: the split count is clamped to the grid.
  const int seg_len = min(rows.length(s), max_splits * kAttnChunk);
  const int nsplit = (seg_len + kAttnChunk - 1) / kAttnChunk;
  if (split >= max(nsplit, 1)) return;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int half = lane >> 4;
  const int l16 = lane & 15;

  float qf[R][8];
#pragma unroll
  for (int r = 0; r < R; ++r)
    unpack8<T>(reinterpret_cast<const uint4*>(q + ((int64_t)s * R + r) * kHeadDim)[l16], qf[r]);

  float m[R], l[R], acc[R][8];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    m[r] = -CUDART_INF_F;
    l[r] = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] = 0.0f;
  }

  const int warp_row0 = split * kAttnChunk + warp * kRowsPerWarp;
  int n_hit = 0, n_miss = 0;
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    uint4 kr[kRowsPerHalf], vr[kRowsPerHalf];
    bool ok[kRowsPerHalf];
#pragma unroll
    for (int j = 0; j < kRowsPerHalf; ++j) {
      const int i = warp_row0 + it * 2 * kRowsPerHalf + 2 * j + half;
      ok[j] = false;
      kr[j] = make_uint4(0, 0, 0, 0);
      vr[j] = kr[j];
      const uint4 *kp, *vp;
      int64_t pos;
      if (i < seg_len && rows.locate(s, i, kp, vp, pos, n_hit, n_miss)) {
        kr[j] = __ldcs(kp + l16);
        vr[j] = __ldcs(vp + l16);
        ok[j] = true;
        rows.keep(s, i, pos, l16, kr[j], vr[j]);
      }
    }
    float sc[kRowsPerHalf][R];
#pragma unroll
    for (int j = 0; j < kRowsPerHalf; ++j) {
      float kf[8];
      unpack8<T>(kr[j], kf);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        float p = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) p = fmaf(qf[r][c], kf[c], p);
        p += __shfl_xor_sync(0xffffffffu, p, 8);
        p += __shfl_xor_sync(0xffffffffu, p, 4);
        p += __shfl_xor_sync(0xffffffffu, p, 2);
        p += __shfl_xor_sync(0xffffffffu, p, 1);
        sc[j][r] = ok[j] ? p * scale_log2 : -CUDART_INF_F;
      }
    }
    float mb[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      float x = m[r];
#pragma unroll
      for (int j = 0; j < kRowsPerHalf; ++j) x = fmaxf(x, sc[j][r]);
      mb[r] = x;
      const float corr = (x == -CUDART_INF_F) ? 1.0f : exp2f(m[r] - x);
      l[r] *= corr;
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[r][c] *= corr;
      m[r] = x;
    }
#pragma unroll
    for (int j = 0; j < kRowsPerHalf; ++j) {
      float vf[8];
      unpack8<T>(vr[j], vf);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float p = (mb[r] == -CUDART_INF_F) ? 0.0f : exp2f(sc[j][r] - mb[r]);
        l[r] += p;
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[r][c] = fmaf(p, vf[c], acc[r][c]);
      }
    }
  }

  rows.count(s, n_hit, n_miss);

  // Combine the two half-warps (they hold disjoint rows, same channels).
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float mo = __shfl_xor_sync(0xffffffffu, m[r], 16);
    const float lo = __shfl_xor_sync(0xffffffffu, l[r], 16);
    const float M = fmaxf(m[r], mo);
    const float wa = weight(m[r], M), wb = weight(mo, M);
    l[r] = l[r] * wa + lo * wb;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float ao = __shfl_xor_sync(0xffffffffu, acc[r][c], 16);
      acc[r][c] = acc[r][c] * wa + ao * wb;
    }
    m[r] = M;
    if (lane == 0) {
      s_m[warp][r] = m[r];
      s_l[warp][r] = l[r];
    }
    if (half == 0) {
#pragma unroll
      for (int c = 0; c < 8; ++c) s_o[warp][r][8 * l16 + c] = acc[r][c];
    }
  }
  __syncthreads();

  // Combine the warps; write the output (one split) or this split's partial.
  float* pml = ws.part_ml + ((int64_t)s * max_splits + split) * R * 2;
  float* po = ws.part_o + ((int64_t)s * max_splits + split) * R * kHeadDim;
  for (int idx = tid; idx < R * kHeadDim; idx += kAttnThreads) {
    const int r = idx / kHeadDim;
    const int d = idx % kHeadDim;
    float M = -CUDART_INF_F;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, s_m[w][r]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float f = weight(s_m[w][r], M);
      L += s_l[w][r] * f;
      O += s_o[w][r][d] * f;
    }
    if (nsplit <= 1) {
      write_final<OutT>(out, lse, s, r, R, d, M, L, O);
    } else {
      po[r * kHeadDim + d] = O;
      if (d == 0) {
        pml[2 * r] = M;
        pml[2 * r + 1] = L;
      }
    }
  }
  if (nsplit <= 1) return;

  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&ws.counters[s], 1u);
    s_last = (prev == (unsigned int)nsplit - 1u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Last split: per-head max and normaliser (warp per head), then the
  // weighted sum of the partial outputs.  A thread owns one float4 column
  // (head r, channels 4*d4..4*d4+3) and every kTpp-th split; the kTpp threads
  // of a column are adjacent lanes, summed by a shuffle tree at the end.
  const float* ml = ws.part_ml + (int64_t)s * max_splits * R * 2;
  const float* po_all = ws.part_o + (int64_t)s * max_splits * R * kHeadDim;
  constexpr int kPairs = R * (kHeadDim / 4);
  constexpr int kTpp = kAttnThreads / kPairs >= 8 ? 8
                       : kAttnThreads / kPairs >= 4 ? 4
                       : kAttnThreads / kPairs >= 2 ? 2 : 1;
  static_assert(kPairs <= kAttnThreads, "one float4 column per thread at most");
  static_assert(R <= kWarps, "one warp per head in the merge");
  const int pair = tid / kTpp;
  const int sub = tid % kTpp;
  const bool has_pair = pair < kPairs;
  const int pr = has_pair ? pair / (kHeadDim / 4) : 0;
  const int d4 = pair % (kHeadDim / 4);
  const int64_t jstride = (int64_t)R * kHeadDim / 4;
  float4 acc4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (nsplit <= kMergeChunk) {
    // One pass (every split's weight fits s_wt): each thread issues its first
    // kMergeAhead partial loads, then warp r reads head r's (m, l) pairs once
    // into registers for the max, the normaliser and the weights, while those
    // loads are in flight.  Same arithmetic and order as the chunked path.
    constexpr int kMergeAhead = 8;
    constexpr int kPerLane = kMergeChunk / 32;
    const float4* col = reinterpret_cast<const float4*>(po_all + (int64_t)pr * kHeadDim) + d4;
    float4 pre[kMergeAhead];
#pragma unroll
    for (int u = 0; u < kMergeAhead; ++u) {
      const int jj = sub + u * kTpp;
      pre[u] = (has_pair && jj < nsplit) ? __ldcg(col + jj * jstride) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    if (warp < R) {
      const int r = warp;
      float2 e[kPerLane];
#pragma unroll
      for (int k = 0; k < kPerLane; ++k) {
        const int j = lane + 32 * k;
        e[k] = j < nsplit ? __ldcg(reinterpret_cast<const float2*>(ml + ((int64_t)j * R + r) * 2))
                          : make_float2(-CUDART_INF_F, 0.0f);
      }
      float M = -CUDART_INF_F;
#pragma unroll
      for (int k = 0; k < kPerLane; ++k) M = fmaxf(M, e[k].x);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.0f;
#pragma unroll
      for (int k = 0; k < kPerLane; ++k) {
        const int j = lane + 32 * k;
        const float w = weight(e[k].x, M);
        if (j < nsplit) {
          L += e[k].y * w;
          s_wt[j][r] = w;
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      if (lane == 0) {
        s_M[r] = M;
        s_L[r] = L;
      }
    }
    __syncthreads();
    if (has_pair) {
#pragma unroll
      for (int u = 0; u < kMergeAhead; ++u) {
        const int jj = sub + u * kTpp;
        if (jj < nsplit) {
          const float w = s_wt[jj][pr];
          acc4.x = fmaf(w, pre[u].x, acc4.x);
          acc4.y = fmaf(w, pre[u].y, acc4.y);
          acc4.z = fmaf(w, pre[u].z, acc4.z);
          acc4.w = fmaf(w, pre[u].w, acc4.w);
        }
      }
#pragma unroll 8
      for (int jj = sub + kMergeAhead * kTpp; jj < nsplit; jj += kTpp) {
        const float w = s_wt[jj][pr];
        const float4 o = __ldcg(col + jj * jstride);
        acc4.x = fmaf(w, o.x, acc4.x);
        acc4.y = fmaf(w, o.y, acc4.y);
        acc4.z = fmaf(w, o.z, acc4.z);
        acc4.w = fmaf(w, o.w, acc4.w);
      }
    }
  } else {
    for (int r = warp; r < R; r += kWarps) {
      float M = -CUDART_INF_F;
      for (int j = lane; j < nsplit; j += 32) M = fmaxf(M, __ldcg(ml + ((int64_t)j * R + r) * 2));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
      float L = 0.0f;
      for (int j = lane; j < nsplit; j += 32) {
        const float* e = ml + ((int64_t)j * R + r) * 2;
        L += __ldcg(e + 1) * weight(__ldcg(e), M);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
      if (lane == 0) {
        s_M[r] = M;
        s_L[r] = L;
      }
    }
    __syncthreads();
    // Chunks of kMergeChunk splits: their weights are computed once into
    // shared memory; the unrolled loop keeps 8 partial loads in flight.
    for (int j0 = 0; j0 < nsplit; j0 += kMergeChunk) {
      const int n = min(kMergeChunk, nsplit - j0);
      for (int idx = tid; idx < n * R; idx += kAttnThreads) {
        const int jj = idx / R, rr = idx % R;
        s_wt[jj][rr] = weight(__ldcg(ml + ((int64_t)(j0 + jj) * R + rr) * 2), s_M[rr]);
      }
      __syncthreads();
      if (has_pair) {
        const float4* col = reinterpret_cast<const float4*>(po_all + ((int64_t)j0 * R + pr) * kHeadDim) + d4;
#pragma unroll 8
        for (int jj = sub; jj < n; jj += kTpp) {
          const float w = s_wt[jj][pr];
          const float4 o = __ldcg(col + jj * jstride);
          acc4.x = fmaf(w, o.x, acc4.x);
          acc4.y = fmaf(w, o.y, acc4.y);
          acc4.z = fmaf(w, o.z, acc4.z);
          acc4.w = fmaf(w, o.w, acc4.w);
        }
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int off = kTpp / 2; off > 0; off >>= 1) {
    acc4.x += __shfl_xor_sync(0xffffffffu, acc4.x, off);
    acc4.y += __shfl_xor_sync(0xffffffffu, acc4.y, off);
    acc4.z += __shfl_xor_sync(0xffffffffu, acc4.z, off);
    acc4.w += __shfl_xor_sync(0xffffffffu, acc4.w, off);
  }
  if (has_pair && sub == 0) {
    const float M = s_M[pr], L = s_L[pr];
    write_final<OutT>(out, lse, s, pr, R, 4 * d4 + 0, M, L, acc4.x);
    write_final<OutT>(out, lse, s, pr, R, 4 * d4 + 1, M, L, acc4.y);
    write_final<OutT>(out, lse, s, pr, R, 4 * d4 + 2, M, L, acc4.z);
    write_final<OutT>(out, lse, s, pr, R, 4 * d4 + 3, M, L, acc4.w);
  }
  if (tid == 0) ws.counters[s] = 0u;
}

template <typename T, typename OutT, typename Rows>
int launch_rows(const Rows& rows, const void* q, int S, int R, int max_splits, float scale_log2,
                const AttnWorkspace& ws, void* out, float* lse, cudaStream_t stream) {
  dim3 grid(max_splits, S);
#define TW_ATTN_CASE(RR)                                                                    \
  case RR:                                                                                  \
    return launch_pdl(attention_kernel<T, RR, OutT, Rows>, grid, dim3(kAttnThreads), 0,     \
                      stream, rows, (const T*)q, scale_log2, max_splits, ws, (OutT*)out, lse);
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

template <typename T, typename OutT>
int launch_attention(const void* q, const void* k, const void* v, const int32_t* cu, int S, int R,
                     int max_splits, float scale_log2, const AttnWorkspace& ws, void* out,
                     float* lse, cudaStream_t stream) {
  FlatRows rows{(const uint4*)k, (const uint4*)v, cu};
  return launch_rows<T, OutT>(rows, q, S, R, max_splits, scale_log2, ws, out, lse, stream);
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
  if (max_splits > 1 && ((uintptr_t)workspace & 15) != 0) return TW_ERR_BAD_ARG;  // float4 merge
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

namespace tw {

// tw_attend_union, with the protected rows read from a stage the selection
// launch filled (stage null: every row from its source).
int attend_union_impl(const void* slab_k, const void* slab_v, const uint64_t* entry_dirs,
                      int64_t n_entries, int64_t max_len, int first_entry, int groups,
                      int64_t old_length, const int32_t* union_pos, int64_t pos_stride,
                      const int32_t* union_count, const void* cur_k, const void* cur_v,
                      const void* q, int heads_per_group, int max_rows_per_group, int head_dim,
                      int dtype, float softmax_scale, void* out, int out_dtype, float* lse,
                      int32_t* error_flag, void* workspace, size_t workspace_bytes,
                      const tw_row_reuse* reuse, const ProtectedStage* stage,
                      cudaStream_t stream) {
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  if ((!entry_dirs && (!slab_k || !slab_v)) || !union_pos || !union_count || !cur_k || !cur_v ||
      !q || !out || groups <= 0 || groups > 65535 || heads_per_group <= 0 || first_entry < 0 ||
      (entry_dirs && first_entry + groups > n_entries) ||
      old_length < 0 || old_length > max_len || pos_stride < old_length ||
      max_rows_per_group < 1 || !(softmax_scale > 0.0f))
    return TW_ERR_BAD_ARG;
  if (heads_per_group > kMaxHeadsPerGroup) return TW_ERR_UNSUPPORTED;
  if (dtype != TW_F16 && dtype != TW_BF16) return TW_ERR_UNSUPPORTED;
  if (out_dtype != dtype && out_dtype != TW_F32) return TW_ERR_BAD_ARG;
  if ((((uintptr_t)slab_k | (uintptr_t)slab_v | (uintptr_t)cur_k | (uintptr_t)cur_v |
        (uintptr_t)q) & 15) != 0)
    return TW_ERR_BAD_ARG;
  const int max_splits = attn_max_splits(max_rows_per_group);
  AttnWorkspace ws{};
  const size_t need = attn_ws_bytes(groups, heads_per_group, max_splits, &ws,
                                    reinterpret_cast<char*>(workspace));
  if (max_splits > 1 && (!workspace || workspace_bytes < need)) return TW_ERR_CAPACITY;
  if (max_splits > 1 && ((uintptr_t)workspace & 15) != 0) return TW_ERR_BAD_ARG;  // float4 merge
  UnionRows rows{(const uint4*)slab_k, (const uint4*)slab_v,
                 (const unsigned long long*)entry_dirs, n_entries, max_len, first_entry,
                 old_length, union_pos, pos_stride, union_count, (const uint4*)cur_k,
                 (const uint4*)cur_v, error_flag,
                 nullptr, 0, 0u, 0u, nullptr, nullptr, 0, nullptr, nullptr, 0, nullptr};
  if (reuse) {
    const size_t next_bytes = (size_t)groups * reuse->rows_stride * kHeadDim * 2;
    const size_t prev_bytes = (size_t)reuse->prev_rows * kHeadDim * 2;
    auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
      const char* x = (const char*)a;
      const char* y = (const char*)b;
      return x < y + nb && y < x + na;
    };
    if (!reuse->row_map || reuse->map_stride <= old_length || !reuse->next_k || !reuse->next_v ||
        reuse->rows_stride < max_rows_per_group || reuse->next_tag == 0 ||
        reuse->next_tag == reuse->prev_tag ||
        (((uintptr_t)reuse->next_k | (uintptr_t)reuse->next_v) & 15) != 0 ||
        overlap(reuse->next_k, next_bytes, reuse->next_v, next_bytes))
      return TW_ERR_BAD_ARG;
    if (reuse->prev_tag != 0 &&
        (!reuse->prev_k || !reuse->prev_v || reuse->prev_rows <= 0 ||
         (((uintptr_t)reuse->prev_k | (uintptr_t)reuse->prev_v) & 15) != 0 ||
         overlap(reuse->prev_k, prev_bytes, reuse->next_k, next_bytes) ||
         overlap(reuse->prev_k, prev_bytes, reuse->next_v, next_bytes) ||
         overlap(reuse->prev_v, prev_bytes, reuse->next_k, next_bytes) ||
         overlap(reuse->prev_v, prev_bytes, reuse->next_v, next_bytes)))
      return TW_ERR_BAD_ARG;
    rows.row_map = (unsigned long long*)reuse->row_map;
    rows.map_stride = reuse->map_stride;
    rows.prev_tag = reuse->prev_tag;
    rows.next_tag = reuse->next_tag;
    rows.prev_k = (const uint4*)reuse->prev_k;
    rows.prev_v = (const uint4*)reuse->prev_v;
    rows.prev_rows = reuse->prev_tag != 0 ? reuse->prev_rows : 0;
    rows.next_k = (uint4*)reuse->next_k;
    rows.next_v = (uint4*)reuse->next_v;
    rows.rows_stride = reuse->rows_stride;
    rows.row_counts = reuse->row_counts;
  }
  if (stage && stage->stage_k) {
    if (!stage->stage_v || stage->old_length != old_length ||
        stage->stage_rows < stage->n_sink + (old_length - stage->recent_start) ||
        (((uintptr_t)stage->stage_k | (uintptr_t)stage->stage_v) & 15) != 0)
      return TW_ERR_BAD_ARG;
    rows.stage = *stage;
  }
  const float scale_log2 = softmax_scale * 1.4426950408889634f;
  cudaStream_t st = stream;
  if (dtype == TW_F16) {
    if (out_dtype == TW_F32)
      return launch_rows<__half, float>(rows, q, groups, heads_per_group, max_splits, scale_log2,
                                        ws, out, lse, st);
    return launch_rows<__half, __half>(rows, q, groups, heads_per_group, max_splits, scale_log2,
                                       ws, out, lse, st);
  }
  if (out_dtype == TW_F32)
    return launch_rows<__nv_bfloat16, float>(rows, q, groups, heads_per_group, max_splits,
                                             scale_log2, ws, out, lse, st);
  return launch_rows<__nv_bfloat16, __nv_bfloat16>(rows, q, groups, heads_per_group, max_splits,
                                                   scale_log2, ws, out, lse, st);
}

}  // namespace tw

extern "C" int tw_attend_union(const void* slab_k, const void* slab_v,
                               const uint64_t* entry_dirs, int64_t n_entries, int64_t max_len,
                               int first_entry, int groups, int64_t old_length,
                               const int32_t* union_pos, int64_t pos_stride,
                               const int32_t* union_count, const void* cur_k, const void* cur_v,
                               const void* q, int heads_per_group, int max_rows_per_group,
                               int head_dim, int dtype, float softmax_scale, void* out,
                               int out_dtype, float* lse, int32_t* error_flag, void* workspace,
                               size_t workspace_bytes, const tw_row_reuse* reuse, void* stream) {
  return attend_union_impl(slab_k, slab_v, entry_dirs, n_entries, max_len, first_entry, groups,
                           old_length, union_pos, pos_stride, union_count, cur_k, cur_v, q,
                           heads_per_group, max_rows_per_group, head_dim, dtype, softmax_scale,
                           out, out_dtype, lse, error_flag, workspace, workspace_bytes, reuse,
                           nullptr, (cudaStream_t)stream);
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
constexpr int kNoAllocMaxDevices = 64;  // device ordinals 0..63 (TW_ERR_UNSUPPORTED beyond)
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kNoAllocMaxDevices];  // null until a lookup on that device succeeds

// Device address of this device's scratch array.  Only a successful lookup
// is kept: a failed one (e.g. a first call made during stream capture)
// returns TW_ERR_CUDA and the next call tries again.
int noalloc_scratch(void** ptr) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  if (dev < 0 || dev >= kNoAllocMaxDevices) return TW_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || !p) {
      set_last_cuda_error(err != cudaSuccess ? err : cudaErrorInvalidSymbol);
      return TW_ERR_CUDA;
    }
    g_noalloc_ptr[dev] = p;
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
