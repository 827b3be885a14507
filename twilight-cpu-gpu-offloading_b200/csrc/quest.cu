// Quest stage: page min/max metadata, upper-bound page scores, top-k pages.
//
// Reference: hi/quest_offload_cache.py:276-289 (metadata),
// hi/twilight_fused_quest.py:13-46 (score and its summation order),
// hi/twilight_offload_cache.py:1136-1166 (top-k + B0 expansion).
#include "select_math.cuh"

namespace tw {

// One CTA per (page, entry); thread d reduces the block_size rows of channel d.
// min/max are exact in the K dtype; the first occurrence wins on equal values.
template <typename T>
__global__ void quest_page_meta_kernel(const T* __restrict__ keys, int64_t key_entry_stride,
                                       int sink, int block, int first_page,
                                       T* __restrict__ pmin, T* __restrict__ pmax,
                                       int64_t meta_entry_stride) {
  const int page = first_page + blockIdx.x;
  const int entry = blockIdx.y;
  const int d = threadIdx.x;  // blockDim.x == kHeadDim
  const T* base = keys + entry * key_entry_stride + ((int64_t)sink + (int64_t)page * block) * kHeadDim + d;
  T vmin = base[0];
  T vmax = vmin;
  float fmin = to_f32(vmin), fmax = fmin;
  for (int t = 1; t < block; ++t) {
    T x = base[(int64_t)t * kHeadDim];
    float fx = to_f32(x);
    if (fx < fmin) { fmin = fx; vmin = x; }
    if (fx > fmax) { fmax = fx; vmax = x; }
  }
  const int64_t out = entry * meta_entry_stride + (int64_t)page * kHeadDim + d;
  pmin[out] = vmin;
  pmax[out] = vmax;
}

// Warp per page, all R query heads of the group share each min/max load.
// Lane l holds channels l, l+32, l+64, l+96; per head the products are added in
// that order (mul and add separately rounded), then reduced by shfl-down 1..16.
template <typename T, int R, typename QT>
__global__ void quest_score_kernel(const QT* __restrict__ q, const T* __restrict__ pmin,
                                   const T* __restrict__ pmax, int n_pages,
                                   int64_t meta_group_stride, float* __restrict__ scores) {
  pdl_wait();
  pdl_launch_dependents();
  const int g = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  float qr[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int c = 0; c < 4; ++c) qr[r][c] = to_f32(q[((int64_t)g * R + r) * kHeadDim + lane + 32 * c]);

  const T* gmin = pmin + g * meta_group_stride;
  const T* gmax = pmax + g * meta_group_stride;
  for (int p = blockIdx.x * warps + warp; p < n_pages; p += gridDim.x * warps) {
    float sc[R];
    quest_page_score<T, R>(qr, gmin, gmax, p, lane, sc);
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) scores[((int64_t)g * R + r) * n_pages + p] = sc[r];
    }
  }
}

// Radix select of the k largest of n scores per row (one CTA per row).
// 4 passes of 8-bit digits over order-preserving keys held in shared memory
// find the k-th largest key; the output is every page above it plus the
// lowest-index pages equal to it, in ascending page order.
constexpr int kTopkThreads = 512;

__global__ void __launch_bounds__(kTopkThreads)
topk_pages_kernel(const float* __restrict__ scores, int n, int k, int32_t* __restrict__ out) {
  pdl_wait();
  pdl_launch_dependents();
  extern __shared__ uint32_t keys[];  // n keys
  __shared__ uint32_t hist[256];
  __shared__ uint32_t scan_scratch[32];
  __shared__ uint32_t s_prefix, s_remaining;
  const int row = blockIdx.x;
  const float* src = scores + (int64_t)row * n;
  for (int i = threadIdx.x; i < n; i += blockDim.x) keys[i] = float_key(src[i]);
  if (threadIdx.x == 0) {
    s_prefix = 0u;
    s_remaining = (uint32_t)k;
  }
  __syncthreads();

  uint32_t mask = 0u;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0u;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t key = keys[i];
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l owns bins 8l .. 8l+7; suffix sums from the top bin down.
      const int lane = threadIdx.x;
      uint32_t local[8];
      uint32_t sum = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        local[j] = hist[8 * lane + j];
        sum += local[j];
      }
      // inclusive suffix over lanes (lane 31 = highest bins)
      uint32_t suffix = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        uint32_t y = __shfl_down_sync(0xffffffffu, suffix, off);
        if (lane + off < 32) suffix += y;
      }
      const uint32_t above = suffix - sum;  // count in bins of higher lanes
      const uint32_t need = s_remaining;
      __syncwarp();
      // the crossing lane: above < need <= suffix
      if (above < need && need <= suffix) {
        uint32_t acc = above;
        for (int j = 7; j >= 0; --j) {
          if (acc + local[j] >= need) {
            s_prefix = prefix | ((uint32_t)(8 * lane + j) << shift);
            s_remaining = need - acc;
            break;
          }
          acc += local[j];
        }
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t kth = s_prefix;       // k-th largest key
  const uint32_t ties = s_remaining;   // how many elements equal to kth to keep

  // Contiguous segment per thread; two block scans give tie ranks and output slots.
  const int seg = (n + blockDim.x - 1) / blockDim.x;
  const int beg = min(n, (int)threadIdx.x * seg);
  const int end = min(n, beg + seg);
  uint32_t gt = 0u, eq = 0u;
  for (int i = beg; i < end; ++i) {
    const uint32_t key = keys[i];
    gt += key > kth;
    eq += key == kth;
  }
  uint32_t total;
  const uint32_t eq_before = block_exclusive_scan(eq, scan_scratch, &total);
  const uint32_t take_eq = (eq_before >= ties) ? 0u : min(eq, ties - eq_before);
  const uint32_t base = block_exclusive_scan(gt + take_eq, scan_scratch, &total);
  int32_t* dst = out + (int64_t)row * k;
  uint32_t slot = base, eq_seen = 0u;
  for (int i = beg; i < end; ++i) {
    const uint32_t key = keys[i];
    bool take = key > kth;
    if (key == kth) {
      take = eq_seen < take_eq;
      ++eq_seen;
    }
    if (take) dst[slot++] = i;
  }
}

template <typename T>
int launch_quest_meta(const void* keys, int64_t key_entry_stride, int n_entries, int sink,
                      int block, int first_page, int n_pages, void* pmin, void* pmax,
                      int64_t meta_entry_stride, cudaStream_t stream) {
  dim3 grid(n_pages, n_entries);
  quest_page_meta_kernel<T><<<grid, kHeadDim, 0, stream>>>(
      (const T*)keys, key_entry_stride, sink, block, first_page, (T*)pmin, (T*)pmax,
      meta_entry_stride);
  return check_launch();
}

template <typename T, int R, typename QT>
int launch_quest_score_r(const void* q, const void* pmin, const void* pmax, int groups,
                         int n_pages, int64_t stride, float* scores, cudaStream_t stream) {
  constexpr int kThreads = 256;
  const int warps = kThreads / 32;
  int blocks_x = (n_pages + warps - 1) / warps;
  dim3 grid(blocks_x, groups);
  return launch_pdl(quest_score_kernel<T, R, QT>, grid, dim3(kThreads), 0, stream,
                    (const QT*)q, (const T*)pmin, (const T*)pmax, n_pages, stride, scores);
}

template <typename T, typename QT>
int launch_quest_score(const void* q, const void* pmin, const void* pmax, int groups, int R,
                       int n_pages, int64_t stride, float* scores, cudaStream_t stream) {
#define TW_QS_CASE(RR) \
  case RR: return launch_quest_score_r<T, RR, QT>(q, pmin, pmax, groups, n_pages, stride, scores, stream);
  switch (R) {
    TW_QS_CASE(1) TW_QS_CASE(2) TW_QS_CASE(3) TW_QS_CASE(4)
    TW_QS_CASE(5) TW_QS_CASE(6) TW_QS_CASE(7) TW_QS_CASE(8)
    default: return TW_ERR_UNSUPPORTED;
  }
#undef TW_QS_CASE
}

// q in fp32 (q_dtype TW_F32) or in the K dtype (converted exactly on load).
int quest_score_dispatch(const void* q, int q_dtype, const void* pmin, const void* pmax, int groups,
                         int R, int n_pages, int64_t stride, int dtype, float* scores,
                         cudaStream_t stream) {
  if (q_dtype == TW_F32) {
    TW_DISPATCH_KV_DTYPE(dtype, T,
                         return launch_quest_score<T, float>(q, pmin, pmax, groups, R, n_pages,
                                                             stride, scores, stream));
  }
  if (q_dtype != dtype) return TW_ERR_BAD_ARG;
  TW_DISPATCH_KV_DTYPE(dtype, T,
                       return launch_quest_score<T, T>(q, pmin, pmax, groups, R, n_pages, stride,
                                                       scores, stream));
}

constexpr int kTopkMaxN = 16384;

int launch_topk_pages(const float* scores, int rows, int n, int k, int32_t* out,
                      cudaStream_t stream) {
  const size_t smem = (size_t)n * sizeof(uint32_t);
  static DynSmemOptIn opt_in;
  const int st = ensure_dyn_smem((const void*)topk_pages_kernel, opt_in,
                                 kTopkMaxN * (int)sizeof(uint32_t));
  if (st != TW_OK) return st;
  return launch_pdl(topk_pages_kernel, dim3(rows), dim3(kTopkThreads), smem, stream, scores, n, k,
                    out);
}

}  // namespace tw

using namespace tw;

extern "C" int tw_quest_page_metadata(const void* keys, int64_t key_entry_stride, int n_entries,
                                      int sink, int block_size, int head_dim, int dtype,
                                      int first_page, int n_pages, void* page_min,
                                      void* page_max, int64_t meta_entry_stride, void* stream) {
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  if (!keys || !page_min || !page_max || n_entries < 0 || sink < 0 || block_size <= 0 ||
      first_page < 0 || n_pages < 0)
    return TW_ERR_BAD_ARG;
  if (n_pages == 0 || n_entries == 0) return TW_OK;
  if (n_entries > 65535) return TW_ERR_BAD_ARG;
  TW_DISPATCH_KV_DTYPE(dtype, T,
                       return launch_quest_meta<T>(keys, key_entry_stride, n_entries, sink,
                                                   block_size, first_page, n_pages, page_min,
                                                   page_max, meta_entry_stride,
                                                   (cudaStream_t)stream));
}

extern "C" int tw_quest_score(const float* q, const void* page_min, const void* page_max,
                              int groups, int heads_per_group, int n_pages,
                              int64_t meta_group_stride, int head_dim, int dtype, float* scores,
                              void* stream) {
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  if (!q || !page_min || !page_max || !scores || groups <= 0 || n_pages < 0 ||
      heads_per_group <= 0 || groups > 65535)
    return TW_ERR_BAD_ARG;
  if (heads_per_group > kMaxHeadsPerGroup) return TW_ERR_UNSUPPORTED;
  if (n_pages == 0) return TW_OK;
  return quest_score_dispatch(q, TW_F32, page_min, page_max, groups, heads_per_group, n_pages,
                              meta_group_stride, dtype, scores, (cudaStream_t)stream);
}

extern "C" int tw_topk_pages(const float* scores, int rows, int n, int k, int32_t* out_pages,
                             void* stream) {
  if (!scores || !out_pages || rows < 0 || n < 0 || k < 0 || k > n) return TW_ERR_BAD_ARG;
  if (n > kTopkMaxN) return TW_ERR_UNSUPPORTED;
  if (rows == 0 || k == 0) return TW_OK;
  return launch_topk_pages(scores, rows, n, k, out_pages, (cudaStream_t)stream);
}
