// Twilight top-p pruning fused with the GQA union, one thread-block cluster
// per KV group and one CTA per query head of the group.
//
// Reference: top-p via argsort / softmax / per-row cumsum / searchsorted + 1
// (hi/twilight_exact_top_p_graph.py:19-32, hi/twilight_offload_cache.py:1266-1310,
// dynamic budget :1347-1354); GQA union bitmap + sink/recent ranges
// (hi/twilight_offload_cache.py:1527-1549) and its sorted decode via
// np.flatnonzero (:1602-1614).
//
// Top-p without a sort: softmax masses are fixed-point integers (e * 2^48), so
// their sums are exact and order-free.  A 4-pass radix search over the
// logits' order-preserving keys finds the key K* where the mass of the keys
// above K* is < target <= mass of the keys >= K*; the count is the number of
// keys above K* plus the fewest K*-ties (lowest candidate index first) that
// reach the target.  Each CTA then ORs its selected positions into the
// cluster leader's shared-memory bitmap over distributed shared memory; the
// leader writes the sorted union by a popcount scan.
#include <cooperative_groups.h>

#include "tw_common.cuh"

namespace cg = cooperative_groups;

namespace tw {

constexpr int kTopPThreads = 512;

struct TopPArgs {
  const float* logits;
  const int32_t* pages;
  int R;
  int b0;
  int block;
  int sink;
  double top_p;
  int64_t old_length;
  int64_t sink_end;
  int64_t recent_start;
  int32_t* union_pos;
  int64_t pos_stride;
  int32_t* union_count;
  int32_t* head_count;
  int32_t* head_pos;
  int32_t* error_flag;
};

__device__ __forceinline__ int64_t cand_position(const int32_t* prow, int n, int block, int sink) {
  return (int64_t)sink + (int64_t)prow[n / block] * block + (n % block);
}

// Dynamic shared memory layout: keys[n] u32 | mass[n] u64 | bitmap[words] u32 (leader only).
__global__ void __launch_bounds__(kTopPThreads)
top_p_union_kernel(TopPArgs a) {
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ unsigned long long hist_mass[256];
  __shared__ uint32_t hist_cnt[256];
  __shared__ uint32_t scan_scratch[32];
  __shared__ unsigned long long s_red[32];
  __shared__ uint32_t s_prefix;
  __shared__ unsigned long long s_mass_gt, s_target;
  __shared__ uint32_t s_cnt_gt;
  __shared__ float s_max;

  const int R = a.R;
  const int rank = (int)cluster.block_rank();  // query head within the group
  const int g = blockIdx.x / R;
  const int row = g * R + rank;
  const int n = a.b0 * a.block;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;

  const int64_t L = a.old_length;
  const int words = (int)((L + 31) >> 5);
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem_raw);
  unsigned long long* mass =
      reinterpret_cast<unsigned long long*>(smem_raw + (((size_t)n * 4 + 15) & ~(size_t)15));
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(mass) +
                                                 (size_t)n * 8);

  // Leader: clear the bitmap and set the protected sink / recent ranges.
  if (rank == 0) {
    for (int w = tid; w < words; w += blockDim.x) {
      const int64_t lo = (int64_t)w * 32;
      uint32_t bits = 0u;
      for (int b = 0; b < 32; ++b) {
        const int64_t p = lo + b;
        if (p < L && (p < a.sink_end || p >= a.recent_start)) bits |= 1u << b;
      }
      bitmap[w] = bits;
    }
  }

  const float* lrow = a.logits + (int64_t)row * n;
  const int32_t* prow = a.pages + (int64_t)row * a.b0;

  // 1. keys and the row maximum.
  uint32_t kmax = 0u;
  for (int i = tid; i < n; i += blockDim.x) {
    const uint32_t k = float_key(lrow[i]);
    keys[i] = k;
    kmax = max(kmax, k);
  }
  for (int off = 16; off > 0; off >>= 1) kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, off));
  if (lane == 0) scan_scratch[warp] = kmax;
  __syncthreads();
  if (tid == 0) {
    uint32_t m = 0u;
    for (int w = 0; w < nwarps; ++w) m = max(m, scan_scratch[w]);
    s_max = key_float(m);
  }
  __syncthreads();
  const float lmax = s_max;

  // 2. fixed-point masses and their exact total.
  unsigned long long part = 0ull;
  for (int i = tid; i < n; i += blockDim.x) {
    const float d = __fsub_rn(key_float(keys[i]), lmax);
    const unsigned long long m = mass_of(det_exp((double)d));
    mass[i] = m;
    part += m;
  }
  for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  if (lane == 0) s_red[warp] = part;
  __syncthreads();
  if (tid == 0) {
    unsigned long long z = 0ull;
    for (int w = 0; w < nwarps; ++w) z += s_red[w];
    double t = ceil(__dmul_rn((double)z, a.top_p));
    unsigned long long target = (t >= (double)z) ? z : (unsigned long long)t;
    if (target == 0ull) target = 1ull;
    s_target = target;
    s_mass_gt = 0ull;
    s_cnt_gt = 0u;
    s_prefix = 0u;
  }
  __syncthreads();

  // 3. radix search for the threshold key by mass.
  uint32_t mask = 0u;
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += blockDim.x) {
      hist_mass[b] = 0ull;
      hist_cnt[b] = 0u;
    }
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = tid; i < n; i += blockDim.x) {
      const uint32_t key = keys[i];
      if ((key & mask) == prefix) {
        const uint32_t b = (key >> shift) & 255u;
        atomicAdd(&hist_mass[b], mass[i]);
        atomicAdd(&hist_cnt[b], 1u);
      }
    }
    __syncthreads();
    if (warp == 0) {
      const unsigned long long target = s_target;
      const unsigned long long base_mass = s_mass_gt;
      const uint32_t base_cnt = s_cnt_gt;
      unsigned long long lm[8];
      uint32_t lc[8];
      unsigned long long sm = 0ull;
      uint32_t sc = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        lm[j] = hist_mass[8 * lane + j];
        lc[j] = hist_cnt[8 * lane + j];
        sm += lm[j];
        sc += lc[j];
      }
      unsigned long long suf_m = sm;
      uint32_t suf_c = sc;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const unsigned long long ym = __shfl_down_sync(0xffffffffu, suf_m, off);
        const uint32_t yc = __shfl_down_sync(0xffffffffu, suf_c, off);
        if (lane + off < 32) {
          suf_m += ym;
          suf_c += yc;
        }
      }
      const unsigned long long above_m = base_mass + suf_m - sm;
      const uint32_t above_c = base_cnt + suf_c - sc;
      __syncwarp();
      // crossing lane: above_m < target <= above_m + sm (exactly one lane; sm > 0 there)
      if (above_m < target && target <= above_m + sm) {
        unsigned long long acc_m = above_m;
        uint32_t acc_c = above_c;
        for (int j = 7; j >= 0; --j) {
          if (acc_m + lm[j] >= target) {
            s_prefix = prefix | ((uint32_t)(8 * lane + j) << shift);
            s_mass_gt = acc_m;
            s_cnt_gt = acc_c;
            break;
          }
          acc_m += lm[j];
          acc_c += lc[j];
        }
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t kstar = s_prefix;
  const unsigned long long mass_gt = s_mass_gt;
  const uint32_t cnt_gt = s_cnt_gt;
  const unsigned long long target = s_target;
  // every K*-tie has the same logit, hence the same mass
  const unsigned long long m_tie =
      mass_of(det_exp((double)__fsub_rn(key_float(kstar), lmax)));
  unsigned long long need_ull = (m_tie > 0ull) ? (target - mass_gt + m_tie - 1ull) / m_tie : 1ull;

  // 4. tie ranks in candidate order and the per-row outputs.
  const int seg = (n + blockDim.x - 1) / blockDim.x;
  const int beg = min(n, tid * seg);
  const int end = min(n, beg + seg);
  uint32_t eq = 0u, gt = 0u;
  for (int i = beg; i < end; ++i) {
    eq += keys[i] == kstar;
    gt += keys[i] > kstar;
  }
  uint32_t total_eq;
  const uint32_t eq_before = block_exclusive_scan(eq, scan_scratch, &total_eq);
  const uint32_t need = (uint32_t)min(need_ull, (unsigned long long)total_eq);
  const uint32_t take_eq = (eq_before >= need) ? 0u : min(eq, need - eq_before);
  uint32_t total_sel;
  const uint32_t slot0 = block_exclusive_scan(gt + take_eq, scan_scratch, &total_sel);
  if (tid == 0) a.head_count[row] = (int32_t)(cnt_gt + need);

  // All rows are final and the leader's bitmap is initialised.
  cluster.sync();

  uint32_t* leader_bitmap = cluster.map_shared_rank(bitmap, 0);
  int32_t* hp = a.head_pos ? a.head_pos + (int64_t)row * n : nullptr;
  uint32_t slot = slot0, seen = 0u;
  bool bad = false;
  for (int i = beg; i < end; ++i) {
    const uint32_t key = keys[i];
    bool take = key > kstar;
    if (key == kstar) {
      take = seen < take_eq;
      ++seen;
    }
    if (!take) continue;
    const int64_t pos = cand_position(prow, i, a.block, a.sink);
    if (hp) hp[slot] = (int32_t)pos;
    ++slot;
    if (pos < 0 || pos >= L) {
      bad = true;
      continue;
    }
    atomicOr(&leader_bitmap[pos >> 5], 1u << (pos & 31));
  }
  if (bad && a.error_flag) atomicExch(a.error_flag, TW_ERR_INVALID_INDEX);
  cluster.sync();

  if (rank != 0) return;
  // 5. leader: sorted union by popcount scan over contiguous word segments.
  const int wseg = (words + blockDim.x - 1) / blockDim.x;
  const int wbeg = min(words, tid * wseg);
  const int wend = min(words, wbeg + wseg);
  uint32_t cnt = 0u;
  for (int w = wbeg; w < wend; ++w) cnt += __popc(bitmap[w]);
  uint32_t total_union;
  uint32_t out = block_exclusive_scan(cnt, scan_scratch, &total_union);
  int32_t* dst = a.union_pos + (int64_t)g * a.pos_stride;
  for (int w = wbeg; w < wend; ++w) {
    uint32_t bits = bitmap[w];
    while (bits) {
      const int b = __ffs(bits) - 1;
      bits &= bits - 1;
      dst[out++] = w * 32 + b;
    }
  }
  if (tid == 0) a.union_count[g] = (int32_t)total_union;
}

size_t top_p_smem_bytes(int n, int64_t old_length) {
  const size_t keys = (((size_t)n * 4) + 15) & ~(size_t)15;
  const size_t words = (size_t)((old_length + 31) / 32);
  return keys + (size_t)n * 8 + words * 4;
}

int launch_top_p_union(const TopPArgs& args, int groups, cudaStream_t stream) {
  const int n = args.b0 * args.block;
  const size_t smem = top_p_smem_bytes(n, args.old_length);
  int device = 0;
  cudaGetDevice(&device);
  int max_optin = 0;
  cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  // static shared: histograms + scratch (~3.5 KB)
  if (smem + 4096 > (size_t)max_optin) return TW_ERR_CAPACITY;
  cudaError_t err = cudaFuncSetAttribute(top_p_union_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (err == cudaSuccess)
    err = cudaFuncSetAttribute(top_p_union_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups * args.R, 1, 1);
  cfg.blockDim = dim3(kTopPThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = args.R;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  err = cudaLaunchKernelEx(&cfg, top_p_union_kernel, args);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return check_launch();
}

}  // namespace tw

using namespace tw;

extern "C" int tw_top_p_union(const float* logits, const int32_t* pages, int groups,
                              int heads_per_group, int b0_pages, int block_size, int sink,
                              double top_p, int64_t old_length, int64_t sink_end,
                              int64_t recent_start, int32_t* union_pos, int64_t pos_stride,
                              int32_t* union_count, int32_t* head_count, int32_t* head_pos,
                              int32_t* error_flag, void* stream) {
  if (!logits || !pages || !union_pos || !union_count || !head_count || groups <= 0 ||
      heads_per_group <= 0 || b0_pages <= 0 || block_size <= 0 || sink < 0 || old_length < 0 ||
      !(top_p > 0.0 && top_p <= 1.0) || sink_end < 0 || sink_end > old_length ||
      recent_start < sink_end || recent_start > old_length || pos_stride < old_length)
    return TW_ERR_BAD_ARG;
  if (heads_per_group > kMaxHeadsPerGroup) return TW_ERR_UNSUPPORTED;
  const int64_t n = (int64_t)b0_pages * block_size;
  if (n > 65536 || old_length > ((int64_t)1 << 30)) return TW_ERR_UNSUPPORTED;
  TopPArgs args{logits,     pages,     heads_per_group, b0_pages,     block_size, sink,
                top_p,      old_length, sink_end,       recent_start, union_pos,  pos_stride,
                union_count, head_count, head_pos,      error_flag};
  return launch_top_p_union(args, groups, (cudaStream_t)stream);
}
