// Twilight top-p pruning fused with the GQA union, one thread-block cluster
// per KV group and one CTA per query head of the group.
//
// Reference: top-p via argsort / softmax / per-row cumsum / searchsorted + 1
// (hi/twilight_exact_top_p_graph.py:19-32, hi/twilight_offload_cache.py:1266-1310,
// dynamic budget :1347-1354); GQA union bitmap + sink/recent ranges
// (hi/twilight_offload_cache.py:1527-1549) and its sorted decode via
// np.flatnonzero (:1602-1614).
//
// Softmax masses are fixed-point integers (e * 2^48, e = exp(l - max) by the
// deterministic det_exp), so their sums are exact and order-free.  The count
// is the fewest candidates, in descending logit order with ties taken in
// candidate order, whose mass reaches ceil(p * total):
//  * fast path: candidates are binned linearly in (max - logit) over 2048
//    bins, an order-preserving partition (a higher logit never lands in a
//    later bin); one scan of the exact per-bin masses finds the bin where the
//    cumulative mass crosses the target, and the few candidates of that bin
//    are ranked exactly (logit key, then candidate index) to finish the count;
//  * fallback, when the crossing bin holds more than 256 candidates (e.g. many
//    equal logits): a 4-pass radix search over the logits' order-preserving
//    keys for the threshold key, then the fewest ties that reach the target.
// Each CTA then ORs its selected positions, one 32-bit word per page, into
// the cluster leader's shared-memory bitmap over distributed shared memory;
// the leader writes the sorted union by a popcount scan.
#include <cooperative_groups.h>

#include "append.cuh"
#include "select_math.cuh"

namespace cg = cooperative_groups;

namespace tw {

constexpr int kTopPThreads = 1024;

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

// Bits of the 32 positions lo .. lo+31 that lie below x.
__device__ __forceinline__ uint32_t bits_below(int64_t x, int64_t lo) {
  if (x <= lo) return 0u;
  if (x >= lo + 32) return 0xffffffffu;
  return (1u << (uint32_t)(x - lo)) - 1u;
}

__device__ __forceinline__ int64_t cand_position(const int32_t* prow, int n, int block, int sink) {
  return (int64_t)sink + (int64_t)prow[n / block] * block + (n % block);
}

__host__ __device__ __forceinline__ size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

// Dynamic shared memory: keys u32[n] | mass u64[n] | bitmap u32[words] | sel u8[n].
__host__ __device__ __forceinline__ size_t top_p_head_bytes(int n) {
  return align16((size_t)n * 4) + (size_t)n * 8;
}

__device__ __forceinline__ unsigned long long target_of(unsigned long long z, double top_p) {
  const double t = ceil(__dmul_rn((double)z, top_p));
  unsigned long long target = (t >= (double)z) ? z : (unsigned long long)t;
  return target == 0ull ? 1ull : target;
}

constexpr int kTopPBins = 2048;
constexpr int kTopPSmallBin = 256;

// The binned fixed-point mass histogram of a row's candidates: bin b of
// candidate i is min(kTopPBins - 1, (lmax - logit_i) * kTopPBins / span).
__device__ __forceinline__ float top_p_inv_width(float lmax, float lmin) {
  const float span = __fsub_rn(lmax, lmin);
  return span > 0.0f ? __fdiv_rn((float)kTopPBins, span) : 0.0f;
}
__device__ __forceinline__ int top_p_bin(float d, float inv_w) {
  return min(kTopPBins - 1, (int)__fmul_rn(-d, inv_w));
}

// Top-p count and selection of one row from its keys, masses and mass
// histogram, by the whole CTA (kTopPThreads threads).  keys [n]: the
// order-preserving keys of the logits; mass [n]: mass_of(det_exp(logit - lmax));
// bin_mass / bin_cnt [kTopPBins] (16-byte aligned): the histogram, whose total
// is the row's total mass.  On return sel[i] = 1 for the selected candidates;
// returns the count.
__device__ int top_p_select(const uint32_t* keys, const unsigned long long* mass,
                            unsigned char* sel, int n, double top_p, float lmax, float inv_w,
                            const unsigned long long* bin_mass, const uint32_t* bin_cnt) {
  __shared__ unsigned long long list[kTopPSmallBin];
  __shared__ unsigned long long ranked[kTopPSmallBin];
  __shared__ unsigned long long hist_mass[256];
  __shared__ uint32_t hist_cnt[256];
  __shared__ uint32_t scan_scratch[32];
  __shared__ unsigned long long scan64[32];
  __shared__ unsigned long long stage[kTopPThreads / 32][32];
  __shared__ uint32_t s_prefix, s_cnt_gt, s_list_n, s_bcnt;
  __shared__ unsigned long long s_mass_gt, s_target;
  __shared__ int s_bstar, s_count;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  if (tid == 0) {
    s_list_n = 0u;
    s_bstar = -1;
  }

  // 3. crossing bin: bins in order (highest logits first), two per thread.
  constexpr int kBinsPerThread = kTopPBins / kTopPThreads;
  static_assert(kBinsPerThread == 2, "bins are read in pairs");
  const ulonglong2 bm2 = reinterpret_cast<const ulonglong2*>(bin_mass)[tid];
  const uint2 bc2 = reinterpret_cast<const uint2*>(bin_cnt)[tid];
  const unsigned long long bm[kBinsPerThread] = {bm2.x, bm2.y};
  const uint32_t bc[kBinsPerThread] = {bc2.x, bc2.y};
  const unsigned long long bm_local = bm[0] + bm[1];
  const uint32_t bc_local = bc[0] + bc[1];
  unsigned long long z, mrun;
  uint32_t ctotal, crun;
  block_exclusive_scan_pair(bm_local, bc_local, scan64, scan_scratch, &mrun, &crun, &z, &ctotal);
  const unsigned long long target = target_of(z, top_p);
#pragma unroll
  for (int j = 0; j < kBinsPerThread; ++j) {
    const int b = kBinsPerThread * tid + j;
    if (mrun < target && target <= mrun + bm[j]) {
      s_bstar = b;
      s_bcnt = bc[j];
      s_mass_gt = mrun;
      s_cnt_gt = crun;
    }
    mrun += bm[j];
    crun += bc[j];
  }
  __syncthreads();
  const int bstar = s_bstar;

  int count;
  if (bstar >= 0 && s_bcnt <= (uint32_t)kTopPSmallBin) {
    // 4a. rank the crossing bin's candidates exactly and walk their masses.
    for (int i = tid; i < n; i += blockDim.x) {
      const float d = __fsub_rn(key_float(keys[i]), lmax);
      const int b = top_p_bin(d, inv_w);
      sel[i] = b < bstar ? 1 : 0;
      if (b == bstar) list[atomicAdd(&s_list_n, 1u)] = rank_key(keys[i], i);
    }
    __syncthreads();
    const int m_in = (int)s_list_n;
    for (int t = tid; t < m_in; t += blockDim.x) {
      const unsigned long long me = list[t];
      int r = 0;
      for (int j = 0; j < m_in; ++j) r += list[j] > me;
      ranked[r] = me;
    }
    __syncthreads();
    if (warp == 0) {
      unsigned long long base = s_mass_gt;
      int taken = m_in;
      for (int c0 = 0; c0 < m_in; c0 += 32) {
        const int j = c0 + lane;
        unsigned long long v = j < m_in ? mass[rank_index(ranked[j])] : 0ull;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const unsigned long long y = __shfl_up_sync(0xffffffffu, v, off);
          if (lane >= off) v += y;
        }
        const unsigned hit = __ballot_sync(0xffffffffu, j < m_in && base + v >= target);
        if (hit) {
          taken = c0 + __ffs(hit);
          break;
        }
        base += __shfl_sync(0xffffffffu, v, 31);
      }
      if (lane == 0) s_count = (int)s_cnt_gt + taken;
      __syncwarp();
      for (int j = lane; j < taken; j += 32) sel[rank_index(ranked[j])] = 1;
    }
    __syncthreads();
    count = s_count;
  } else {
    // 4b. fallback: radix search over the order-preserving keys.
    if (tid == 0) {
      s_target = target;
      s_mass_gt = 0ull;
      s_cnt_gt = 0u;
      s_prefix = 0u;
    }
    __syncthreads();

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
      // Warp-aggregated histogram: lanes with the same bin are grouped with
      // match.any and each group's leader adds the group's mass (staged per
      // warp in shared memory) and count with one atomic each.
      for (int base = warp * 32; base < n; base += nwarps * 32) {
        const int i = base + lane;
        uint32_t bin = 256u;
        unsigned long long mv = 0ull;
        if (i < n) {
          const uint32_t key = keys[i];
          if ((key & mask) == prefix) {
            bin = (key >> shift) & 255u;
            mv = mass[i];
          }
        }
        const unsigned peers = __match_any_sync(0xffffffffu, bin);
        stage[warp][lane] = mv;
        __syncwarp();
        if (bin != 256u && lane == __ffs(peers) - 1) {
          unsigned long long sum = 0ull;
          for (unsigned p = peers; p; p &= p - 1) sum += stage[warp][__ffs(p) - 1];
          atomicAdd(&hist_mass[bin], sum);
          atomicAdd(&hist_cnt[bin], (uint32_t)__popc(peers));
        }
        __syncwarp();
      }
      __syncthreads();
      if (warp == 0) {
        const unsigned long long tgt = s_target;
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
        // crossing lane: above_m < target <= above_m + sm (exactly one lane)
        if (above_m < tgt && tgt <= above_m + sm) {
          unsigned long long acc_m = above_m;
          uint32_t acc_c = above_c;
          for (int j = 7; j >= 0; --j) {
            if (acc_m + lm[j] >= tgt) {
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
    // every K*-tie has the same logit, hence the same mass
    const unsigned long long m_tie =
        mass_of(det_exp((double)__fsub_rn(key_float(kstar), lmax)));
    const unsigned long long need_ull =
        (m_tie > 0ull) ? (target - mass_gt + m_tie - 1ull) / m_tie : 1ull;
    // tie ranks in candidate order
    const int seg = (n + blockDim.x - 1) / blockDim.x;
    const int beg = min(n, tid * seg);
    const int end = min(n, beg + seg);
    uint32_t eq = 0u;
    for (int i = beg; i < end; ++i) eq += keys[i] == kstar;
    uint32_t total_eq;
    const uint32_t eq_before = block_exclusive_scan(eq, scan_scratch, &total_eq);
    const uint32_t need = (uint32_t)min(need_ull, (unsigned long long)total_eq);
    const uint32_t take_eq = (eq_before >= need) ? 0u : min(eq, need - eq_before);
    uint32_t seen = 0u;
    for (int i = beg; i < end; ++i) {
      const uint32_t key = keys[i];
      bool take = key > kstar;
      if (key == kstar) {
        take = seen < take_eq;
        ++seen;
      }
      sel[i] = take ? 1 : 0;
    }
    count = (int)(cnt_gt + need);
  }
  __syncthreads();

  return count;
}

// Top-p count and selection of one row, by the whole CTA (kTopPThreads threads).
// lrow: the row's n logits (global or shared memory); keys may alias lrow
// (each thread overwrites only the logits it has read).  On return sel[i] = 1
// for the selected candidates; returns the count.
__device__ int top_p_row(const float* lrow, int n, double top_p, uint32_t* keys,
                         unsigned long long* mass, unsigned char* sel) {
  __shared__ __align__(16) unsigned long long bin_mass[kTopPBins];
  __shared__ __align__(16) uint32_t bin_cnt[kTopPBins];
  __shared__ uint32_t s_kmax, s_kmin;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  for (int b = tid; b < kTopPBins; b += blockDim.x) {
    bin_mass[b] = 0ull;
    bin_cnt[b] = 0u;
  }
  if (tid == 0) {
    s_kmax = 0u;
    s_kmin = 0xffffffffu;
  }
  __syncthreads();

  // 1. keys, row max and min.
  uint32_t kmax = 0u, kmin = 0xffffffffu;
  for (int i = tid; i < n; i += blockDim.x) {
    const uint32_t k = float_key(lrow[i]);
    keys[i] = k;
    kmax = max(kmax, k);
    kmin = min(kmin, k);
  }
  for (int off = 16; off > 0; off >>= 1) {
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, off));
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, off));
  }
  if (lane == 0) {
    atomicMax(&s_kmax, kmax);
    atomicMin(&s_kmin, kmin);
  }
  __syncthreads();
  const float lmax = key_float(s_kmax);
  const float inv_w = top_p_inv_width(lmax, key_float(s_kmin));

  // 2. masses and the binned mass histogram.
  for (int i = tid; i < n; i += blockDim.x) {
    const float d = __fsub_rn(key_float(keys[i]), lmax);
    const unsigned long long m = mass_of(det_exp((double)d));
    mass[i] = m;
    const int b = top_p_bin(d, inv_w);
    atomicAdd(&bin_mass[b], m);
    atomicAdd(&bin_cnt[b], 1u);
  }
  __syncthreads();
  return top_p_select(keys, mass, sel, n, top_p, lmax, inv_w, bin_mass, bin_cnt);
}

// ORs the row's selected positions (sel over its candidate pages prow) into
// the cluster leader's bitmap over distributed shared memory, one remote OR
// per selected page (its block_size candidates are consecutive positions);
// pages wider than 32 positions OR per candidate.  Returns true when a
// position fell outside [0, L).
__device__ bool or_selection(uint32_t* leader_bitmap, const int32_t* prow, const unsigned char* sel,
                             int b0, int block, int sink, int64_t L) {
  bool bad = false;
  for (int pg = threadIdx.x; pg < b0; pg += blockDim.x) {
    const int64_t pos0 = (int64_t)sink + (int64_t)prow[pg] * block;
    if (block <= 32) {
      uint32_t m32 = 0u;
      for (int j = 0; j < block; ++j) m32 |= (uint32_t)sel[pg * block + j] << j;
      if (!m32) continue;
      if (pos0 < 0 || pos0 + block > L) {
        bad = true;
        continue;
      }
      const uint32_t sh = (uint32_t)(pos0 & 31);
      atomicOr(&leader_bitmap[pos0 >> 5], m32 << sh);
      if (sh + (uint32_t)block > 32u && (m32 >> (32u - sh)))
        atomicOr(&leader_bitmap[(pos0 >> 5) + 1], m32 >> (32u - sh));
    } else {
      for (int j = 0; j < block; ++j) {
        if (!sel[pg * block + j]) continue;
        const int64_t pos = pos0 + j;
        if (pos < 0 || pos >= L) {
          bad = true;
          continue;
        }
        atomicOr(&leader_bitmap[pos >> 5], 1u << (pos & 31));
      }
    }
  }
  return bad;
}

__global__ void __launch_bounds__(kTopPThreads)
top_p_union_kernel(TopPArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint32_t scan_scratch[32];
  __shared__ uint32_t s_woff[kTopPThreads];

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
      reinterpret_cast<unsigned long long*>(smem_raw + align16((size_t)n * 4));
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem_raw + top_p_head_bytes(n));
  unsigned char* sel = reinterpret_cast<unsigned char*>(bitmap + words);

  // Leader: clear the bitmap and set the protected sink / recent ranges.
  if (rank == 0) {
    const int64_t sink_hi = min(a.sink_end, L);
    for (int w = tid; w < words; w += blockDim.x) {
      const int64_t lo = (int64_t)w * 32;
      bitmap[w] = bits_below(sink_hi, lo) | (bits_below(L, lo) & ~bits_below(a.recent_start, lo));
    }
  }
  const float* lrow = a.logits + (int64_t)row * n;
  const int32_t* prow = a.pages + (int64_t)row * a.b0;
  const int count = top_p_row(lrow, n, a.top_p, keys, mass, sel);

  // Per-row outputs: the count and (optionally) the selected positions in
  // candidate order, i.e. ascending positions (pages are ascending).
  if (tid == 0) a.head_count[row] = count;
  if (a.head_pos) {
    const int seg = (n + blockDim.x - 1) / blockDim.x;
    const int beg = min(n, tid * seg);
    const int end = min(n, beg + seg);
    uint32_t c = 0u;
    for (int i = beg; i < end; ++i) c += sel[i];
    uint32_t total;
    uint32_t slot = block_exclusive_scan(c, scan_scratch, &total);
    int32_t* hp = a.head_pos + (int64_t)row * n;
    for (int i = beg; i < end; ++i)
      if (sel[i]) hp[slot++] = (int32_t)cand_position(prow, i, a.block, a.sink);
  }

  // All rows are final and the leader's bitmap is initialised.
  cluster.sync();

  uint32_t* leader_bitmap = cluster.map_shared_rank(bitmap, 0);
  const bool bad = or_selection(leader_bitmap, prow, sel, a.b0, a.block, a.sink, L);
  if (bad && a.error_flag) atomicExch(a.error_flag, TW_ERR_INVALID_INDEX);
  cluster.sync();

  if (rank != 0) return;
  // Leader: sorted union.  Words are taken 1024 at a time (one per thread):
  // an exclusive scan of their popcounts gives each word's output offset, then
  // warp w writes word (32 * pass + w)'s set bits, one lane per bit, so a
  // word's positions go to consecutive addresses in one coalesced store.
  int32_t* dst = a.union_pos + (int64_t)g * a.pos_stride;
  uint32_t total_union = 0u;
  for (int c0 = 0; c0 < words; c0 += kTopPThreads) {
    const int w = c0 + tid;
    const uint32_t bits = w < words ? bitmap[w] : 0u;
    uint32_t chunk_total;
    s_woff[tid] = total_union + block_exclusive_scan((uint32_t)__popc(bits), scan_scratch, &chunk_total);
    __syncthreads();
    const int chunk_words = min(kTopPThreads, words - c0);
    for (int j = warp; j < chunk_words; j += nwarps) {
      const uint32_t word = bitmap[c0 + j];
      if ((word >> lane) & 1u)
        dst[s_woff[j] + __popc(word & ((1u << lane) - 1u))] = (c0 + j) * 32 + lane;
    }
    total_union += chunk_total;
    __syncthreads();
  }
  if (tid == 0) a.union_count[g] = (int32_t)total_union;
}

size_t top_p_smem_bytes(int n, int64_t old_length) {
  const size_t words = (size_t)((old_length + 31) / 32);
  return top_p_head_bytes(n) + words * 4 + (size_t)n;
}

int launch_top_p_union(const TopPArgs& args, int groups, cudaStream_t stream) {
  const int n = args.b0 * args.block;
  const size_t smem = top_p_smem_bytes(n, args.old_length);
  static int optin_cache[kMaxDevices];
  static int static_smem_cache[kMaxDevices];
  static DynSmemOptIn opt_in;
  int max_optin = 0;
  int st = cached_device_attribute(cudaDevAttrMaxSharedMemoryPerBlockOptin, optin_cache, max_optin);
  if (st != TW_OK) return st;
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  int static_smem = (device >= 0 && device < kMaxDevices) ? static_smem_cache[device] : 0;
  if (static_smem <= 0) {
    cudaFuncAttributes fa{};
    err = cudaFuncGetAttributes(&fa, top_p_union_kernel);
    if (err != cudaSuccess) {
      set_last_cuda_error(err);
      return TW_ERR_CUDA;
    }
    static_smem = (int)fa.sharedSizeBytes;
    if (device >= 0 && device < kMaxDevices) static_smem_cache[device] = static_smem;
  }
  if (smem + (size_t)static_smem > (size_t)max_optin) return TW_ERR_CAPACITY;
  st = ensure_dyn_smem((const void*)top_p_union_kernel, opt_in, (int)smem);
  if (st != TW_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups * args.R, 1, 1);
  cfg.blockDim = dim3(kTopPThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = args.R;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  err = cudaLaunchKernelEx(&cfg, top_p_union_kernel, args);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return check_launch();
}

// ---- whole-layer selection in one launch ---------------------------------------------------
// One thread-block cluster of C CTAs per query-head row (g, r) of the layer,
// G*R row clusters in all, runs the four selection stages of its row with
// every intermediate in the shared memory of its leader CTA (rank 0):
//  1. Quest scores: the C CTAs split the candidate pages, 4 threads per page
//     (quest_page_score4); the scores go to the leader over distributed
//     shared memory;
//  2. top-k pages: the leader radix-selects the row's B0 pages (as
//     topk_pages_kernel), ascending;
//  3. INT4 estimate: the C CTAs split the row's candidates; logits go to the
//     leader;
//  4. top-p: the leader counts and marks the row's selection (top_p_row);
//  5. GQA union: the leader ORs its selected candidates into the group's
//     bitmap in global memory (one bit per candidate position, bit 0 =
//     position sink) and counts its row in; the row cluster that counts in
//     last writes the group's sorted union [0, sink_end) U bitmap U
//     [recent_start, old_length), then clears the bitmap and the count, so
//     the merge region is zero again for the next launch.  No row cluster
//     waits for another, so they need not be resident together.
// Scores, pages, logits, counts and unions are bit-identical to the
// per-stage kernels (same arithmetic, select_math.cuh).
// C is the largest cluster size (<= 8) for which every cluster of the launch
// is resident at once (one SM per CTA).  One further cluster, when the caller
// asks for it, does work independent of this step's selection while the row
// clusters run, with no cluster barrier (so that its host reads never hold
// up a barrier): it appends the new token (position old_length, beyond every
// row the selection and the attention read) and stages the protected rows
// (ProtectedStage) with 16-byte loads.
constexpr int kSelMaxCluster = 8;  // portable cluster size

__host__ __device__ constexpr bool select_fused_r(int R) { return R >= 1 && R <= kMaxHeadsPerGroup; }

struct SelectArgs {
  const void* q;          // [G][R][D], QT
  const void* pmin;       // first group's page min / max, K dtype
  const void* pmax;
  int64_t meta_stride;    // elements between consecutive groups' page arrays
  int n_pages;
  const uint8_t* packed;  // first group's INT4 codes
  const void* scale;
  const void* minimum;
  int64_t entry_stride;   // tokens between consecutive groups' code rows
  int group_size;
  int b0;
  int block;
  int sink;
  double top_p;
  int64_t old_length;
  int64_t sink_end;
  int64_t recent_start;
  float inv_sqrt_d;
  int32_t* pages_out;     // [G][R][b0]
  int32_t* union_pos;
  int64_t pos_stride;
  int32_t* union_count;
  int32_t* head_count;
  int32_t* head_pos;
  int32_t* error_flag;
  int groups;
  int R;
  unsigned int* merge_count;  // [G] row clusters counted in (zero between launches)
  uint32_t* merge_bits;       // [G][merge_words] candidate bitmap (zero between launches)
  int merge_words;
  ProtectedStage stage;       // the extra cluster stages the protected rows when
  AppendArgs append;          // stage.stage_k is set, and appends the new token
  int do_append;              // when do_append is set
  int block_shift;            // block == 1 << block_shift, or -1 (not a power of two)
};

// Merge region of the selection workspace: the last bytes of the caller's
// buffer (so that the per-stage kernels' scores and logits at its start never
// overlap it): count u32[G] at the very end, the bitmap u32[G][words] before.
__host__ __device__ __forceinline__ int merge_words_of(int n_pages, int block) {
  return (int)(((int64_t)n_pages * block + 31) / 32);
}
size_t merge_region_bytes(int groups, int n_pages, int block) {
  const size_t bits = (size_t)groups * merge_words_of(n_pages, block) * 4;
  return ((bits + 255) & ~(size_t)255) + (((size_t)groups * 4 + 255) & ~(size_t)255);
}

struct TopKShared {
  uint32_t hist[256];
  uint32_t scratch[32];
  uint32_t prefix, remaining, resolved;
};

// Dynamic shared memory: the top-k state | scores f32[max(P, words)] (keys
// alias them; the union writer's bitmap words later) | pages i32[b0] | logits
// f32[n] (keys alias them) | mass u64[n] | sel u8[n] | the row's query as
// fp32 [D].
__host__ __device__ __forceinline__ size_t select_smem_bytes(int P, int b0, int n, int words) {
  return align16(sizeof(TopKShared)) + align16((size_t)max(P, words) * 4) +
         align16((size_t)b0 * 4) + align16((size_t)n * 4) + align16((size_t)n * 8) +
         align16((size_t)n) + (size_t)kHeadDim * 4;
}

// Top-k pages of a row by the leader CTA: keys [P] (order-preserving score
// keys) -> the B0 = k selected page indices ascending in s_pages and gout:
// every key above the k-th largest and the lowest-index ties of it, by the
// 4-pass radix select of topk_pages_kernel.
__device__ void topk_row(const uint32_t* keys, int P, int k, int32_t* s_pages, int32_t* gout,
                         TopKShared& sh) {
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  if (tid == 0) {
    sh.prefix = 0u;
    sh.remaining = (uint32_t)k;
    sh.resolved = 0u;
  }
  __syncthreads();
  uint32_t mask = 0u;
  // A pass whose crossing bin holds exactly the keys still needed resolves
  // the selection: every key whose masked prefix is at or above it is taken
  // (k keys in all), the set the remaining passes would also give.
#pragma unroll 1
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = tid; b < 256; b += blockDim.x) sh.hist[b] = 0u;
    __syncthreads();
    const uint32_t prefix = sh.prefix;
    for (int i = tid; i < P; i += blockDim.x) {
      const uint32_t key = keys[i];
      if ((key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t local[8];
      uint32_t sum = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        local[j] = sh.hist[8 * lane + j];
        sum += local[j];
      }
      uint32_t suffix = sum;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_down_sync(0xffffffffu, suffix, off);
        if (lane + off < 32) suffix += y;
      }
      const uint32_t above = suffix - sum;
      const uint32_t need = sh.remaining;
      __syncwarp();
      if (above < need && need <= suffix) {
        uint32_t acc = above;
        for (int j = 7; j >= 0; --j) {
          if (acc + local[j] >= need) {
            sh.prefix = prefix | ((uint32_t)(8 * lane + j) << shift);
            sh.remaining = need - acc;
            sh.resolved = (local[j] == need - acc) ? 1u : 0u;
            break;
          }
          acc += local[j];
        }
      }
    }
    mask |= 255u << shift;
    __syncthreads();
    if (sh.resolved) break;
  }
  const uint32_t kth = sh.prefix;
  const uint32_t ties = sh.remaining;
  // masked keys above kth and the first `ties` masked keys equal to it, in
  // index order (mask covers the passes run)
  const int seg = (P + blockDim.x - 1) / blockDim.x;
  const int beg = min(P, tid * seg);
  const int end = min(P, beg + seg);
  uint32_t gt = 0u, eq = 0u;
  for (int i = beg; i < end; ++i) {
    const uint32_t key = keys[i] & mask;
    gt += key > kth;
    eq += key == kth;
  }
  uint32_t total;
  const uint32_t eq_before = block_exclusive_scan(eq, sh.scratch, &total);
  const uint32_t take_eq = (eq_before >= ties) ? 0u : min(eq, ties - eq_before);
  const uint32_t base = block_exclusive_scan(gt + take_eq, sh.scratch, &total);
  uint32_t slot = base, eq_seen = 0u;
  for (int i = beg; i < end; ++i) {
    const uint32_t key = keys[i] & mask;
    bool take = key > kth;
    if (key == kth) {
      take = eq_seen < take_eq;
      ++eq_seen;
    }
    if (take) {
      s_pages[slot] = i;
      gout[slot] = i;
      ++slot;
    }
  }
  __syncthreads();
}

template <typename T, typename QT>
__global__ void __launch_bounds__(kTopPThreads)
select_rows_kernel(SelectArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  cg::cluster_group cluster = cg::this_cluster();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ uint32_t s_woff[kTopPThreads];
  __shared__ uint32_t s_ctotal[kSelMaxCluster];
  __shared__ uint32_t s_last;
  // The query again for the INT4 phase, each 4-lane group's 32-channel slice
  // rotated by 4 * slice: the four slices' 16-byte loads of one step then fall
  // in four different bank groups (no bank conflict).
  __shared__ __align__(16) float s_qx[kHeadDim];

  const int C = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const int R = a.R;
  const int row = blockIdx.x / C;  // g * R + r
  if (row >= a.groups * R) {  // the extra cluster: no cluster barrier, no shared memory
    const int cta = (int)blockIdx.x - a.groups * R * C;
    const int flat = cta * (int)blockDim.x + (int)threadIdx.x;
    if (a.do_append && flat < a.groups * kHeadDim)
      append_token_row<T>(a.append, flat / kHeadDim, flat % kHeadDim);
    if (a.stage.stage_k) stage_protected_rows(a.stage, a.groups, cta, C);
    return;
  }
  const int g = row / R;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  const int P = a.n_pages;
  const int n = a.b0 * a.block;
  const int64_t L = a.old_length;
  const bool leader = crank == 0;
  const int words = a.merge_words;

  unsigned char* cur = smem_raw;
  TopKShared& s_topk = *reinterpret_cast<TopKShared*>(cur);
  cur += align16(sizeof(TopKShared));
  float* s_score = reinterpret_cast<float*>(cur);
  cur += align16((size_t)max(P, words) * 4);
  int32_t* s_pages = reinterpret_cast<int32_t*>(cur);
  cur += align16((size_t)a.b0 * 4);
  float* s_logit = reinterpret_cast<float*>(cur);
  cur += align16((size_t)n * 4);
  unsigned long long* mass = reinterpret_cast<unsigned long long*>(cur);
  cur += align16((size_t)n * 8);
  unsigned char* sel = cur;
  cur += align16((size_t)n);
  float* s_q = reinterpret_cast<float*>(cur);

  const T* scale = reinterpret_cast<const T*>(a.scale);
  const T* minimum = reinterpret_cast<const T*>(a.minimum);
  const int ngroups = kHeadDim / a.group_size;
  const int64_t tbase = (int64_t)g * a.entry_stride + a.sink;
  const T* gmin = reinterpret_cast<const T*>(a.pmin) + (int64_t)g * a.meta_stride;
  const T* gmax = reinterpret_cast<const T*>(a.pmax) + (int64_t)g * a.meta_stride;
  const int per_cta = (P + C - 1) / C;
  const int p_beg = min(P, crank * per_cta);
  const int p_end = min(P, p_beg + per_cta);
  // This CTA's Quest min / max range is requested from DRAM into L2 before
  // anything waits on memory, so the score loads below wait on L2 rather than
  // each on a DRAM round trip.
  if (tid < 2 && p_end > p_beg)
    prefetch_l2((tid == 0 ? gmin : gmax) + (int64_t)p_beg * kHeadDim,
                (size_t)(p_end - p_beg) * kHeadDim * sizeof(T));
  {
    const QT* qg = reinterpret_cast<const QT*>(a.q) + (int64_t)row * kHeadDim;
    for (int i = tid; i < kHeadDim; i += blockDim.x) {
      const float v = to_f32(qg[i]);
      s_q[i] = v;
      const int slice = i >> 5;
      s_qx[32 * slice + (((i & 31) + 4 * slice) & 31)] = v;
    }
  }
  __syncthreads();  // s_q, s_qx

  // 1. Quest scores of the row's query head over the group's candidate pages.
  {
    float* owner_scores = cluster.map_shared_rank(s_score, 0);
    const int j4 = lane & 3;
    const int pages_per_pass = (int)(blockDim.x >> 2);
    for (int base = p_beg + warp * 8; base < p_end; base += pages_per_pass) {
      const int p = base + (lane >> 2);  // base is warp-uniform: the 4-lane shuffles
      const bool valid = p < p_end;
      const float sc = quest_page_score4<T>(s_q, gmin, gmax, valid ? p : p_beg, j4, valid);
      if (valid && j4 == 0) owner_scores[p] = sc;
    }
  }
  cluster.sync();

  // 2. top-k pages of the row, ascending.
  if (leader) {
    uint32_t* keys = reinterpret_cast<uint32_t*>(s_score);
    for (int i = tid; i < P; i += blockDim.x) keys[i] = float_key(s_score[i]);
    __syncthreads();
    topk_row(keys, P, a.b0, s_pages, a.pages_out + (int64_t)row * a.b0, s_topk);
  }
  cluster.sync();

  // 3. INT4 estimate: the C CTAs split the row's candidates.
  {
    if (!leader) {  // this CTA's copy of the row's pages (the loop reads them per candidate)
      const int32_t* src = cluster.map_shared_rank(s_pages, 0);
      for (int i = tid; i < a.b0; i += blockDim.x) s_pages[i] = src[i];
    }
    __syncthreads();
    const int chunk = (n + C - 1) / C;
    const int c_beg = min(n, crank * chunk);
    const int c_end = min(n, c_beg + chunk);
    const int sub = lane & 3;
    const int tok = lane >> 2;
    float qr[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(s_qx + 32 * sub + ((4 * j + 4 * sub) & 31));
      qr[4 * j] = v.x;
      qr[4 * j + 1] = v.y;
      qr[4 * j + 2] = v.z;
      qr[4 * j + 3] = v.w;
    }
    const int grp = (32 * sub) / a.group_size;
    const int32_t* prow = s_pages;
    float* lout = cluster.map_shared_rank(s_logit, 0);
    constexpr int kStep = kTopPThreads / 4;  // candidates per pass of the CTA
    constexpr int kAhead = 2;                // passes whose loads are in flight together
    // Each 4-lane group estimates one candidate per pass; the codes of kAhead
    // passes are loaded before their arithmetic, so their latencies overlap.
    // Candidate i is token sink + prow[i / block] * block + i % block of the
    // group's entry.
    auto token_of = [&](int i) -> int64_t {
      int pg, t;
      if (a.block_shift >= 0) {
        pg = i >> a.block_shift;
        t = i & (a.block - 1);
      } else {
        pg = i / a.block;
        t = i - pg * a.block;
      }
      return tbase + (int64_t)prow[pg] * a.block + t;
    };
    for (int base0 = c_beg + warp * 8; base0 < c_end; base0 += kAhead * kStep) {  // warp-uniform
      uint4 codes[kAhead];
      T sv[kAhead];
      float mv[kAhead];
#pragma unroll
      for (int u = 0; u < kAhead; ++u) {
        const int i = base0 + u * kStep + tok;
        codes[u] = make_uint4(0u, 0u, 0u, 0u);
        sv[u] = from_f32<T>(0.0f);
        mv[u] = 0.0f;
        if (i < c_end) {
          const int64_t tr = token_of(i);
          codes[u] = __ldg(reinterpret_cast<const uint4*>(a.packed + tr * (kHeadDim / 2)) + sub);
          sv[u] = scale[tr * ngroups + grp];
          mv[u] = to_f32(minimum[tr * ngroups + grp]);
        }
      }
#pragma unroll
      for (int u = 0; u < kAhead; ++u) {
        const int base = base0 + u * kStep;
        if (base >= c_end) break;  // warp-uniform
        const float logit = int4_logit(int4_dot32<T>(codes[u], sv[u], mv[u], qr), a.inv_sqrt_d);
        if (base + tok < c_end && sub == 0) lout[base + tok] = logit;
      }
    }
  }
  cluster.sync();

  // 4. top-p of the row; its selection into the group's merge bitmap.
  unsigned int* gcount = a.merge_count + g;
  uint32_t* gbits = a.merge_bits + (int64_t)g * words;
  if (leader) {
    const int count = top_p_row(s_logit, n, a.top_p, reinterpret_cast<uint32_t*>(s_logit), mass, sel);
    if (tid == 0) a.head_count[row] = count;
    if (a.head_pos) {
      const int seg = (n + blockDim.x - 1) / blockDim.x;
      const int beg = min(n, tid * seg);
      const int end = min(n, beg + seg);
      uint32_t c = 0u;
      for (int i = beg; i < end; ++i) c += sel[i];
      uint32_t total;
      uint32_t slot = block_exclusive_scan(c, s_topk.scratch, &total);
      int32_t* hp = a.head_pos + (int64_t)row * n;
      for (int i = beg; i < end; ++i)
        if (sel[i]) hp[slot++] = (int32_t)cand_position(s_pages, i, a.block, a.sink);
    }
    // candidate bit b = page * block + j (position sink + b)
    bool bad = false;
    for (int pg = tid; pg < a.b0; pg += blockDim.x) {
      const int page = s_pages[pg];
      if (page < 0 || page >= P) {
        bad = true;
        continue;
      }
      const int64_t b_page = (int64_t)page * a.block;
      for (int j = 0; j < a.block;) {
        const int64_t b = b_page + j;
        const int take = min(a.block - j, 32 - (int)(b & 31));
        uint32_t m32 = 0u;
        for (int t = 0; t < take; ++t) m32 |= (uint32_t)sel[pg * a.block + j + t] << t;
        if (m32) atomicOr(&gbits[b >> 5], m32 << (uint32_t)(b & 31));
        j += take;
      }
    }
    if (bad && a.error_flag) atomicExch(a.error_flag, TW_ERR_INVALID_INDEX);
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned int prev = atomicAdd(gcount, 1u);
      __threadfence();
      const uint32_t last = (prev == (unsigned int)R - 1u) ? 1u : 0u;
      // to every CTA's own copy: after the barrier below no CTA reads the
      // leader's shared memory, so each may exit on its own
      for (int c = 0; c < C; ++c) *cluster.map_shared_rank(&s_last, c) = last;
    }
  }
  cluster.sync();

  // 5. The row cluster counted in last writes the group's sorted union.  CTA
  //    c takes the bitmap words [c*ws, (c+1)*ws) into its shared memory and
  //    clears them in global memory; the word totals go to every CTA over
  //    distributed shared memory; CTA 0 also writes the sink range, CTA C-1
  //    the recent window and the count.
  if (s_last) {
    __threadfence();
    const int ws = (words + C - 1) / C;
    const int w_beg = min(words, crank * ws);
    const int w_end = min(words, w_beg + ws);
    const int nw = w_end - w_beg;
    uint32_t* s_words = reinterpret_cast<uint32_t*>(s_score);
    uint32_t mine = 0u;
    for (int w = tid; w < nw; w += blockDim.x) {
      const uint32_t x = __ldcg(gbits + w_beg + w);
      s_words[w] = x;
      mine += __popc(x);
      gbits[w_beg + w] = 0u;
    }
    uint32_t ctotal;
    {
      const uint32_t excl = block_exclusive_scan(mine, s_topk.scratch, &ctotal);
      if (nw <= (int)blockDim.x) s_woff[tid] = excl;  // word tid is thread tid's only word
    }
    if (tid == 0)
      for (int c = 0; c < C; ++c) cluster.map_shared_rank(s_ctotal, c)[crank] = ctotal;
    cluster.sync();  // totals exchanged; no shared memory of another CTA is read after this
    uint32_t running = 0u;
    for (int c = 0; c < crank; ++c) running += s_ctotal[c];
    int32_t* dst = a.union_pos + (int64_t)g * a.pos_stride;
    const int64_t sink_hi = min(a.sink_end, L);
    if (crank == 0)
      for (int64_t p = tid; p < sink_hi; p += blockDim.x) dst[p] = (int32_t)p;
    for (int c0 = 0; c0 < nw; c0 += kTopPThreads) {
      const int chunk_words = min(kTopPThreads, nw - c0);
      uint32_t chunk_total = ctotal;
      if (nw > (int)blockDim.x) {  // several words per thread: offsets of this chunk
        const int w = c0 + tid;
        const uint32_t bits = w < nw ? s_words[w] : 0u;
        s_woff[tid] = block_exclusive_scan((uint32_t)__popc(bits), s_topk.scratch, &chunk_total);
        __syncthreads();
      }
      for (int j = warp; j < chunk_words; j += nwarps) {
        const uint32_t word = s_words[c0 + j];
        if ((word >> lane) & 1u)
          dst[sink_hi + running + s_woff[j] + __popc(word & ((1u << lane) - 1u))] =
              (int32_t)(a.sink + (int64_t)(w_beg + c0 + j) * 32 + lane);
      }
      running += chunk_total;
      __syncthreads();
    }
    if (crank == C - 1) {
      const int64_t recent_lo = max(a.recent_start, sink_hi);
      int32_t* rdst = dst + sink_hi + running;
      for (int64_t p = recent_lo + tid; p < L; p += blockDim.x) rdst[p - recent_lo] = (int32_t)p;
      if (tid == 0) a.union_count[g] = (int32_t)(sink_hi + running + (L - recent_lo));
    }
    if (crank == 0 && tid == 0) *gcount = 0u;
  }
}

// Whether the fused selection serves this shape (shared memory fitting one CTA).
bool select_fused_supported(int R, int P, int b0, int block, int64_t L, size_t* smem) {
  if (!select_fused_r(R) || b0 <= 0 || P <= 0) return false;
  const int64_t n = (int64_t)b0 * block;
  if (n > 65536 || L > ((int64_t)1 << 30)) return false;
  *smem = select_smem_bytes(P, b0, (int)n, merge_words_of(P, block));
  return *smem <= 160 * 1024;
}

// Cluster size: the largest C <= 8 for which all `clusters` clusters of C
// CTAs (one SM each, at the shared memory the selection may use) are resident
// at once on this device, queried once per device and kernel; 1 when none is.
template <typename T, typename QT>
int select_cluster_size(int clusters) {
  static std::mutex mu;
  static int max_active[kMaxDevices][kSelMaxCluster + 1];  // 0: not queried, -1: failed
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 1;
  std::lock_guard<std::mutex> lk(mu);
  const void* fn = (const void*)select_rows_kernel<T, QT>;
  for (int c = kSelMaxCluster; c >= 2; --c) {
    if (max_active[dev][c] == 0) {
      int count = -1;
      if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024) ==
          cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c, 1, 1);
        cfg.blockDim = dim3(kTopPThreads, 1, 1);
        cfg.dynamicSmemBytes = 160 * 1024;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = c;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int k = 0;
        if (cudaOccupancyMaxActiveClusters(&k, fn, &cfg) == cudaSuccess && k > 0) count = k;
      }
      cudaGetLastError();  // a refused query leaves no error behind
      max_active[dev][c] = count;
    }
    if (max_active[dev][c] >= clusters) return c;
  }
  return 1;
}

template <typename T, typename QT>
int launch_select_rows(const SelectArgs& a, size_t smem, cudaStream_t stream) {
  static DynSmemOptIn opt_in;
  const int rows = a.groups * a.R;
  const bool extra = a.stage.stage_k != nullptr || a.do_append;
  const int cluster = select_cluster_size<T, QT>(rows + (extra ? 1 : 0));
  if (extra && (int64_t)a.groups * kHeadDim > (int64_t)cluster * kTopPThreads)
    return TW_ERR_UNSUPPORTED;  // the extra cluster covers 128 threads per group's append
  const int st = ensure_dyn_smem((const void*)select_rows_kernel<T, QT>, opt_in, (int)smem);
  if (st != TW_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((rows + (extra ? 1 : 0)) * cluster, 1, 1);
  cfg.blockDim = dim3(kTopPThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, select_rows_kernel<T, QT>, a);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return check_launch();
}

// The whole Twilight selection of one layer in one launch when the shape
// allows it (shared memory fitting a CTA); returns TW_ERR_UNSUPPORTED
// otherwise, and the caller runs the per-stage kernels.  Same arguments and
// checks as tw_select_layer's stages; q in fp32 or the K dtype.  workspace:
// the caller's selection workspace (its last merge_region_bytes hold the
// union merge state and must be zero before the first call; every call
// leaves them zero).
int select_layer_fused(const void* q, int q_dtype, const void* pmin, const void* pmax,
                       int64_t meta_stride, int n_pages, const uint8_t* packed, const void* scale,
                       const void* minimum, int64_t entry_stride, int groups, int R, int b0,
                       int block, int sink, int group_size, int dtype, double top_p,
                       int64_t old_length, int64_t sink_end, int64_t recent_start,
                       int32_t* pages_out, int32_t* union_pos, int64_t pos_stride,
                       int32_t* union_count, int32_t* head_count, int32_t* head_pos,
                       int32_t* error_flag, void* workspace, size_t workspace_bytes,
                       const ProtectedStage* stage, const AppendArgs* append,
                       cudaStream_t stream) {
  if (!q || !pmin || !pmax || !packed || !scale || !minimum || !pages_out || !union_pos ||
      !union_count || !head_count || groups <= 0 || groups > (1 << 27) || R <= 0 ||
      n_pages <= 0 || b0 <= 0 || b0 > n_pages || block <= 0 || sink < 0 || old_length < 0 ||
      !(top_p > 0.0 && top_p <= 1.0) || sink_end < 0 || sink_end > old_length ||
      recent_start < sink_end || recent_start > old_length || pos_stride < old_length)
    return TW_ERR_BAD_ARG;
  if (R > kMaxHeadsPerGroup) return TW_ERR_UNSUPPORTED;
  if (group_size != 32 && group_size != 64 && group_size != 128) return TW_ERR_UNSUPPORTED;
  if (dtype != TW_F16 && dtype != TW_BF16) return TW_ERR_UNSUPPORTED;
  if (q_dtype != TW_F32 && q_dtype != dtype) return TW_ERR_BAD_ARG;
  // candidate positions sink + page * block must lie in [sink_end, recent_start)
  if ((int64_t)sink + (int64_t)n_pages * block > recent_start || sink < sink_end)
    return TW_ERR_UNSUPPORTED;
  if ((int64_t)groups * R * kSelMaxCluster > (int64_t)INT32_MAX / 2) return TW_ERR_UNSUPPORTED;
  size_t smem = 0;
  if (!select_fused_supported(R, n_pages, b0, block, old_length, &smem)) return TW_ERR_UNSUPPORTED;
  // 16-byte page-row loads (8 channels) in the Quest phase
  if ((((uintptr_t)pmin | (uintptr_t)pmax) & 15) != 0 || meta_stride % 8 != 0)
    return TW_ERR_UNSUPPORTED;
  const size_t merge = merge_region_bytes(groups, n_pages, block);
  if (!workspace || workspace_bytes < merge || ((uintptr_t)workspace & 3) != 0)
    return TW_ERR_CAPACITY;
  SelectArgs a{};
  a.q = q;
  a.pmin = pmin;
  a.pmax = pmax;
  a.meta_stride = meta_stride;
  a.n_pages = n_pages;
  a.packed = packed;
  a.scale = scale;
  a.minimum = minimum;
  a.entry_stride = entry_stride;
  a.group_size = group_size;
  a.b0 = b0;
  a.block = block;
  a.sink = sink;
  a.top_p = top_p;
  a.old_length = old_length;
  a.sink_end = sink_end;
  a.recent_start = recent_start;
  a.inv_sqrt_d = inv_sqrt_head_dim(kHeadDim);
  a.pages_out = pages_out;
  a.union_pos = union_pos;
  a.pos_stride = pos_stride;
  a.union_count = union_count;
  a.head_count = head_count;
  a.head_pos = head_pos;
  a.error_flag = error_flag;
  a.groups = groups;
  a.R = R;
  {
    // merge region at the end of the caller's buffer (4-byte aligned words)
    char* end = reinterpret_cast<char*>(workspace) + (workspace_bytes & ~(size_t)3);
    const size_t count_bytes = ((size_t)groups * 4 + 255) & ~(size_t)255;
    a.merge_count = reinterpret_cast<unsigned int*>(end - count_bytes);
    a.merge_words = merge_words_of(n_pages, block);
    a.merge_bits = reinterpret_cast<uint32_t*>(end - merge);
  }
  a.block_shift = -1;
  for (int b = 0; b < 31; ++b)
    if (block == (1 << b)) a.block_shift = b;
  if (stage && stage->stage_k) {
    if (!stage->stage_v || (!stage->dirs && (!stage->slab_k || !stage->slab_v)) ||
        stage->first_entry < 0 || stage->first_entry + (int64_t)groups > stage->n_entries ||
        old_length > stage->max_len || stage->n_sink != sink_end ||
        stage->recent_start != recent_start || stage->old_length != old_length ||
        stage->stage_rows < sink_end + (old_length - recent_start) ||
        (((uintptr_t)stage->stage_k | (uintptr_t)stage->stage_v | (uintptr_t)stage->slab_k |
          (uintptr_t)stage->slab_v) & 15) != 0)
      return TW_ERR_BAD_ARG;
    a.stage = *stage;
  }
  if (append) {
    a.append = *append;
    a.do_append = 1;
  }
  if (dtype == TW_F16)
    return q_dtype == TW_F32 ? launch_select_rows<__half, float>(a, smem, stream)
                             : launch_select_rows<__half, __half>(a, smem, stream);
  return q_dtype == TW_F32 ? launch_select_rows<__nv_bfloat16, float>(a, smem, stream)
                           : launch_select_rows<__nv_bfloat16, __nv_bfloat16>(a, smem, stream);
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
