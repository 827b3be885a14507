// Zero-copy row gathers: the GPU reads the selected K/V rows straight from the
// pinned, device-mapped host slab (or from device memory) with 16-byte loads
// and writes them into the flat attention layout.
//
// Reference: gather_kv (hi/cpu_kv_gather.cpp:3-16), assemble_zero_copy miss
// branch (hi/resident_zero_copy.cu:7-42), the flat CPU gather + chunked H2D +
// direct attention layout of update_layer_gqa_group_ragged
// (hi/twilight_offload_cache.py:2973-3101, :3307-3310), and the per-query-head
// packing of QuestTopKOffloadedCache (hi/quest_offload_cache.py:403-511, :724-987).
#include "tw_common.cuh"

namespace tw {

// Each thread moves one 16-byte vector of a row; kUnroll rows are loaded
// before any is stored so that many host-link reads are in flight.
constexpr int kGatherThreads = 256;
constexpr int kGatherUnroll = 4;

__global__ void __launch_bounds__(kGatherThreads)
gather_kv_kernel(const uint4* __restrict__ k, const uint4* __restrict__ v, uint4* __restrict__ ok,
                 uint4* __restrict__ ov, const int64_t* __restrict__ rows, int64_t n,
                 int64_t source_rows, int vec_per_row, int32_t* error_flag) {
  const int rows_per_cta = kGatherThreads / vec_per_row;
  const int sub_row = threadIdx.x / vec_per_row;
  const int col = threadIdx.x % vec_per_row;
  if (sub_row >= rows_per_cta) return;
  const int64_t stride = (int64_t)gridDim.x * rows_per_cta;
  for (int64_t base = (int64_t)blockIdx.x * rows_per_cta + sub_row; base < n;
       base += stride * kGatherUnroll) {
    uint4 kv[kGatherUnroll], vv[kGatherUnroll];
    int64_t idx[kGatherUnroll];
    bool ok_row[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      idx[u] = base + u * stride;
      ok_row[u] = false;
      if (idx[u] < n) {
        const int64_t r = rows[idx[u]];
        if (r >= 0 && r < source_rows) {
          ok_row[u] = true;
          kv[u] = __ldcs(k + r * vec_per_row + col);
          vv[u] = __ldcs(v + r * vec_per_row + col);
        } else if (error_flag) {
          atomicExch(error_flag, TW_ERR_INVALID_INDEX);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      if (ok_row[u]) {
        ok[idx[u] * vec_per_row + col] = kv[u];
        ov[idx[u] * vec_per_row + col] = vv[u];
      }
    }
  }
}

// Group offsets in the flat layout: off[g] = sum_{g' < g} (count[g'] + 1).
constexpr int kMaxGroups = 64;

// Rows of the union layout: group g occupies [off[g], off[g] + count[g] + 1);
// its last row is the current token.
// Row-0 address of entry e: from the entry directory when given, else the slab.
__device__ __forceinline__ void entry_rows(const uint4* slab_k, const uint4* slab_v,
                                           const unsigned long long* dirs, int64_t n_entries,
                                           int64_t max_len, int64_t e, int vec,
                                           const uint4*& kb, const uint4*& vb) {
  if (dirs) {
    kb = reinterpret_cast<const uint4*>(dirs[e]);
    vb = reinterpret_cast<const uint4*>(dirs[n_entries + e]);
  } else {
    kb = slab_k + e * max_len * vec;
    vb = slab_v + e * max_len * vec;
  }
}

// Previous-token row reuse for the union gather: a direct-addressed row map
// per group ((tag << 32) | row per position) points into the previous step's
// kept rows; this gather keeps its own output rows and records them with
// next_tag.  row_map == nullptr: no reuse.
struct GatherReuse {
  unsigned long long* row_map;
  int64_t map_stride;
  unsigned prev_tag;
  unsigned next_tag;
  const uint4* k;
  const uint4* v;
  int64_t prev_rows;
  int32_t* row_counts;
  // Previous row of position p of group g, or -1; lane 0 of the 16-lane row
  // group reads the entry and broadcasts it.
  __device__ __forceinline__ int64_t row_of(int g, int64_t p) const {
    const unsigned half_mask = 0xffffu << (threadIdx.x & 16);
    unsigned long long e = 0;
    if ((threadIdx.x & 15) == 0) e = row_map[(int64_t)g * map_stride + p];
    e = __shfl_sync(half_mask, e, 0, 16);
    const int64_t row = (int64_t)(e & 0xffffffffull);
    return (prev_tag != 0 && (unsigned)(e >> 32) == prev_tag && row < prev_rows) ? row : -1;
  }
};

template <int kVec>
__global__ void __launch_bounds__(kGatherThreads)
gather_union_kernel(const uint4* __restrict__ slab_k, const uint4* __restrict__ slab_v,
                    const unsigned long long* __restrict__ dirs, int64_t n_entries,
                    int64_t max_len, int first_entry, int groups, int64_t old_length,
                    const int32_t* __restrict__ union_pos, int64_t pos_stride,
                    const int32_t* __restrict__ union_count, const uint4* __restrict__ cur_k,
                    const uint4* __restrict__ cur_v, uint4* __restrict__ out_k,
                    uint4* __restrict__ out_v, int64_t rows_cap, int32_t* __restrict__ cu_seqlens,
                    int32_t* error_flag, GatherReuse prev) {
  static_assert(kVec == 16, "a row is one 16-lane half-warp");
  pdl_wait();
  pdl_launch_dependents();
  __shared__ int64_t off[kMaxGroups + 1];
  __shared__ int s_hits[kMaxGroups], s_misses[kMaxGroups];
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int g = 0; g < groups; ++g) {
      off[g] = acc;
      acc += (int64_t)union_count[g] + 1;
    }
    off[groups] = acc;
    if (blockIdx.x == 0) {
      for (int g = 0; g <= groups; ++g) cu_seqlens[g] = (int32_t)off[g];
      if (acc > rows_cap && error_flag) atomicExch(error_flag, TW_ERR_CAPACITY);
    }
  }
  if (threadIdx.x < kMaxGroups) {
    s_hits[threadIdx.x] = 0;
    s_misses[threadIdx.x] = 0;
  }
  __syncthreads();
  const int64_t total = min(off[groups], rows_cap);
  constexpr int rows_per_cta = kGatherThreads / kVec;
  const int sub_row = threadIdx.x / kVec;
  const int col = threadIdx.x % kVec;
  const int64_t stride = (int64_t)gridDim.x * rows_per_cta;
  for (int64_t base = (int64_t)blockIdx.x * rows_per_cta + sub_row; base < total;
       base += stride * kGatherUnroll) {
    uint4 kv[kGatherUnroll], vv[kGatherUnroll];
    int64_t t[kGatherUnroll], tpos[kGatherUnroll];
    int tg[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      t[u] = base + u * stride;
      tpos[u] = -1;
      if (t[u] >= total) continue;
      int g = 0;
      while (g + 1 < groups && off[g + 1] <= t[u]) ++g;
      tg[u] = g;
      const int64_t i = t[u] - off[g];
      const int32_t cnt = union_count[g];
      if (i < cnt) {
        const int64_t pos = union_pos[(int64_t)g * pos_stride + i];
        if (pos < 0 || pos >= old_length) {
          if (error_flag) atomicExch(error_flag, TW_ERR_INVALID_INDEX);
          kv[u] = make_uint4(0, 0, 0, 0);
          vv[u] = kv[u];
        } else {
          tpos[u] = pos;
          const int64_t j = prev.row_map ? prev.row_of(g, pos) : -1;
          if (j >= 0) {
            kv[u] = __ldcs(prev.k + j * kVec + col);
            vv[u] = __ldcs(prev.v + j * kVec + col);
            if (col == 0 && prev.row_counts) atomicAdd(&s_hits[g], 1);
          } else {
            const uint4 *kb, *vb;
            entry_rows(slab_k, slab_v, dirs, n_entries, max_len, (int64_t)first_entry + g, kVec,
                       kb, vb);
            kv[u] = __ldcs(kb + pos * kVec + col);
            vv[u] = __ldcs(vb + pos * kVec + col);
            if (col == 0 && prev.row_counts) atomicAdd(&s_misses[g], 1);
          }
        }
      } else {
        tpos[u] = old_length;
        kv[u] = cur_k[(int64_t)g * kVec + col];
        vv[u] = cur_v[(int64_t)g * kVec + col];
      }
    }
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      if (t[u] >= total) continue;
      out_k[t[u] * kVec + col] = kv[u];
      out_v[t[u] * kVec + col] = vv[u];
      if (prev.row_map && col == 0 && tpos[u] >= 0)
        prev.row_map[(int64_t)tg[u] * prev.map_stride + tpos[u]] =
            ((unsigned long long)prev.next_tag << 32) | (unsigned long long)t[u];
    }
  }
  if (prev.row_counts) {
    __syncthreads();
    if (threadIdx.x < groups && (s_hits[threadIdx.x] | s_misses[threadIdx.x])) {
      atomicAdd(&prev.row_counts[2 * threadIdx.x], s_hits[threadIdx.x]);
      atomicAdd(&prev.row_counts[2 * threadIdx.x + 1], s_misses[threadIdx.x]);
    }
  }
}

// Quest per-query-head layout: segment s = g*R + r has seg_len rows:
// [0, sink_end) then the k pages' rows then [recent_start, old_length) then the
// current token of group g.  The R heads of a group share their sink and
// recent rows and many of their pages, so each distinct source row is read
// over the host link once per group and written to every segment holding it.
// One warp per work item of a group (two rows per 16-byte load, 16 rows in
// flight per warp):
//  - page slot (r, j), item r*k + j: the warp reads the group's R*k page ids
//    and owns the page when no earlier slot names it; the owner loads the
//    page's rows once and writes them to every slot naming it (pages in any
//    order, repeats included);
//  - a chunk of 16 protected rows (the sink rows, then the recent window):
//    loaded once, written to the R segments;
//  - the current token: written to the R segments.
// A group with more than kQuestShareMax page slots does not share pages (each
// slot loads its own).  A page id < 0 or a row at or beyond old_length sets
// TW_ERR_INVALID_INDEX and writes zeros.
constexpr int kQuestShareMax = 1024;
constexpr int kQuestWarps = kGatherThreads / 32;

template <int kVec>
__global__ void __launch_bounds__(kGatherThreads)
gather_quest_kernel(const uint4* __restrict__ slab_k, const uint4* __restrict__ slab_v,
                    const unsigned long long* __restrict__ dirs, int64_t n_entries,
                    int64_t max_len, int first_entry, int groups, int R, int64_t old_length,
                    int64_t sink_end, int64_t recent_start, int sink, int block,
                    const int32_t* __restrict__ pages, int k_pages,
                    const uint4* __restrict__ cur_k, const uint4* __restrict__ cur_v,
                    uint4* __restrict__ out_k, uint4* __restrict__ out_v, int64_t seg_len,
                    int32_t* error_flag) {
  static_assert(kVec == 16, "a half-warp moves one row per load");
  constexpr int kPairs = 8;  // row pairs in flight per warp
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;
  const int l16 = lane & 15;
  const int64_t sel = (int64_t)k_pages * block;
  const int64_t n_prot = sink_end + (old_length - recent_start);
  const int64_t n_chunks = (n_prot + 2 * kPairs - 1) / (2 * kPairs);
  const int64_t slots = (int64_t)R * k_pages;
  const int64_t per_group = slots + n_chunks + 1;
  const int64_t item = (int64_t)blockIdx.x * kQuestWarps + (threadIdx.x >> 5);
  if (item >= per_group * groups) return;
  const int g = (int)(item / per_group);
  const int64_t w = item - (int64_t)g * per_group;
  const int64_t seg0 = (int64_t)g * R;
  const uint4 *kb, *vb;
  entry_rows(slab_k, slab_v, dirs, n_entries, max_len, (int64_t)first_entry + g, kVec, kb, vb);

  if (w == per_group - 1) {  // the current token
    const uint4 ck = cur_k[(int64_t)g * kVec + l16];
    const uint4 cv = cur_v[(int64_t)g * kVec + l16];
    for (int r = half; r < R; r += 2) {
      const int64_t t = (seg0 + r) * seg_len + seg_len - 1;
      out_k[t * kVec + l16] = ck;
      out_v[t * kVec + l16] = cv;
    }
    return;
  }
  uint4 kv[kPairs], vv[kPairs];
  if (w >= slots) {  // protected rows: chunk c covers protected rows [16c, 16c + 16)
    const int64_t t0 = (w - slots) * 2 * kPairs;
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
      const int64_t t = t0 + 2 * q + half;
      if (t < n_prot) {
        const int64_t pos = t < sink_end ? t : recent_start + (t - sink_end);
        kv[q] = __ldcs(kb + pos * kVec + l16);
        vv[q] = __ldcs(vb + pos * kVec + l16);
      }
    }
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int q = 0; q < kPairs; ++q) {
        const int64_t t = t0 + 2 * q + half;
        if (t < n_prot) {
          const int64_t i = t < sink_end ? t : t + sel;
          const int64_t o = ((seg0 + r) * seg_len + i) * kVec + l16;
          out_k[o] = kv[q];
          out_v[o] = vv[q];
        }
      }
    }
    return;
  }

  // page slot w = (r, j) of the group
  const int32_t* gp = pages + seg0 * k_pages;
  const int32_t page = gp[w];
  const bool share = slots <= kQuestShareMax;
  if (share) {
    for (int64_t f0 = 0; f0 < w; f0 += 32) {  // an earlier slot naming the page owns it
      const int64_t f = f0 + lane;
      if (__any_sync(0xffffffffu, f < w && gp[f] == page)) return;
    }
  }
  const int64_t pos0 = (int64_t)sink + (int64_t)page * block;
  for (int b0 = 0; b0 < block; b0 += 2 * kPairs) {
    bool bad = false;
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
      const int row = b0 + 2 * q + half;
      kv[q] = make_uint4(0, 0, 0, 0);
      vv[q] = kv[q];
      if (row < block) {
        const int64_t pos = pos0 + row;
        if (page >= 0 && pos < old_length) {
          kv[q] = __ldcs(kb + pos * kVec + l16);
          vv[q] = __ldcs(vb + pos * kVec + l16);
        } else {
          bad = true;
        }
      }
    }
    if (bad && error_flag) atomicExch(error_flag, TW_ERR_INVALID_INDEX);
    // every slot from w on naming the page (w itself included)
    for (int64_t f0 = share ? w : 0; f0 < (share ? slots : 1); f0 += 32) {
      const int64_t f = f0 + lane;
      unsigned m = share ? __ballot_sync(0xffffffffu, f < slots && gp[f] == page) : 1u;
      while (m) {
        const int bit = __ffs(m) - 1;
        m &= m - 1;
        const int64_t ff = share ? f0 + bit : w;
        const int64_t rr = ff / k_pages;
        const int64_t jj = ff - rr * k_pages;
        const int64_t base = (seg0 + rr) * seg_len + sink_end + jj * block + b0;
#pragma unroll
        for (int q = 0; q < kPairs; ++q) {
          const int row = 2 * q + half;
          if (b0 + row < block) {
            const int64_t o = (base + row) * kVec + l16;
            out_k[o] = kv[q];
            out_v[o] = vv[q];
          }
        }
      }
    }
  }
}

int gather_grid(int64_t rows, int rows_per_cta) {
  static int sm_cache[kMaxDevices];
  int sms = 148;
  if (cached_device_attribute(cudaDevAttrMultiProcessorCount, sm_cache, sms) != TW_OK) sms = 148;
  const int64_t want = (rows + (int64_t)rows_per_cta * kGatherUnroll - 1) /
                       ((int64_t)rows_per_cta * kGatherUnroll);
  const int64_t cap = (int64_t)sms * 8;
  const int64_t g = want < cap ? want : cap;
  return (int)(g < 1 ? 1 : g);
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

}  // namespace tw

using namespace tw;

extern "C" int tw_gather_kv(const void* k, const void* v, void* out_k, void* out_v,
                            const int64_t* rows, int64_t n, int64_t source_rows,
                            int64_t row_bytes, int32_t* error_flag, void* stream) {
  if (n < 0 || source_rows < 0 || row_bytes <= 0 || (row_bytes % 16) != 0 ||
      row_bytes / 16 > kGatherThreads)
    return TW_ERR_BAD_ARG;
  if (n == 0) return TW_OK;
  if (!k || !v || !out_k || !out_v || !rows) return TW_ERR_BAD_ARG;
  if (!aligned16(k) || !aligned16(v) || !aligned16(out_k) || !aligned16(out_v))
    return TW_ERR_BAD_ARG;
  const int vec = (int)(row_bytes / 16);
  const int grid = gather_grid(n, kGatherThreads / vec);
  gather_kv_kernel<<<grid, kGatherThreads, 0, (cudaStream_t)stream>>>(
      (const uint4*)k, (const uint4*)v, (uint4*)out_k, (uint4*)out_v, rows, n, source_rows, vec,
      error_flag);
  return check_launch();
}

extern "C" int tw_gather_union(const void* slab_k, const void* slab_v,
                               const uint64_t* entry_dirs, int64_t n_entries, int64_t max_len,
                               int first_entry, int groups, int64_t old_length,
                               const int32_t* union_pos, int64_t pos_stride,
                               const int32_t* union_count, const void* cur_k, const void* cur_v,
                               int head_dim, int dtype, void* out_k, void* out_v,
                               int64_t rows_cap, int32_t* cu_seqlens, int32_t* error_flag,
                               const tw_row_reuse* reuse, void* stream) {
  if (head_dim != kHeadDim || (dtype != TW_F16 && dtype != TW_BF16)) return TW_ERR_UNSUPPORTED;
  if ((!entry_dirs && (!slab_k || !slab_v)) || !union_pos || !union_count || !cur_k || !cur_v ||
      !out_k || !out_v || !cu_seqlens || groups <= 0 || groups > kMaxGroups || first_entry < 0 ||
      old_length < 0 || old_length > max_len || rows_cap <= 0 ||
      (entry_dirs && first_entry + groups > n_entries))
    return TW_ERR_BAD_ARG;
  if (!aligned16(slab_k) || !aligned16(slab_v) || !aligned16(cur_k) || !aligned16(cur_v) ||
      !aligned16(out_k) || !aligned16(out_v))
    return TW_ERR_BAD_ARG;
  GatherReuse prev{nullptr, 0, 0u, 0u, nullptr, nullptr, 0, nullptr};
  if (reuse) {
    // the kept rows are out_k / out_v themselves (packed)
    const size_t out_bytes = (size_t)rows_cap * kHeadDim * 2;
    const size_t prev_bytes = (size_t)reuse->prev_rows * kHeadDim * 2;
    auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
      const char* x = (const char*)a;
      const char* y = (const char*)b;
      return x < y + nb && y < x + na;
    };
    if (reuse->next_k || reuse->next_v || !reuse->row_map || reuse->map_stride <= old_length ||
        reuse->next_tag == 0 || reuse->next_tag == reuse->prev_tag || rows_cap > 0xffffffffll)
      return TW_ERR_BAD_ARG;
    if (reuse->prev_tag != 0 &&
        (!reuse->prev_k || !reuse->prev_v || reuse->prev_rows <= 0 ||
         !aligned16(reuse->prev_k) || !aligned16(reuse->prev_v) ||
         overlap(reuse->prev_k, prev_bytes, out_k, out_bytes) ||
         overlap(reuse->prev_k, prev_bytes, out_v, out_bytes) ||
         overlap(reuse->prev_v, prev_bytes, out_k, out_bytes) ||
         overlap(reuse->prev_v, prev_bytes, out_v, out_bytes)))
      return TW_ERR_BAD_ARG;
    prev.row_map = (unsigned long long*)reuse->row_map;
    prev.map_stride = reuse->map_stride;
    prev.prev_tag = reuse->prev_tag;
    prev.next_tag = reuse->next_tag;
    prev.k = (const uint4*)reuse->prev_k;
    prev.v = (const uint4*)reuse->prev_v;
    prev.prev_rows = reuse->prev_tag != 0 ? reuse->prev_rows : 0;
    prev.row_counts = reuse->row_counts;
  }
  constexpr int kVec = kHeadDim * 2 / 16;  // 16 vectors per 256-byte row
  const int grid = gather_grid(rows_cap, kGatherThreads / kVec);
  return launch_pdl(gather_union_kernel<kVec>, dim3(grid), dim3(kGatherThreads), 0,
                    (cudaStream_t)stream, (const uint4*)slab_k, (const uint4*)slab_v,
                    (const unsigned long long*)entry_dirs, n_entries, max_len, first_entry, groups,
                    old_length, union_pos, pos_stride, union_count, (const uint4*)cur_k,
                    (const uint4*)cur_v, (uint4*)out_k, (uint4*)out_v, rows_cap, cu_seqlens,
                    error_flag, prev);
}

extern "C" int tw_gather_quest_heads(const void* slab_k, const void* slab_v,
                                     const uint64_t* entry_dirs, int64_t n_entries,
                                     int64_t max_len, int first_entry, int groups,
                                     int heads_per_group,
                                     int64_t old_length, int64_t sink_end, int64_t recent_start,
                                     int sink, int block_size, const int32_t* pages, int k_pages,
                                     const void* cur_k, const void* cur_v, int head_dim,
                                     int dtype, void* out_k, void* out_v, int32_t* error_flag,
                                     void* stream) {
  if (head_dim != kHeadDim || (dtype != TW_F16 && dtype != TW_BF16)) return TW_ERR_UNSUPPORTED;
  if ((!entry_dirs && (!slab_k || !slab_v)) || !cur_k || !cur_v || !out_k || !out_v ||
      groups <= 0 || heads_per_group <= 0 || first_entry < 0 || old_length < 0 ||
      old_length > max_len || (entry_dirs && first_entry + groups > n_entries) ||
      sink_end < 0 || sink_end > old_length || recent_start < sink_end ||
      recent_start > old_length || k_pages < 0 || (k_pages > 0 && !pages) || block_size <= 0)
    return TW_ERR_BAD_ARG;
  if (!aligned16(slab_k) || !aligned16(slab_v) || !aligned16(cur_k) || !aligned16(cur_v) ||
      !aligned16(out_k) || !aligned16(out_v))
    return TW_ERR_BAD_ARG;
  const int64_t seg_len =
      sink_end + (int64_t)k_pages * block_size + (old_length - recent_start) + 1;
  constexpr int kVec = kHeadDim * 2 / 16;
  const int64_t n_prot = sink_end + (old_length - recent_start);
  const int64_t per_group = (int64_t)heads_per_group * k_pages + (n_prot + 15) / 16 + 1;
  const int64_t items = per_group * groups;
  const int64_t grid = (items + kQuestWarps - 1) / kQuestWarps;
  if (grid > 0x7fffffffLL) return TW_ERR_UNSUPPORTED;
  gather_quest_kernel<kVec><<<(unsigned)grid, kGatherThreads, 0, (cudaStream_t)stream>>>(
      (const uint4*)slab_k, (const uint4*)slab_v, (const unsigned long long*)entry_dirs, n_entries,
      max_len, first_entry, groups, heads_per_group, old_length, sink_end, recent_start, sink,
      block_size, pages, k_pages, (const uint4*)cur_k, (const uint4*)cur_v, (uint4*)out_k,
      (uint4*)out_v, seg_len, error_flag);
  return check_launch();
}
