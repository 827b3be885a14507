// New-token append, shared by the append kernel (int4.cu) and the selection
// launch, which runs it in its extra cluster (topp_union.cu): the token's K / V
// row to the slab, its running Quest page min / max, its INT4 code.
// Reference: the new-KV write-back (hi/quest_offload_cache.py:230-274,
// hi/twilight_offload_cache.py:551-794) and the prefill-only metadata
// (hi/quest_offload_cache.py:276-289, hi/twilight_offload_cache.py:925-936),
// extended to appended tokens.
#pragma once

#include "tw_common.cuh"

namespace tw {

// Rounding of the `/ 15.0` in affine_int4_pack.  torch on CUDA multiplies by
// the fp32 reciprocal of a CPU-scalar divisor; torch on CPU divides.
enum ScaleDiv : int { kScaleReciprocal = 0, kScaleDivide = 1 };

// Quantise the 4 channels 4*lane .. 4*lane+3 of one row held by a warp.
// group_size in {32, 64, 128}: lanes 0..31 split into groups of group_size/4.
// Returns the two packed bytes for this lane (low byte = channels 0,1).
template <typename T>
__device__ __forceinline__ uint16_t quantize_lane(const T (&raw)[4], int group_size, int scale_div,
                                                  T* scale_out, T* min_out) {
  const int lanes_per_group = group_size >> 2;
  float x[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = to_f32(raw[i]);
  float mn = fminf(fminf(x[0], x[1]), fminf(x[2], x[3]));
  float mx = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
  for (int off = 1; off < lanes_per_group; off <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  // (maximum - minimum) is computed in the K dtype, then widened.
  const float diff = to_f32(from_f32<T>(__fsub_rn(mx, mn)));
  const float clamped = fmaxf(diff, 1e-9f);
  const float sc32 = scale_div == kScaleDivide ? __fdiv_rn(clamped, 15.0f)
                                               : __fmul_rn(clamped, __fdiv_rn(1.0f, 15.0f));
  const T sc_t = from_f32<T>(sc32);
  const float sc = to_f32(sc_t);
  const T mn_t = from_f32<T>(mn);  // exact: mn is a K-dtype value
  uint32_t codes[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float c = rintf(__fdiv_rn(__fsub_rn(x[i], mn), sc));
    if (!(c >= 0.0f)) c = 0.0f;  // negatives and NaN (0/0) -> 0, as clamp + uint8 cast
    if (c > 15.0f) c = 15.0f;
    codes[i] = (uint32_t)c;
  }
  if ((threadIdx.x & (lanes_per_group - 1)) == 0) {
    *scale_out = sc_t;
    *min_out = mn_t;
  }
  return (uint16_t)((codes[0] | (codes[1] << 4)) | ((codes[2] | (codes[3] << 4)) << 8));
}

struct AppendArgs {
  uint4* slab_k;                    // K / V planes of the slab (dirs null), or null
  uint4* slab_v;
  const unsigned long long* dirs;   // [2][n_entries] row-0 addresses, or null
  int64_t n_entries;
  int64_t max_len;
  int first_entry;
  int64_t position;                 // the token's position (old_length)
  const void* cur_k;                // [G][D] new rows, K dtype
  const void* cur_v;
  int sink;
  int block;
  void* pmin;                       // page min / max of entry 0 (null: skipped)
  void* pmax;
  int64_t meta_entry_stride;        // elements between entries' page arrays
  uint8_t* packed;                  // INT4 codes / scale / min of entry 0 (null: skipped)
  void* scale;
  void* minimum;
  int group_size;
  int scale_div;
};

// The argument checks of tw_append_token (TW_OK or an error status).
inline int check_append_args(const void* slab_k, const void* slab_v, const uint64_t* dirs,
                             int64_t n_entries, int64_t max_len, int first_entry, int groups,
                             int64_t position, const void* cur_k, const void* cur_v, int sink,
                             int block, const void* pmin, const void* pmax, const uint8_t* packed,
                             const void* scale, const void* minimum, int group_size) {
  if (!cur_k || !cur_v || groups <= 0 || first_entry < 0 || position < 0 ||
      position >= max_len || block <= 0 || sink < 0)
    return TW_ERR_BAD_ARG;
  if ((slab_k == nullptr) != (slab_v == nullptr)) return TW_ERR_BAD_ARG;
  if (dirs && first_entry + groups > n_entries) return TW_ERR_BAD_ARG;
  if ((pmin == nullptr) != (pmax == nullptr)) return TW_ERR_BAD_ARG;
  if (packed != nullptr && (!scale || !minimum ||
                            (group_size != 32 && group_size != 64 && group_size != 128)))
    return TW_ERR_BAD_ARG;
  if ((slab_k && ((uintptr_t)slab_k & 15)) || ((uintptr_t)cur_k & 15) || ((uintptr_t)cur_v & 15))
    return TW_ERR_BAD_ARG;
  return TW_OK;
}

inline AppendArgs make_append_args(void* slab_k, void* slab_v, const uint64_t* dirs,
                                   int64_t n_entries, int64_t max_len, int first_entry,
                                   int64_t position, const void* cur_k, const void* cur_v,
                                   int sink, int block, void* pmin, void* pmax,
                                   int64_t meta_entry_stride, uint8_t* packed, void* scale,
                                   void* minimum, int group_size) {
  AppendArgs a{};
  a.slab_k = (uint4*)slab_k;
  a.slab_v = (uint4*)slab_v;
  a.dirs = (const unsigned long long*)dirs;
  a.n_entries = n_entries;
  a.max_len = max_len;
  a.first_entry = first_entry;
  a.position = position;
  a.cur_k = cur_k;
  a.cur_v = cur_v;
  a.sink = sink;
  a.block = block;
  a.pmin = pmin;
  a.pmax = pmax;
  a.meta_entry_stride = meta_entry_stride;
  a.packed = packed;
  a.scale = scale;
  a.minimum = minimum;
  a.group_size = packed ? group_size : 128;
  a.scale_div = kScaleReciprocal;
  return a;
}

// Group g's append by its 128 threads d = 0..127 (four whole warps, d = 0..31
// being the first): the row to the slab, the element d of the running page
// min / max, and the INT4 code by the first warp.
template <typename T>
__device__ __forceinline__ void append_token_row(const AppendArgs& a, int g, int d) {
  const int entry = a.first_entry + g;
  const T* krow = reinterpret_cast<const T*>(a.cur_k) + (int64_t)g * kHeadDim;
  const T* vrow = reinterpret_cast<const T*>(a.cur_v) + (int64_t)g * kHeadDim;
  constexpr int kVecPerRow = kHeadDim * sizeof(T) / 16;
  if (a.slab_k != nullptr || a.dirs != nullptr) {
    uint4* kb = a.dirs ? reinterpret_cast<uint4*>(a.dirs[entry])
                       : a.slab_k + (int64_t)entry * a.max_len * kVecPerRow;
    uint4* vb = a.dirs ? reinterpret_cast<uint4*>(a.dirs[a.n_entries + entry])
                       : a.slab_v + (int64_t)entry * a.max_len * kVecPerRow;
    if (d < kVecPerRow) {
      kb[a.position * kVecPerRow + d] = reinterpret_cast<const uint4*>(krow)[d];
    } else if (d < 2 * kVecPerRow) {
      const int j = d - kVecPerRow;
      vb[a.position * kVecPerRow + j] = reinterpret_cast<const uint4*>(vrow)[j];
    }
  }
  if (a.pmin != nullptr && a.position >= a.sink) {
    T* pmin = reinterpret_cast<T*>(a.pmin);
    T* pmax = reinterpret_cast<T*>(a.pmax);
    const int64_t rel = a.position - a.sink;
    const int64_t page = rel / a.block;
    const int64_t off = rel % a.block;
    const int64_t idx = (int64_t)entry * a.meta_entry_stride + page * kHeadDim + d;
    const T x = krow[d];
    if (off == 0) {
      pmin[idx] = x;
      pmax[idx] = x;
    } else {
      const float fx = to_f32(x);
      if (fx < to_f32(pmin[idx])) pmin[idx] = x;
      if (fx > to_f32(pmax[idx])) pmax[idx] = x;
    }
  }
  if (a.packed != nullptr && d < 32) {
    const int lane = d;
    T raw[4];
    const uint2 v = *reinterpret_cast<const uint2*>(krow + 4 * lane);
    memcpy(raw, &v, sizeof(v));
    const int ngroups = kHeadDim / a.group_size;
    const int64_t orow = (int64_t)entry * a.max_len + a.position;
    const int grp = (4 * lane) / a.group_size;
    T* scale = reinterpret_cast<T*>(a.scale);
    T* minimum = reinterpret_cast<T*>(a.minimum);
    const uint16_t bytes = quantize_lane<T>(raw, a.group_size, a.scale_div,
                                            scale + orow * ngroups + grp,
                                            minimum + orow * ngroups + grp);
    reinterpret_cast<uint16_t*>(a.packed + orow * (kHeadDim / 2))[lane] = bytes;
  }
}

}  // namespace tw
