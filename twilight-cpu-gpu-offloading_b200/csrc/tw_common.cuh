// Shared device helpers for the sm_100a sparse decode-attention kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <mutex>
#include <utility>

#include "../../include/twilight_b200.h"

namespace tw {

constexpr int kHeadDim = 128;          // the only head_dim the path supports
constexpr int kMaxHeadsPerGroup = 8;   // R <= 8 (one cluster of R CTAs per group)

// Thread-local record of the last CUDA error (tw_last_cuda_error).
void set_last_cuda_error(cudaError_t err);

inline int check_launch() {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

// Launch-time state kept per device so that the per-call path makes no
// attribute queries: the dynamic shared memory a kernel has been opted into,
// and device attributes read once.
constexpr int kMaxDevices = 64;

struct DynSmemOptIn {
  std::mutex mu;
  int bytes[kMaxDevices] = {};
};

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) only when this launch needs
// more than the function was opted into on the current device.
inline int ensure_dyn_smem(const void* func, DynSmemOptIn& st, int bytes) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    std::lock_guard<std::mutex> lk(st.mu);
    if (st.bytes[dev] >= bytes) return TW_OK;
    err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (err == cudaSuccess) st.bytes[dev] = bytes;
  } else if (err == cudaSuccess) {
    err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  }
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

// Device attribute `attr` of the current device, queried once per device.
inline int cached_device_attribute(cudaDeviceAttr attr, int (&cache)[kMaxDevices], int& value) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err == cudaSuccess && dev >= 0 && dev < kMaxDevices && cache[dev] > 0) {
    value = cache[dev];
    return TW_OK;
  }
  if (err == cudaSuccess) err = cudaDeviceGetAttribute(&value, attr, dev);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  if (dev >= 0 && dev < kMaxDevices) cache[dev] = value;  // benign race: same value
  return TW_OK;
}

// Programmatic dependent launch.  The decode-path kernels are launched with
// launch_pdl, so each may be scheduled while the previous kernel of the stream
// is still running; every such kernel calls pdl_wait() before its first
// global memory access (the wait returns once the previous grid has completed
// and its writes are visible; without a programmatic predecessor it returns at
// once), then pdl_launch_dependents() so that the next kernel can be
// scheduled early.  Launch gaps between the kernels of a layer-step vanish.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return check_launch();
}

// Protected rows of a layer-step staged in device memory.  Every group's union
// holds its sink rows [0, n_sink) and its recent window [recent_start,
// old_length); neither depends on the selection.  The selection launch copies
// them from the slab (or the entry directory's rows) into stage_k / stage_v
// [G][stage_rows][D] while its other clusters select, so the host link carries
// them while it would otherwise idle, and the attention reads them from device
// memory.  Staged row j of group g: position j (j < n_sink), else position
// recent_start + j - n_sink.  stage_k == nullptr: nothing is staged.
struct ProtectedStage {
  const uint4* slab_k;              // K plane of the slab (dirs == nullptr)
  const uint4* slab_v;
  const unsigned long long* dirs;   // [2][n_entries] row-0 addresses, or null
  int64_t n_entries;
  int64_t max_len;
  int first_entry;
  uint4* stage_k;
  uint4* stage_v;
  int64_t stage_rows;               // >= n_sink + (old_length - recent_start)
  int64_t n_sink;
  int64_t recent_start;
  int64_t old_length;
};

constexpr int kVecPerRow16 = 16;  // 16-byte vectors per 128-dim fp16 / bf16 row

// The staged index of position pos, or -1 when pos is not a protected row.
__device__ __forceinline__ int64_t stage_index(const ProtectedStage& s, int64_t pos) {
  if (pos < s.n_sink) return pos;
  if (pos >= s.recent_start) return s.n_sink + (pos - s.recent_start);
  return -1;
}

// Copies the protected rows of `groups` groups (K and V) into the stage; the
// calling CTAs are `ctas` CTAs of blockDim.x threads, this one being number
// `cta`.  Each thread keeps 4 rows' vectors of K and V in flight.
__device__ __forceinline__ void stage_protected_rows(const ProtectedStage& s, int groups, int cta,
                                                     int ctas) {
  const int64_t rows = s.n_sink + (s.old_length - s.recent_start);
  const int64_t total = (int64_t)groups * rows * kVecPerRow16;
  const int64_t nthreads = (int64_t)ctas * blockDim.x;
  constexpr int kInFlight = 4;
  for (int64_t base = (int64_t)cta * blockDim.x + threadIdx.x; base < total;
       base += nthreads * kInFlight) {
    uint4 kv[kInFlight], vv[kInFlight];
    int64_t dst[kInFlight];
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      const int64_t v = base + u * nthreads;
      dst[u] = -1;
      if (v < total) {
        const int64_t row = v / kVecPerRow16;  // g * rows + j
        const int l16 = (int)(v % kVecPerRow16);
        const int64_t g = row / rows;
        const int64_t j = row - g * rows;
        const int64_t pos = j < s.n_sink ? j : s.recent_start + (j - s.n_sink);
        const int64_t e = (int64_t)s.first_entry + g;
        const uint4* kp;
        const uint4* vp;
        if (s.dirs) {
          kp = reinterpret_cast<const uint4*>(s.dirs[e]) + pos * kVecPerRow16;
          vp = reinterpret_cast<const uint4*>(s.dirs[s.n_entries + e]) + pos * kVecPerRow16;
        } else {
          kp = s.slab_k + (e * s.max_len + pos) * kVecPerRow16;
          vp = s.slab_v + (e * s.max_len + pos) * kVecPerRow16;
        }
        kv[u] = __ldcs(kp + l16);
        vv[u] = __ldcs(vp + l16);
        dst[u] = (g * s.stage_rows + j) * kVecPerRow16 + l16;
      }
    }
#pragma unroll
    for (int u = 0; u < kInFlight; ++u) {
      if (dst[u] >= 0) {
        s.stage_k[dst[u]] = kv[u];
        s.stage_v[dst[u]] = vv[u];
      }
    }
  }
}

// Bulk prefetch of the 16-byte granules covering [p, p + bytes) into L2, in
// pieces of at most 64 KB (one instruction each; no data is returned).
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
  if (bytes == 0) return;
  uintptr_t a = (uintptr_t)p & ~(uintptr_t)15;
  const uintptr_t e = ((uintptr_t)p + bytes + 15) & ~(uintptr_t)15;
  while (a < e) {
    const uint32_t n = (uint32_t)((e - a) < 65536 ? (e - a) : 65536);
    asm volatile(
        "{\n\t.reg .u64 ga;\n\tcvta.to.global.u64 ga, %0;\n\t"
        "cp.async.bulk.prefetch.L2.global [ga], %1;\n\t}" ::"l"(a),
        "r"(n)
        : "memory");
    a += n;
  }
}

// 8 fp16 / bf16 values of a 16-byte vector as floats.
template <typename T> __device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]);
template <> __device__ __forceinline__ void unpack8<__half>(const uint4& u, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <> __device__ __forceinline__ void unpack8<__nv_bfloat16>(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }

// Order-preserving map of an fp32 value to uint32 (larger float -> larger key).
// -0.0 is folded onto +0.0 so that equal values compare equal, as in torch.topk.
__device__ __forceinline__ uint32_t float_key(float f) {
  if (f == 0.0f) f = 0.0f;
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// Deterministic e^x for x <= 0 in IEEE double, written from the Taylor series
// of e^r on |r| <= ln2/2 after the reduction x = k*ln2 + r.  Every operation is
// an explicitly rounded add or multiply, so the same sequence in the C oracle
// (compiled without contraction) gives bit-identical results.
// Inputs below -700 return 0 (their fixed-point mass is 0 either way), which
// keeps 2^k a normal double built from its bit pattern.
__device__ __forceinline__ double det_exp(double x) {
  if (!(x >= -700.0)) return 0.0;
  const double log2e = 1.4426950408889634;   // log2(e)
  const double ln2 = 0.6931471805599453;     // ln(2)
  double t = __dmul_rn(x, log2e);
  double k = floor(__dadd_rn(t, 0.5));
  double r = __dadd_rn(x, -__dmul_rn(k, ln2));
  // Horner on 1/n!, n = 0..13
  double p = 1.0 / 6227020800.0;                 // 1/13!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 479001600.0);   // 1/12!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 39916800.0);    // 1/11!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 3628800.0);     // 1/10!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 362880.0);      // 1/9!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 40320.0);       // 1/8!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 5040.0);        // 1/7!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 720.0);         // 1/6!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 120.0);         // 1/5!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 24.0);          // 1/4!
  p = __dadd_rn(__dmul_rn(p, r), 1.0 / 6.0);           // 1/3!
  p = __dadd_rn(__dmul_rn(p, r), 0.5);                 // 1/2!
  p = __dadd_rn(__dmul_rn(p, r), 1.0);                 // 1/1!
  p = __dadd_rn(__dmul_rn(p, r), 1.0);                 // 1/0!
  const long long biased = (long long)k + 1023;
  const double two_k = __longlong_as_double(biased << 52);
  return __dmul_rn(p, two_k);
}

// Fixed-point softmax mass: e * 2^48 truncated.  Sums of up to 65536 masses
// fit in 64 bits and are exact, hence order-independent.
constexpr double kMassScale = 281474976710656.0;  // 2^48
__device__ __forceinline__ unsigned long long mass_of(double e) {
  return __double2ull_rz(__dmul_rn(e, kMassScale));
}

// Block-wide exclusive scan of one uint32 per thread (blockDim.x <= 1024).
// `scratch` needs 32 words.  Returns the exclusive prefix; *total gets the sum.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* scratch,
                                                         uint32_t* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  uint32_t x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = (lane < nwarps) ? scratch[lane] : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    scratch[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  uint32_t warp_base = (warp > 0) ? scratch[warp - 1] : 0u;
  *total = scratch[nwarps - 1];
  __syncthreads();
  return warp_base + x - v;
}

// 64-bit variant of block_exclusive_scan (scratch: 32 u64).
__device__ __forceinline__ unsigned long long block_exclusive_scan_u64(
    unsigned long long v, unsigned long long* scratch, unsigned long long* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  unsigned long long x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    unsigned long long y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = (lane < nwarps) ? scratch[lane] : 0ull;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      unsigned long long y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    scratch[lane] = w;
  }
  __syncthreads();
  const unsigned long long warp_base = (warp > 0) ? scratch[warp - 1] : 0ull;
  *total = scratch[nwarps - 1];
  __syncthreads();
  return warp_base + x - v;
}

// block_exclusive_scan_u64 and block_exclusive_scan of two values at once (one
// set of block barriers; scratch64 / scratch32: 32 entries each).
__device__ __forceinline__ void block_exclusive_scan_pair(
    unsigned long long v, uint32_t c, unsigned long long* scratch64, uint32_t* scratch32,
    unsigned long long* prefix, uint32_t* cprefix, unsigned long long* total,
    uint32_t* ctotal) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  unsigned long long x = v;
  uint32_t xc = c;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, x, off);
    const uint32_t yc = __shfl_up_sync(0xffffffffu, xc, off);
    if (lane >= off) {
      x += y;
      xc += yc;
    }
  }
  if (lane == 31) {
    scratch64[warp] = x;
    scratch32[warp] = xc;
  }
  __syncthreads();
  if (warp == 0) {
    unsigned long long w = (lane < nwarps) ? scratch64[lane] : 0ull;
    uint32_t wc = (lane < nwarps) ? scratch32[lane] : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const unsigned long long y = __shfl_up_sync(0xffffffffu, w, off);
      const uint32_t yc = __shfl_up_sync(0xffffffffu, wc, off);
      if (lane >= off) {
        w += y;
        wc += yc;
      }
    }
    scratch64[lane] = w;
    scratch32[lane] = wc;
  }
  __syncthreads();
  *prefix = ((warp > 0) ? scratch64[warp - 1] : 0ull) + x - v;
  *cprefix = ((warp > 0) ? scratch32[warp - 1] : 0u) + xc - c;
  *total = scratch64[nwarps - 1];
  *ctotal = scratch32[nwarps - 1];
  __syncthreads();
}

// In-place bitonic sort, descending, of n (a power of two) 64-bit keys in
// shared memory by the whole block.  The caller synchronises before the call;
// the sorted keys are visible to all threads on return.
__device__ __forceinline__ void bitonic_sort_desc(unsigned long long* s, int n) {
  for (int k = 2; k <= n; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int t = threadIdx.x; t < (n >> 1); t += blockDim.x) {
        const int i = ((t & ~(j - 1)) << 1) | (t & (j - 1));
        const int p = i | j;
        const unsigned long long a = s[i], b = s[p];
        const bool desc = (i & k) == 0;
        if (desc ? (a < b) : (a > b)) {
          s[i] = b;
          s[p] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Sort key of candidate i with order-preserving float key k: larger k first,
// then lower i first (the rank order the selection uses for ties).
__device__ __forceinline__ unsigned long long rank_key(uint32_t k, int i) {
  return ((unsigned long long)k << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i);
}
__device__ __forceinline__ int rank_index(unsigned long long rk) {
  return (int)(0xffffffffu - (uint32_t)(rk & 0xffffffffull));
}

__host__ __device__ __forceinline__ int next_pow2(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}

}  // namespace tw

#define TW_DISPATCH_KV_DTYPE(dtype, T, ...)                 \
  do {                                                      \
    if ((dtype) == TW_F16) {                                \
      using T = __half;                                     \
      __VA_ARGS__;                                          \
    } else if ((dtype) == TW_BF16) {                        \
      using T = __nv_bfloat16;                              \
      __VA_ARGS__;                                          \
    } else {                                                \
      return TW_ERR_BAD_ARG;                                \
    }                                                       \
  } while (0)
