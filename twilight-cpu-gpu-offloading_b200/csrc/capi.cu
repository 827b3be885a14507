// C ABI glue: status text, mapped host slab allocation and the whole-layer
// Twilight selection that chains the Quest and INT4/top-p kernels.
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <unordered_map>

#include "append.cuh"
#include "tw_common.cuh"

namespace tw {

static thread_local int g_last_cuda_error = 0;

void set_last_cuda_error(cudaError_t err) { g_last_cuda_error = (int)err; }

inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace tw

using namespace tw;

// Kernel launchers defined in the other translation units.
extern "C" int tw_quest_score(const float*, const void*, const void*, int, int, int, int64_t, int,
                              int, float*, void*);
extern "C" int tw_topk_pages(const float*, int, int, int, int32_t*, void*);
extern "C" int tw_int4_qk(const float*, const uint8_t*, const void*, const void*, int64_t,
                          const int32_t*, int, int, int, int, int, int, int, int, float*, void*);
extern "C" int tw_top_p_union(const float*, const int32_t*, int, int, int, int, int, double,
                              int64_t, int64_t, int64_t, int32_t*, int64_t, int32_t*, int32_t*,
                              int32_t*, int32_t*, void*);

namespace tw {
int select_layer_fused(const void* q, int q_dtype, const void* pmin, const void* pmax,
                       int64_t meta_stride, int n_pages, const uint8_t* packed, const void* scale,
                       const void* minimum, int64_t entry_stride, int groups, int R, int b0,
                       int block, int sink, int group_size, int dtype, double top_p,
                       int64_t old_length, int64_t sink_end, int64_t recent_start,
                       int32_t* pages_out, int32_t* union_pos, int64_t pos_stride,
                       int32_t* union_count, int32_t* head_count, int32_t* head_pos,
                       int32_t* error_flag, void* workspace, size_t workspace_bytes,
                       const ProtectedStage* stage, const AppendArgs* append,
                       cudaStream_t stream);
size_t merge_region_bytes(int groups, int n_pages, int block);
int attend_union_impl(const void* slab_k, const void* slab_v, const uint64_t* entry_dirs,
                      int64_t n_entries, int64_t max_len, int first_entry, int groups,
                      int64_t old_length, const int32_t* union_pos, int64_t pos_stride,
                      const int32_t* union_count, const void* cur_k, const void* cur_v,
                      const void* q, int heads_per_group, int max_rows_per_group, int head_dim,
                      int dtype, float softmax_scale, void* out, int out_dtype, float* lse,
                      int32_t* error_flag, void* workspace, size_t workspace_bytes,
                      const tw_row_reuse* reuse, const ProtectedStage* stage,
                      cudaStream_t stream);
int quest_score_dispatch(const void* q, int q_dtype, const void* pmin, const void* pmax, int groups,
                         int R, int n_pages, int64_t stride, int dtype, float* scores,
                         cudaStream_t stream);
}  // namespace tw
int launch_int4_qk(const void* q, int q_dtype, const uint8_t* packed, const void* scale,
                   const void* minimum, int64_t entry_stride_tokens, const int32_t* pages,
                   int groups, int R, int b0_pages, int block_size, int sink, int group_size,
                   int dtype, float* logits, cudaStream_t stream);

extern "C" int tw_attend_union(const void*, const void*, const uint64_t*, int64_t, int64_t, int,
                               int, int64_t, const int32_t*, int64_t, const int32_t*, const void*,
                               const void*, const void*, int, int, int, int, float, void*, int,
                               float*, int32_t*, void*, size_t, const tw_row_reuse*, void*);
extern "C" int tw_append_token(void*, void*, const uint64_t*, int64_t, int64_t, int, int, int64_t,
                               const void*, const void*, int, int, int, int, void*, void*, int64_t,
                               uint8_t*, void*, void*, int, void*);

extern "C" const char* tw_status_string(int status) {
  switch (status) {
    case TW_OK: return "ok";
    case TW_ERR_INVALID_INDEX: return "row index out of bounds";
    case TW_ERR_BAD_ARG: return "invalid argument";
    case TW_ERR_CAPACITY: return "capacity exceeded";
    case TW_ERR_ORDER: return "strict sequential entry order violated";
    case TW_ERR_CUDA: return "CUDA error";
    case TW_ERR_TIMEOUT: return "device wait timed out";
    case TW_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    default: return "unknown status";
  }
}

extern "C" int tw_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" int tw_abi_version(void) { return 3; }

extern "C" int tw_host_alloc_mapped(size_t bytes, void** host_ptr, void** device_ptr) {
  if (!host_ptr || !device_ptr || bytes == 0) return TW_ERR_BAD_ARG;
  *host_ptr = nullptr;
  *device_ptr = nullptr;
  void* h = nullptr;
  cudaError_t err = cudaHostAlloc(&h, bytes, cudaHostAllocMapped | cudaHostAllocPortable);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  void* d = nullptr;
  err = cudaHostGetDevicePointer(&d, h, 0);
  if (err != cudaSuccess) {
    cudaFreeHost(h);
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  *host_ptr = h;
  *device_ptr = d;
  return TW_OK;
}

// ---- NUMA-placed slabs -----------------------------------------------------------------------
// Anonymous memory bound to one host NUMA node (mbind before first touch),
// then page-locked and mapped for the GPU with cudaHostRegister.  Regions are
// remembered so that tw_host_free unregisters and unmaps them.
namespace tw {
namespace {
std::mutex g_numa_mu;
std::unordered_map<void*, size_t> g_numa_regions;
constexpr long kMpolBind = 2;      // MPOL_BIND
constexpr long kMpolFNode = 1;     // MPOL_F_NODE
constexpr long kMpolFAddr = 2;     // MPOL_F_ADDR
}  // namespace
}  // namespace tw

extern "C" int tw_host_alloc_mapped_numa(size_t bytes, int numa_node, void** host_ptr,
                                         void** device_ptr, int* bound_node) {
  if (!host_ptr || !device_ptr || bytes == 0) return TW_ERR_BAD_ARG;
  *host_ptr = nullptr;
  *device_ptr = nullptr;
  if (bound_node) *bound_node = -1;
  int node = numa_node;
  if (node < 0) {
    int dev = 0, id = -1;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&id, cudaDevAttrHostNumaId, dev) == cudaSuccess)
      node = id;
    cudaGetLastError();
  }
  const size_t align = (size_t)2 << 20;
  const size_t len = (bytes + align - 1) / align * align;
  void* h = mmap(nullptr, len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
  if (h == MAP_FAILED) return TW_ERR_CAPACITY;
  madvise(h, len, MADV_HUGEPAGE);
  if (node >= 0 && node < 1024) {
    unsigned long mask[1024 / (8 * sizeof(unsigned long))] = {};
    mask[node / (8 * sizeof(unsigned long))] = 1ul << (node % (8 * sizeof(unsigned long)));
    if (syscall(SYS_mbind, h, len, kMpolBind, mask, (unsigned long)(node + 2), 0ul) == 0 &&
        bound_node)
      *bound_node = node;
  }
  cudaError_t err = cudaHostRegister(h, len, cudaHostRegisterMapped | cudaHostRegisterPortable);
  if (err != cudaSuccess) {
    munmap(h, len);
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  void* d = nullptr;
  err = cudaHostGetDevicePointer(&d, h, 0);
  if (err != cudaSuccess) {
    cudaHostUnregister(h);
    munmap(h, len);
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  {
    std::lock_guard<std::mutex> lk(g_numa_mu);
    g_numa_regions[h] = len;
  }
  *host_ptr = h;
  *device_ptr = d;
  return TW_OK;
}

extern "C" int tw_host_numa_node(const void* host_ptr, int* node) {
  if (!host_ptr || !node) return TW_ERR_BAD_ARG;
  int n = -1;
  if (syscall(SYS_get_mempolicy, &n, nullptr, 0ul, host_ptr, kMpolFNode | kMpolFAddr) != 0) {
    *node = -1;
    return TW_ERR_UNSUPPORTED;
  }
  *node = n;
  return TW_OK;
}

extern "C" int tw_host_free(void* host_ptr) {
  if (!host_ptr) return TW_OK;
  size_t numa_len = 0;
  {
    std::lock_guard<std::mutex> lk(g_numa_mu);
    auto it = g_numa_regions.find(host_ptr);
    if (it != g_numa_regions.end()) {
      numa_len = it->second;
      g_numa_regions.erase(it);
    }
  }
  if (numa_len) {
    const cudaError_t e = cudaHostUnregister(host_ptr);
    munmap(host_ptr, numa_len);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return TW_ERR_CUDA;
    }
    return TW_OK;
  }
  cudaError_t err = cudaFreeHost(host_ptr);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

extern "C" int tw_host_device_pointer(void* host_ptr, void** device_ptr) {
  if (!host_ptr || !device_ptr) return TW_ERR_BAD_ARG;
  cudaError_t err = cudaHostGetDevicePointer(device_ptr, host_ptr, 0);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

extern "C" int tw_slab_write_rows(const void* src, int64_t src_entry_stride_rows, void* dst,
                                  int64_t dst_entry_stride_rows, int n_entries, int64_t n_rows,
                                  int64_t row_bytes, void* stream) {
  if (n_entries < 0 || n_rows < 0 || row_bytes <= 0 || src_entry_stride_rows < n_rows ||
      dst_entry_stride_rows < n_rows)
    return TW_ERR_BAD_ARG;
  if (n_entries == 0 || n_rows == 0) return TW_OK;
  if (!src || !dst) return TW_ERR_BAD_ARG;
  const cudaError_t err = cudaMemcpy2DAsync(
      dst, (size_t)(dst_entry_stride_rows * row_bytes), src,
      (size_t)(src_entry_stride_rows * row_bytes), (size_t)(n_rows * row_bytes), (size_t)n_entries,
      cudaMemcpyDefault, (cudaStream_t)stream);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return TW_ERR_CUDA;
  }
  return TW_OK;
}

// Workspace: scores [G*R*P] fp32 | logits [G*R*b0*block] fp32 (the per-stage
// kernels), then the fused selection's union merge region (count u32[G] and
// candidate bitmap u32[G][ceil(P*block/32)], at the end of the caller's
// buffer; zero before the first call, left zero by every call).
extern "C" size_t tw_select_layer_workspace_size(int groups, int heads_per_group, int n_pages,
                                                 int b0_pages, int block_size) {
  if (groups <= 0 || heads_per_group <= 0 || n_pages < 0 || b0_pages < 0 || block_size <= 0)
    return 0;
  const size_t rows = (size_t)groups * heads_per_group;
  return align256(rows * (size_t)n_pages * sizeof(float)) +
         align256(rows * (size_t)b0_pages * block_size * sizeof(float)) +
         merge_region_bytes(groups, n_pages, block_size);
}

extern "C" int tw_select_layer(const float* q, const void* page_min, const void* page_max,
                               int64_t meta_group_stride, int n_pages, const uint8_t* packed,
                               const void* scale, const void* minimum, int64_t entry_stride_tokens,
                               int groups, int heads_per_group, int b0_pages, int block_size,
                               int sink, int head_dim, int group_size, int dtype, double top_p,
                               int64_t old_length, int64_t sink_end, int64_t recent_start,
                               int32_t* pages_out, int32_t* union_pos, int64_t pos_stride,
                               int32_t* union_count, int32_t* head_count, int32_t* head_pos,
                               int32_t* error_flag, void* workspace, size_t workspace_bytes,
                               void* stream) {
  if (b0_pages <= 0 || b0_pages > n_pages || !pages_out) return TW_ERR_BAD_ARG;
  const size_t need =
      tw_select_layer_workspace_size(groups, heads_per_group, n_pages, b0_pages, block_size);
  if (need == 0) return TW_ERR_BAD_ARG;
  if (!workspace || workspace_bytes < need) return TW_ERR_CAPACITY;
  if (head_dim != kHeadDim) return TW_ERR_UNSUPPORTED;
  int st = select_layer_fused(q, TW_F32, page_min, page_max, meta_group_stride, n_pages, packed,
                              scale, minimum, entry_stride_tokens, groups, heads_per_group,
                              b0_pages, block_size, sink, group_size, dtype, top_p, old_length,
                              sink_end, recent_start, pages_out, union_pos, pos_stride,
                              union_count, head_count, head_pos, error_flag, workspace,
                              workspace_bytes, nullptr, nullptr, (cudaStream_t)stream);
  if (st != TW_ERR_UNSUPPORTED) return st;
  // per-stage kernels (shapes the fused selection does not serve)
  const size_t rows = (size_t)groups * heads_per_group;
  float* scores = reinterpret_cast<float*>(workspace);
  float* logits = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                           align256(rows * (size_t)n_pages * sizeof(float)));
  st = tw_quest_score(q, page_min, page_max, groups, heads_per_group, n_pages,
                          meta_group_stride, head_dim, dtype, scores, stream);
  if (st != TW_OK) return st;
  st = tw_topk_pages(scores, (int)rows, n_pages, b0_pages, pages_out, stream);
  if (st != TW_OK) return st;
  st = tw_int4_qk(q, packed, scale, minimum, entry_stride_tokens, pages_out, groups,
                  heads_per_group, b0_pages, block_size, sink, head_dim, group_size, dtype,
                  logits, stream);
  if (st != TW_OK) return st;
  return tw_top_p_union(logits, pages_out, groups, heads_per_group, b0_pages, block_size, sink,
                        top_p, old_length, sink_end, recent_start, union_pos, pos_stride,
                        union_count, head_count, head_pos, error_flag, stream);
}

extern "C" size_t tw_decode_layer_args_size(void) { return sizeof(tw_decode_layer_args); }

extern "C" size_t tw_row_reuse_size(void) { return sizeof(tw_row_reuse); }

// The four per-stage selection kernels of a layer-step (shapes the fused
// selection does not serve); pmin .. minimum are the first entry's arrays.
static int select_stages(const tw_decode_layer_args* a, const void* pmin, const void* pmax,
                         const uint8_t* packed, const void* scale, const void* minimum,
                         cudaStream_t st) {
  const int G = a->groups, R = a->heads_per_group;
  const size_t rows = (size_t)G * R;
  float* scores = reinterpret_cast<float*>(a->select_workspace);
  float* logits = reinterpret_cast<float*>(reinterpret_cast<char*>(a->select_workspace) +
                                           align256(rows * (size_t)a->n_pages * sizeof(float)));
  int rc = quest_score_dispatch(a->q, a->dtype, pmin, pmax, G, R, a->n_pages,
                                a->page_capacity * kHeadDim, a->dtype, scores, st);
  if (rc != TW_OK) return rc;
  rc = tw_topk_pages(scores, (int)rows, a->n_pages, a->b0_pages, a->pages, st);
  if (rc != TW_OK) return rc;
  rc = launch_int4_qk(a->q, a->dtype, packed, scale, minimum, a->max_len, a->pages, G, R,
                      a->b0_pages, a->block_size, a->sink, a->int4_group_size, a->dtype, logits, st);
  if (rc != TW_OK) return rc;
  return tw_top_p_union(logits, a->pages, G, R, a->b0_pages, a->block_size, a->sink, a->top_p,
                        a->old_length, a->sink_end, a->recent_start, a->union_pos, a->pos_stride,
                        a->union_count, a->head_count, a->head_pos, a->error_flag, st);
}

extern "C" int tw_twilight_decode_layer(const tw_decode_layer_args* a, void* stream) {
  if (!a) return TW_ERR_BAD_ARG;
  if (a->dtype != TW_F16 && a->dtype != TW_BF16) return TW_ERR_UNSUPPORTED;
  if (a->b0_pages <= 0 || a->b0_pages > a->n_pages || a->groups <= 0 || a->first_entry < 0 ||
      !a->q || !a->k_new || !a->v_new || !a->out || !a->pages)
    return TW_ERR_BAD_ARG;
  const int G = a->groups, R = a->heads_per_group;
  const size_t need = tw_select_layer_workspace_size(G, R, a->n_pages, a->b0_pages, a->block_size);
  if (need == 0) return TW_ERR_BAD_ARG;
  if (!a->select_workspace || a->select_workspace_bytes < need) return TW_ERR_CAPACITY;
  if (a->int4_group_size != 32 && a->int4_group_size != 64 && a->int4_group_size != 128)
    return TW_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  const size_t elem = 2;  // fp16 / bf16
  const int ngroups = kHeadDim / a->int4_group_size;
  const int64_t e0 = a->first_entry;
  const char* pmin = (const char*)a->page_min + e0 * a->page_capacity * kHeadDim * elem;
  const char* pmax = (const char*)a->page_max + e0 * a->page_capacity * kHeadDim * elem;
  const uint8_t* packed = a->packed + e0 * a->max_len * (kHeadDim / 2);
  const char* scale = (const char*)a->scale + e0 * a->max_len * ngroups * elem;
  const char* minimum = (const char*)a->minimum + e0 * a->max_len * ngroups * elem;
  // Protected-row staging (not with row reuse, whose kept rows serve them).
  ProtectedStage stage{};
  const bool staged = a->stage_k != nullptr && a->reuse == nullptr;
  if (staged) {
    if (!a->stage_v || a->stage_rows < a->sink_end + (a->old_length - a->recent_start))
      return TW_ERR_CAPACITY;
    stage.slab_k = (const uint4*)a->slab_k;
    stage.slab_v = (const uint4*)a->slab_v;
    stage.dirs = (const unsigned long long*)a->entry_dirs;
    stage.n_entries = a->n_entries > 0 ? a->n_entries : (int64_t)a->first_entry + G;
    stage.max_len = a->max_len;
    stage.first_entry = a->first_entry;
    stage.stage_k = (uint4*)a->stage_k;
    stage.stage_v = (uint4*)a->stage_v;
    stage.stage_rows = a->stage_rows;
    stage.n_sink = a->sink_end;
    stage.recent_start = a->recent_start;
    stage.old_length = a->old_length;
  }
  // The new token's append runs in the selection launch (one CTA per group):
  // it writes position old_length, which neither this step's selection nor
  // its attention reads.
  AppendArgs app{};
  bool fuse_append = false;
  if (a->append) {
    const int st_app = check_append_args(
        a->slab_k, a->slab_v, a->entry_dirs, a->n_entries, a->max_len, a->first_entry, G,
        a->old_length, a->k_new, a->v_new, a->sink, a->block_size, a->page_min, a->page_max,
        a->packed, a->scale, a->minimum, a->int4_group_size);
    if (st_app != TW_OK) return st_app;
    app = make_append_args(a->slab_k, a->slab_v, a->entry_dirs, a->n_entries, a->max_len,
                           a->first_entry, a->old_length, a->k_new, a->v_new, a->sink,
                           a->block_size, a->page_min, a->page_max, a->page_capacity * kHeadDim,
                           a->packed, a->scale, a->minimum, a->int4_group_size);
    fuse_append = true;  // one CTA per group of the selection launch appends
  }
  int rc = select_layer_fused(a->q, a->dtype, pmin, pmax, a->page_capacity * kHeadDim, a->n_pages,
                              packed, scale, minimum, a->max_len, G, R, a->b0_pages, a->block_size,
                              a->sink, a->int4_group_size, a->dtype, a->top_p, a->old_length,
                              a->sink_end, a->recent_start, a->pages, a->union_pos, a->pos_stride,
                              a->union_count, a->head_count, a->head_pos, a->error_flag,
                              a->select_workspace, a->select_workspace_bytes,
                              staged ? &stage : nullptr, fuse_append ? &app : nullptr, st);
  bool stage_filled = staged;
  if (rc == TW_ERR_UNSUPPORTED) {
    rc = select_stages(a, pmin, pmax, packed, scale, minimum, st);
    stage_filled = false;  // the per-stage kernels stage nothing
    fuse_append = false;   // nor append
  }
  if (rc != TW_OK) return rc;
  rc = attend_union_impl(a->slab_k, a->slab_v, a->entry_dirs, a->n_entries, a->max_len,
                         a->first_entry, G, a->old_length,
                         a->union_pos, a->pos_stride, a->union_count, a->k_new, a->v_new, a->q, R,
                         a->max_rows_per_group, kHeadDim, a->dtype,
                         1.0f / sqrtf((float)kHeadDim), a->out, a->out_dtype, nullptr,
                         a->error_flag, a->attn_workspace, a->attn_workspace_bytes, a->reuse,
                         stage_filled ? &stage : nullptr, st);
  if (rc != TW_OK || !a->append || fuse_append) return rc;
  return tw_append_token(a->slab_k, a->slab_v, a->entry_dirs, a->n_entries, a->max_len,
                         a->first_entry, G, a->old_length,
                         a->k_new, a->v_new, kHeadDim, a->dtype, a->sink, a->block_size,
                         a->page_min, a->page_max, a->page_capacity * kHeadDim, a->packed,
                         a->scale, a->minimum, a->int4_group_size, stream);
}
