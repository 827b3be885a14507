// C ABI glue: status text, mapped host slab allocation and the whole-layer
// Twilight selection that chains the Quest and INT4/top-p kernels.
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

extern "C" int tw_abi_version(void) { return 1; }

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

extern "C" int tw_host_free(void* host_ptr) {
  if (!host_ptr) return TW_OK;
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

// Workspace: scores [G*R*P] fp32 | logits [G*R*b0*block] fp32.
extern "C" size_t tw_select_layer_workspace_size(int groups, int heads_per_group, int n_pages,
                                                 int b0_pages, int block_size) {
  if (groups <= 0 || heads_per_group <= 0 || n_pages < 0 || b0_pages < 0 || block_size <= 0)
    return 0;
  const size_t rows = (size_t)groups * heads_per_group;
  return align256(rows * (size_t)n_pages * sizeof(float)) +
         align256(rows * (size_t)b0_pages * block_size * sizeof(float));
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
  const size_t rows = (size_t)groups * heads_per_group;
  float* scores = reinterpret_cast<float*>(workspace);
  float* logits = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                           align256(rows * (size_t)n_pages * sizeof(float)));
  int st = tw_quest_score(q, page_min, page_max, groups, heads_per_group, n_pages,
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
