/*
 * twilight_b200.h — C ABI of the B200 (sm_100a) sparse decode-attention path.
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream handle
 * (cudaStream_t passed as void*; NULL = legacy default stream) and returns an
 * int status (TW_OK = 0).  Device buffers are owned by the caller; the library
 * allocates nothing on the device except inside tw_host_alloc_mapped.
 * All launches are asynchronous on the given stream.
 *
 * Layouts (D = head_dim = 128, E = cache entries = layers x kv_heads,
 * entry = layer * kv_heads + kv_head, exactly as the reference):
 *   slab K / V planes   [E][max_len][D]      K/V dtype, pinned + mapped host
 *   page_min / page_max [E][page_cap][D]     K dtype (Quest metadata)
 *   int4 codes          [E][max_len][D/2]    u8, byte j = code[2j] | code[2j+1] << 4
 *   int4 scale / min    [E][max_len][D/gs]   K dtype, gs = quantisation group
 *   queries             [G][R][D]            fp32 (the reference's q.float())
 *
 * ENTRY DIRECTORY.  Functions that read or write slab rows take
 * (slab_k, slab_v, entry_dirs, n_entries, max_len).  With entry_dirs NULL,
 * row p of entry e is slab_{k,v} + (e*max_len + p)*D elements.  Otherwise
 * entry_dirs is a device array [2][n_entries] of byte addresses: entry_dirs[e]
 * is row 0 of entry e's K and entry_dirs[n_entries+e] of its V, each entry
 * holding max_len contiguous rows.  That places GPU-resident heads in device
 * memory and offloaded heads in the mapped host slab (HeadInfer's head-wise
 * residency, hi/cache.py:5-145) without a second code path.
 *
 * Reference interfaces are cited as path:line inside the reference project
 * (source/headinfer/headinfer/ abbreviated hi/).
 */
#ifndef TWILIGHT_B200_H
#define TWILIGHT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  TW_ERR_INVALID_INDEX mirrors gather_kv's nonzero return for an
 * out-of-range row (hi/cpu_kv_gather.cpp:9-10). */
#define TW_OK 0
#define TW_ERR_INVALID_INDEX 1
#define TW_ERR_BAD_ARG 2
#define TW_ERR_CAPACITY 3
#define TW_ERR_ORDER 4
#define TW_ERR_CUDA 5
#define TW_ERR_TIMEOUT 6
#define TW_ERR_UNSUPPORTED 7

/* dtype codes */
#define TW_F16 0
#define TW_BF16 1
#define TW_F32 2

/* Human-readable status text; never NULL. */
const char* tw_status_string(int status);
/* cudaError_t recorded by the last call that returned TW_ERR_CUDA on this thread. */
int tw_last_cuda_error(void);
/* ABI version of this library. */
int tw_abi_version(void);

/* ---- host slab -------------------------------------------------------------
 * Pinned, device-mapped host allocation for the K/V slab.  Replaces the
 * reference's pin_memory slab (hi/quest_offload_cache.py:100-105) plus the
 * cudaHostGetDevicePointer mapping of its zero-copy path
 * (hi/resident_zero_copy.py:15-29).  *device_ptr is what kernels read. */
int tw_host_alloc_mapped(size_t bytes, void** host_ptr, void** device_ptr);
/* The same on one host NUMA node: anonymous memory bound to `numa_node` (-1:
 * the node closest to the current device, cudaDevAttrHostNumaId) before
 * first touch, then page-locked and mapped with cudaHostRegister.  The slab
 * placement of the reference's multi-GPU plan (each GPU's slab on its own
 * NUMA node; hi/slab_cache.py:37-74 allocates without placement).
 * *bound_node (nullable) receives the node the memory was bound to, or -1
 * when the system refused the binding (the memory is then placed by the
 * default policy).  Freed with tw_host_free. */
int tw_host_alloc_mapped_numa(size_t bytes, int numa_node, void** host_ptr, void** device_ptr,
                              int* bound_node);
/* Host NUMA node holding the page at host_ptr (TW_ERR_UNSUPPORTED without NUMA). */
int tw_host_numa_node(const void* host_ptr, int* node);
int tw_host_free(void* host_ptr);
/* Device address of memory that is already pinned (e.g. torch pin_memory). */
int tw_host_device_pointer(void* host_ptr, void** device_ptr);

/* ---- slab writes -------------------------------------------------------------
 * Rows [0, n_rows) of n_entries consecutive entries, entry e at
 * src + e*src_entry_stride_rows*row_bytes, to dst + e*dst_entry_stride_rows*row_bytes
 * (device or mapped host memory) with one pitched copy on `stream`: the
 * prefill write of K / V into the slab (QuestTopKOffloadedCache's D2H,
 * hi/quest_offload_cache.py:513-537) for a whole layer of entries at once. */
int tw_slab_write_rows(const void* src, int64_t src_entry_stride_rows, void* dst,
                       int64_t dst_entry_stride_rows, int n_entries, int64_t n_rows,
                       int64_t row_bytes, void* stream);

/* ---- Quest metadata ----------------------------------------------------------
 * Page-wise channel min/max of K over complete block_size pages after the sink.
 * Replaces QuestTopKOffloadedCache._build_metadata (hi/quest_offload_cache.py:276-289).
 * keys: [n_entries][key_entry_stride] elements; page p of entry e covers rows
 * sink + p*block_size .. +block_size of that entry.  Pages
 * [first_page, first_page + n_pages) are written to
 * page_min/page_max + e*meta_entry_stride + p*D. */
int tw_quest_page_metadata(const void* keys, int64_t key_entry_stride, int n_entries,
                           int sink, int block_size, int head_dim, int dtype,
                           int first_page, int n_pages,
                           void* page_min, void* page_max, int64_t meta_entry_stride,
                           void* stream);

/* ---- INT4 affine quantiser -----------------------------------------------------
 * Group-wise asymmetric INT4 codes, bit-exact with affine_int4_pack
 * (hi/twilight_offload_cache.py:25-37) applied to K.view(-1, group_size).
 * keys: n_entries x n_tokens rows, row r of entry e at keys + (e*key_entry_stride + r)*D.
 * Outputs row r of entry e at index (e*out_entry_stride + out_row_offset + r). */
int tw_int4_pack(const void* keys, int64_t key_entry_stride, int n_entries, int64_t n_tokens,
                 int head_dim, int group_size, int dtype,
                 uint8_t* packed, void* scale, void* minimum,
                 int64_t out_entry_stride, int64_t out_row_offset, void* stream);
/* As tw_int4_pack with the rounding of the reference's `/ 15.0` made explicit:
 * scale_div 0 = multiply by the fp32 reciprocal (torch executing it on CUDA,
 * the reference's prefill device path; tw_int4_pack's mode), 1 = IEEE divide
 * (torch executing it on CPU). */
int tw_int4_pack_ex(const void* keys, int64_t key_entry_stride, int n_entries, int64_t n_tokens,
                    int head_dim, int group_size, int dtype,
                    uint8_t* packed, void* scale, void* minimum,
                    int64_t out_entry_stride, int64_t out_row_offset, int scale_div,
                    void* stream);

/* ---- Quest upper-bound score ---------------------------------------------------
 * score[g][r][p] = sum_d (q[g][r][d] > 0 ? max[g][p][d] : min[g][p][d]) * q[g][r][d],
 * fp32, summed in the order of the reference's fused kernel
 * (hi/twilight_fused_quest.py:13-46): lane l accumulates d = l, l+32, l+64, l+96,
 * then a shfl-down tree 1,2,4,8,16.  page_min/max: [G][meta_group_stride] elements. */
int tw_quest_score(const float* q, const void* page_min, const void* page_max,
                   int groups, int heads_per_group, int n_pages, int64_t meta_group_stride,
                   int head_dim, int dtype, float* scores, void* stream);

/* ---- Top-k pages ----------------------------------------------------------------
 * For each of `rows` rows of n scores: the k largest, written as ascending page
 * ids [rows][k] (int32).  Replaces torch.topk(sorted=False) + sort
 * (hi/twilight_offload_cache.py:1153-1155; hi/quest_offload_cache.py:373-374).
 * Ties at the k-th value keep the lowest page ids.  Requires k <= n <= 16384. */
int tw_topk_pages(const float* scores, int rows, int n, int k, int32_t* out_pages, void* stream);

/* ---- INT4 QK estimate -------------------------------------------------------------
 * logits[g][r][n] = (sum_d (code*scale + min) * q[g][r][d]) * (1/sqrt(D)) for the
 * b0*block_size candidate tokens sink + pages[g][r][i]*block_size + j.
 * Replaces fused_affine_int4_qk (hi/twilight_fused_qk.py:34-55) and the /sqrt(D)
 * scaling (hi/twilight_offload_cache.py:1261).  packed/scale/minimum point at the
 * layer's first entry; entry g is at +g*entry_stride_tokens rows. */
int tw_int4_qk(const float* q, const uint8_t* packed, const void* scale, const void* minimum,
               int64_t entry_stride_tokens, const int32_t* pages,
               int groups, int heads_per_group, int b0_pages, int block_size, int sink,
               int head_dim, int group_size, int dtype, float* logits, void* stream);

/* ---- Top-p + GQA union ---------------------------------------------------------------
 * Per (g, r) row: the smallest count c such that the c largest-logit candidates
 * hold >= top_p of the softmax mass (the argsort/softmax/cumsum/searchsorted+1
 * rule of hi/twilight_exact_top_p_graph.py:19-32, hi/twilight_offload_cache.py:1266-1310,
 * budget_mode='dynamic').  Then per group g the sorted union of
 * [0, sink_end) U [recent_start, old_length) U the R rows' selected positions
 * (hi/twilight_offload_cache.py:1527-1549 + flatnonzero :1602-1614).
 * union_pos: [G][pos_stride] int32 ascending, union_count: [G], head_count: [G][R].
 * head_pos (nullable): [G][R][b0*block_size] each row's selected positions ascending.
 * error_flag (nullable): set nonzero if a candidate position falls outside
 * [0, old_length).  Launches G clusters of R CTAs (R <= 8). */
int tw_top_p_union(const float* logits, const int32_t* pages,
                   int groups, int heads_per_group, int b0_pages, int block_size, int sink,
                   double top_p, int64_t old_length, int64_t sink_end, int64_t recent_start,
                   int32_t* union_pos, int64_t pos_stride, int32_t* union_count,
                   int32_t* head_count, int32_t* head_pos, int32_t* error_flag, void* stream);

/* ---- whole-layer Twilight selection ----------------------------------------------------
 * Quest score -> top-k pages -> INT4 QK -> top-p + union in one call (4 launches).
 * Replaces TwilightMatchedBudgetOffloadedCache.prepare_layer_selection
 * (hi/twilight_offload_cache.py:996-1843, gpu_compact_gqa_union path).
 * workspace: >= tw_select_layer_workspace_size(...) bytes of device memory,
 * zero-filled once before its first use: its last bytes hold the fused
 * selection's union merge state (a per-group count and candidate bitmap),
 * which every call leaves zero again.  Calls sharing one workspace must not
 * overlap on the GPU.
 * pages_out: [G][R][b0] int32 (the Quest B0 pages, ascending). */
size_t tw_select_layer_workspace_size(int groups, int heads_per_group, int n_pages, int b0_pages,
                                      int block_size);
int tw_select_layer(const float* q, const void* page_min, const void* page_max,
                    int64_t meta_group_stride, int n_pages,
                    const uint8_t* packed, const void* scale, const void* minimum,
                    int64_t entry_stride_tokens,
                    int groups, int heads_per_group, int b0_pages, int block_size, int sink,
                    int head_dim, int group_size, int dtype, double top_p,
                    int64_t old_length, int64_t sink_end, int64_t recent_start,
                    int32_t* pages_out, int32_t* union_pos, int64_t pos_stride,
                    int32_t* union_count, int32_t* head_count, int32_t* head_pos,
                    int32_t* error_flag, void* workspace, size_t workspace_bytes, void* stream);

/* ---- row gather ---------------------------------------------------------------------------
 * out_k[i] = k[rows[i]], out_v[i] = v[rows[i]] for i < n, row_bytes each, read
 * straight from (mapped host or device) memory by the GPU.  Same arguments and
 * bounds contract as gather_kv (hi/cpu_kv_gather.cpp:3-16): an index outside
 * [0, source_rows) is skipped and sets *error_flag (device int32) to 1.
 * row_bytes must be a multiple of 16 and all pointers 16-byte aligned. */
int tw_gather_kv(const void* k, const void* v, void* out_k, void* out_v,
                 const int64_t* rows, int64_t n, int64_t source_rows, int64_t row_bytes,
                 int32_t* error_flag, void* stream);

/* ---- previous-token row reuse -----------------------------------------------------------------------
 * Rows a group gathered at the previous decode step stay in device memory; a
 * row of this step's union whose position the previous step also read (one
 * of its union positions, or its current token) is read from there instead of
 * over the host link.  The reference's previous_token_resident_cache
 * (hi/twilight_offload_cache.py:2457-2608, :2798-3470; hit/miss mapping
 * hi/resident_gpu_mapping.py:103-144, hi/resident_mapping.cpp:6-53;
 * hi/resident_zero_copy.cu:7-42).
 *
 * row_map is a direct-addressed table per group: row_map[g][pos] =
 * (tag << 32) | row, written for every row a step keeps (its union rows and
 * its current token at pos = old_length), where row indexes that step's kept
 * rows.  A step reads row_map[g][pos]; the entry is a hit when its tag equals
 * prev_tag (nonzero) and row < prev_rows, and then the row is read from
 * prev_k / prev_v.  The step then stores its own entries with next_tag.  Each
 * position is read and written by one thread group of one launch, so reads
 * and writes of a step never race.  Zero the table once before the first
 * step; use tags that are nonzero and unique per step of the table's layer
 * (a stale entry never carries the previous tag).
 *
 * tw_attend_union / tw_twilight_decode_layer keep rows strided: row of
 * (group g, index i) = g * rows_stride + i in next_k / next_v [G][rows_stride][D]
 * (union rows in order, then the current token).  tw_gather_union keeps its
 * own packed output (row = its output row): there next_k / next_v must be
 * NULL and rows_stride is unused.  prev_k / prev_v hold prev_rows rows of the
 * previous step's layout, and must not overlap the rows being written.
 * row_counts [G][2] (nullable) accumulates (hit rows, miss rows) of the union
 * (the current token is not counted). */
typedef struct tw_row_reuse {
  uint64_t* row_map;        /* [G][map_stride], map_stride > old_length */
  int64_t map_stride;
  uint32_t prev_tag;        /* 0: no previous rows (every row is a miss) */
  uint32_t next_tag;        /* nonzero, != prev_tag */
  const void* prev_k;
  const void* prev_v;
  int64_t prev_rows;
  void* next_k;
  void* next_v;
  int64_t rows_stride;
  int32_t* row_counts;
} tw_row_reuse;

/* ---- GQA union gather into the attention layout ----------------------------------------------
 * Zero-copy gather of each group's union rows from the host slab, followed by
 * the group's current-token row: out rows [cu[g], cu[g+1]) = slab rows of
 * union_pos[g][0..count_g) then cur[g].  Writes cu_seqlens [G+1] int32.
 * Replaces the flat CPU gather + chunked H2D + direct attention layout of
 * update_layer_gqa_group_ragged (hi/twilight_offload_cache.py:2973-3101, :3307-3310)
 * and the miss branch of assemble_zero_copy (hi/resident_zero_copy.cu:7-42).
 * slab_k/slab_v: device-visible addresses of the K and V planes.
 * Rows beyond rows_cap or positions outside [0, old_length) set *error_flag.
 * reuse (nullable): previous-token row reuse, see tw_row_reuse. */
int tw_gather_union(const void* slab_k, const void* slab_v, const uint64_t* entry_dirs,
                    int64_t n_entries, int64_t max_len, int first_entry,
                    int groups, int64_t old_length,
                    const int32_t* union_pos, int64_t pos_stride, const int32_t* union_count,
                    const void* cur_k, const void* cur_v, int head_dim, int dtype,
                    void* out_k, void* out_v, int64_t rows_cap, int32_t* cu_seqlens,
                    int32_t* error_flag, const tw_row_reuse* reuse, void* stream);

/* ---- Quest per-query-head gather ------------------------------------------------------------------
 * Per (g, r): rows [0, sink_end) U {sink + pages[g][r][i]*block_size + j} U
 * [recent_start, old_length) then the group's current token, each head one
 * segment of the flat layout (segment s = g*R + r, equal lengths
 * seg_len = sink_end + k*block_size + (old_length - recent_start) + 1).
 * Each distinct source row of a group (its sink and recent rows, and a page
 * named by several heads or twice by one) is read once and written to every
 * segment holding it; pages may come in any order.  A page id < 0 or a row at
 * or beyond old_length sets TW_ERR_INVALID_INDEX in error_flag and writes zeros.
 * Replaces _selected_positions + update_layer_flat_ragged packing
 * (hi/quest_offload_cache.py:403-511, :724-987) and the per-entry pack of update
 * (:578-630). */
int tw_gather_quest_heads(const void* slab_k, const void* slab_v, const uint64_t* entry_dirs,
                          int64_t n_entries, int64_t max_len, int first_entry,
                          int groups, int heads_per_group, int64_t old_length,
                          int64_t sink_end, int64_t recent_start, int sink, int block_size,
                          const int32_t* pages, int k_pages,
                          const void* cur_k, const void* cur_v, int head_dim, int dtype,
                          void* out_k, void* out_v, int32_t* error_flag, void* stream);

/* ---- new-token append ------------------------------------------------------------------------------
 * Writes each group's current K/V row to slab position `position`, folds it
 * into the running Quest page min/max (page (position-sink)/block_size, when
 * position >= sink) and INT4-packs it.  page_min/page_max/packed/scale/minimum
 * may be NULL to skip that part.  Replaces the new-KV D2H
 * (hi/quest_offload_cache.py:230-274, hi/twilight_offload_cache.py:551-794) and
 * extends the prefill-only metadata (hi/quest_offload_cache.py:276-289,
 * hi/twilight_offload_cache.py:925-936) to appended tokens. */
int tw_append_token(void* slab_k, void* slab_v, const uint64_t* entry_dirs, int64_t n_entries,
                    int64_t max_len, int first_entry, int groups,
                    int64_t position, const void* cur_k, const void* cur_v,
                    int head_dim, int dtype, int sink, int block_size,
                    void* page_min, void* page_max, int64_t meta_entry_stride,
                    uint8_t* packed, void* scale, void* minimum, int group_size,
                    void* stream);

/* ---- sparse GQA decode attention -------------------------------------------------------------------------
 * out[s][r] = softmax(q[s][r] . K[cu[s]:cu[s+1]]^T * softmax_scale) . V[cu[s]:cu[s+1]]
 * for s < segments, r < heads_per_segment; q_len = 1 so every key is visible.
 * Split-K flash-decode with a log-sum-exp merge, fp32 accumulation.
 * Replaces flash_attn_varlen_func as called by hi/mp.py:258-279 (wrapper :21-52).
 * q: [S][R][D] in `dtype`; k/v: [rows][D] in `dtype`; out: [S][R][D] in out_dtype
 * (dtype or TW_F32); lse (nullable): [S][R] fp32 natural-log sum-exp.
 * max_seqlen_k: an upper bound of cu[s+1]-cu[s] (sizes the split grid).
 * workspace: >= tw_decode_attention_workspace_size(...) bytes, 16-byte aligned;
 * its counter area must be zero before the first call (the kernel leaves it zero). */
size_t tw_decode_attention_workspace_size(int segments, int heads_per_segment, int max_seqlen_k,
                                          int head_dim);
int tw_decode_attention(const void* q, const void* k, const void* v, const int32_t* cu_seqlens,
                        int segments, int heads_per_segment, int max_seqlen_k, int head_dim,
                        int dtype, float softmax_scale, void* out, int out_dtype, float* lse,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ---- fused union gather + decode attention ---------------------------------------------------------
 * The GQA group step without a staged copy: for each group g the split-K
 * attention CTAs read the rows of union_pos[g][0..union_count[g]) straight
 * from the (mapped host) slab, then the group's current token (cur_k/cur_v
 * [G][D]), and write out [G][R][D] (q [G][R][D] in `dtype`).  Same result as
 * tw_gather_union followed by tw_decode_attention.  Replaces the gather + H2D
 * + FlashAttention sequence of hi/twilight_offload_cache.py:2973-3101 and
 * hi/mp.py:258-279.  max_rows_per_group: an upper bound of union_count[g]+1
 * (sizes the split grid and the workspace, as max_seqlen_k of
 * tw_decode_attention_workspace_size(groups, R, max_rows_per_group, D)).
 * Positions outside [0, old_length) are skipped and set *error_flag. */
int tw_attend_union(const void* slab_k, const void* slab_v, const uint64_t* entry_dirs,
                    int64_t n_entries, int64_t max_len, int first_entry,
                    int groups, int64_t old_length, const int32_t* union_pos, int64_t pos_stride,
                    const int32_t* union_count, const void* cur_k, const void* cur_v,
                    const void* q, int heads_per_group, int max_rows_per_group, int head_dim,
                    int dtype, float softmax_scale, void* out, int out_dtype, float* lse,
                    int32_t* error_flag, void* workspace, size_t workspace_bytes,
                    const tw_row_reuse* reuse, void* stream);

/* ---- whole decode layer-step --------------------------------------------------------------------------
 * One decode layer-step of the Twilight GQA path in one call: Quest score ->
 * top-k pages -> INT4 QK -> top-p + union -> fused union gather + attention ->
 * new-token append, with no host synchronisation.  When the fused selection
 * serves the shape this is 2 launches on `stream`: the selection (one
 * thread-block cluster per query-head row), whose CTAs also append the new
 * token (position old_length, which neither the selection nor the attention
 * of this step reads) and stage the protected rows, then the fused
 * attention.  Otherwise the per-stage kernels, the attention and the append
 * kernel run (6 launches).  select_workspace: >=
 * tw_select_layer_workspace_size(...) bytes, zero-filled once before its
 * first use (see tw_select_layer).
 * Replaces prepare_layer_selection + update_layer_gqa_group_ragged + the
 * FlashAttention call of one layer (hi/twilight_offload_cache.py:996-1843,
 * :2610-3602, hi/mp.py:233-279).  Cache pointers (slab, page min/max, INT4
 * codes/scale/min) are the bases of entry 0; the layer's entries are
 * first_entry .. first_entry+groups-1.  q is [G][R][D] in the K/V dtype (the
 * reference selects with q.float(), an exact widening); k_new/v_new [G][D];
 * out [G][R][D] in out_dtype.  Requires 0 < b0_pages <= n_pages.  append != 0
 * also writes the new token at position old_length.  head_pos may be NULL. */
typedef struct tw_decode_layer_args {
  void* slab_k;
  void* slab_v;
  const uint64_t* entry_dirs; /* [2][n_entries] row-0 addresses, or NULL (see ENTRY DIRECTORY) */
  int64_t n_entries;
  int64_t max_len;
  int32_t first_entry;
  int32_t groups;
  int32_t heads_per_group;
  int32_t dtype;
  void* page_min;
  void* page_max;
  int64_t page_capacity;
  int32_t n_pages;
  uint8_t* packed;
  void* scale;
  void* minimum;
  int32_t int4_group_size;
  int32_t sink;
  int32_t block_size;
  int32_t b0_pages;
  double top_p;
  int64_t old_length;
  int64_t sink_end;
  int64_t recent_start;
  const void* q;
  const void* k_new;
  const void* v_new;
  void* out;
  int32_t out_dtype;
  int32_t append;
  int32_t* pages;
  int32_t* union_pos;
  int64_t pos_stride;
  int32_t* union_count;
  int32_t* head_count;
  int32_t* head_pos;
  int32_t* error_flag;
  void* select_workspace;
  size_t select_workspace_bytes;
  void* attn_workspace;
  size_t attn_workspace_bytes;
  int32_t max_rows_per_group;
  const tw_row_reuse* reuse; /* NULL: no row reuse */
  /* Protected-row staging (stage_k NULL: off; ignored when reuse is set).
   * Each group's sink rows [0, sink_end) and recent rows [recent_start,
   * old_length) do not depend on the selection: the selection launch's CTAs
   * copy them (TMA bulk copies started at launch) from the slab into stage_k / stage_v
   * [G][stage_rows][D] (device memory, 16-byte aligned) while the selection
   * runs, and the attention reads them from there, so the host link carries
   * them while it would otherwise idle.  stage_rows >= sink_end +
   * (old_length - recent_start), else TW_ERR_CAPACITY.  No counterpart in the
   * reference, which copies these rows with the rest of the union
   * (hi/twilight_offload_cache.py:2973-3101).  Results are unchanged. */
  void* stage_k;
  void* stage_v;
  int64_t stage_rows;
} tw_decode_layer_args;
int tw_twilight_decode_layer(const tw_decode_layer_args* args, void* stream);
/* sizeof(tw_decode_layer_args), for binding-layout checks. */
size_t tw_decode_layer_args_size(void);
/* sizeof(tw_row_reuse), for binding-layout checks. */
size_t tw_row_reuse_size(void);

/* ---- decode-layer front end: q / k / v projection + rotary embedding -------------------------
 * One token (batch 1): q[h] = RoPE(W_q[h] . hidden), k[h] = RoPE(W_k[h] . hidden),
 * v[h] = W_v[h] . hidden, for n_q_heads / n_kv_heads heads of head_dim 128.
 * Replaces the layer-batched grouped projection + apply_rotary_pos_emb of
 * LlamaAttention_fast_forward (hi/mp.py:90-237) and its graph replay
 * (hi/twilight_projection_graph.py:12-41).  w_q [n_q_heads*128][hidden],
 * w_k / w_v [n_kv_heads*128][hidden] (the row-major nn.Linear weights), hidden
 * [hidden_size], cos / sin [128] for the token's position, all in `dtype`
 * (TW_F16 / TW_BF16), 16-byte aligned; hidden_size a multiple of 256, <= 16384.
 * Outputs q_out [n_q_heads][128] (= [G][R][128]), k_out / v_out
 * [n_kv_heads][128] in `dtype`.  Dot products accumulate in fp32 and are
 * rounded to `dtype`; the rotation rounds each product and the sum to `dtype`. */
int tw_qkv_rope(const void* hidden, const void* w_q, const void* w_k, const void* w_v,
                int hidden_size, int n_q_heads, int n_kv_heads, int head_dim, const void* cos,
                const void* sin, int dtype, void* q_out, void* k_out, void* v_out, void* stream);

/* ---- allocation-free decode attention ---------------------------------------------------------------
 * No counterpart in the reference: an addition of this library.  Same
 * computation, arguments and result as tw_decode_attention, but the caller
 * passes no workspace.  It is for callers that cannot allocate device memory:
 * a serving runtime that has reserved all device memory for its own arena, or
 * a host written in another language that is handed device buffers but has no
 * CUDA allocator to call.  The split-K scratch (merge counters and per-split
 * partials) lives in one fixed array of TW_NOALLOC_SCRATCH_BYTES inside this
 * library; every GPU that loads the library holds its own copy until the
 * process exits.  The call allocates nothing and calls no allocating routine.
 *   - Capacity: returns TW_ERR_CAPACITY (nothing launched) when the scratch
 *     needed exceeds the array: about segments * heads * ceil(max_seqlen_k/128)
 *     * 520 bytes (e.g. 8 segments x 4 heads up to max_seqlen_k ~ 31 000).
 *     A call with max_seqlen_k <= 128 uses no scratch.
 *   - Set-up: the first call on each device looks up the array's device
 *     address (cudaGetSymbolAddress) with that device current; make that
 *     first call before any stream capture.  Only a successful lookup is
 *     kept: if it fails the call returns TW_ERR_CUDA and the next call on
 *     that device tries again.  Device ordinals 0..63 are served; a higher
 *     ordinal returns TW_ERR_UNSUPPORTED.
 *   - Sharing: every call on a device uses the same array, which keeps the
 *     last call's contents (the call clears the counters it needs).  Calls
 *     whose executions overlap on the GPU (e.g. on two streams at once) race
 *     on the array and corrupt each other's results: serialise them. */
#define TW_NOALLOC_SCRATCH_BYTES (4u << 20)
int tw_decode_attention_noalloc(const void* q, const void* k, const void* v,
                                const int32_t* cu_seqlens, int segments, int heads_per_segment,
                                int max_seqlen_k, int head_dim, int dtype, float softmax_scale,
                                void* out, int out_dtype, float* lse, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TWILIGHT_B200_H */
