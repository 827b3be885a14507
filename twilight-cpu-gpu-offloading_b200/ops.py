"""Tensor-level wrappers of the C ABI (device memory from torch, work on the
current CUDA stream).  Every op runs the sm_100a kernels of
libtwilight_b200.so; a CPU tensor is rejected, never computed on the host.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _lib

HEAD_DIM = 128
DTYPE_CODES = {torch.float16: _lib.TW_F16, torch.bfloat16: _lib.TW_BF16, torch.float32: _lib.TW_F32}
SCALE_RECIPROCAL = 0   # "/ 15" as torch on CUDA: x * fp32(1/15)
SCALE_DIVIDE = 1       # "/ 15" as torch on CPU: IEEE division


def _stream(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


def _cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("twilight ops require CUDA tensors (no CPU fallback)")
        if not t.is_contiguous():
            raise ValueError("twilight ops require contiguous tensors")


def _kv_code(dtype: torch.dtype) -> int:
    if dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"K/V dtype must be float16 or bfloat16, got {dtype}")
    return DTYPE_CODES[dtype]


def lib():
    return _lib.load()


# ---------------------------------------------------------------- metadata --

def quest_page_metadata(keys: torch.Tensor, *, sink: int, block_size: int,
                        page_min: torch.Tensor, page_max: torch.Tensor, first_page: int = 0,
                        n_pages: int | None = None) -> int:
    """keys [E, S, D] -> page_min/page_max [E, page_cap, D] pages [first_page, +n_pages).
    hi/quest_offload_cache.py:276-289.  Returns the number of pages written."""
    _cuda(keys, page_min, page_max)
    E, S, D = keys.shape
    if D != HEAD_DIM or page_min.shape[0] != E or page_min.shape != page_max.shape:
        raise ValueError("unexpected metadata shapes")
    complete = max(0, S - sink) // block_size if S > sink else 0
    if n_pages is None:
        n_pages = complete - first_page
    if n_pages < 0 or first_page + n_pages > page_min.shape[1] or first_page + n_pages > complete:
        raise ValueError("page range outside the keys or the metadata capacity")
    _lib.check(lib().tw_quest_page_metadata(
        _ptr(keys), S * D, E, sink, block_size, D, _kv_code(keys.dtype), first_page, n_pages,
        _ptr(page_min), _ptr(page_max), page_min.shape[1] * D, _stream(keys.device)),
        "quest_page_metadata")
    return n_pages


def int4_pack(keys: torch.Tensor, *, group_size: int, packed: torch.Tensor, scale: torch.Tensor,
              minimum: torch.Tensor, out_row_offset: int = 0,
              scale_div: int = SCALE_RECIPROCAL) -> None:
    """keys [E, S, D] -> packed [E, cap, D/2] u8, scale/minimum [E, cap, D/gs] at rows
    out_row_offset.. (hi/twilight_offload_cache.py:25-37 over keys.view(-1, gs))."""
    _cuda(keys, packed, scale, minimum)
    E, S, D = keys.shape
    if packed.dtype != torch.uint8 or packed.shape[0] != E or packed.shape[-1] != D // 2:
        raise ValueError("packed must be uint8 [E, cap, D/2]")
    if scale.dtype != keys.dtype or minimum.dtype != keys.dtype:
        raise ValueError("scale/minimum must have the K dtype")
    cap = packed.shape[1]
    if out_row_offset + S > cap or scale.shape != (E, cap, D // group_size) or minimum.shape != scale.shape:
        raise ValueError("INT4 output capacity or group layout mismatch")
    _lib.check(lib().tw_int4_pack_ex(
        _ptr(keys), S, E, S, D, group_size, _kv_code(keys.dtype), _ptr(packed), _ptr(scale),
        _ptr(minimum), cap, out_row_offset, scale_div, _stream(keys.device)), "int4_pack")


# --------------------------------------------------------------- selection --

def quest_score(q: torch.Tensor, page_min: torch.Tensor, page_max: torch.Tensor, n_pages: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """q [G,R,D] fp32, page_min/max [G, page_cap, D] -> scores [G,R,n_pages] fp32.
    hi/twilight_fused_quest.py:13-46."""
    _cuda(q, page_min, page_max)
    G, R, D = q.shape
    if q.dtype != torch.float32 or page_min.shape[0] != G or n_pages > page_min.shape[1]:
        raise ValueError("quest_score expects fp32 q [G,R,D] and [G,cap,D] metadata")
    if out is None:
        out = torch.empty((G, R, n_pages), device=q.device, dtype=torch.float32)
    _lib.check(lib().tw_quest_score(_ptr(q), _ptr(page_min), _ptr(page_max), G, R, n_pages,
                                    page_min.shape[1] * D, D, _kv_code(page_min.dtype), _ptr(out),
                                    _stream(q.device)), "quest_score")
    return out


def topk_pages(scores: torch.Tensor, k: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """scores [..., n] fp32 -> ascending ids of the k largest [..., k] int32."""
    _cuda(scores)
    n = scores.shape[-1]
    rows = scores.numel() // max(n, 1)
    if out is None:
        out = torch.empty((*scores.shape[:-1], k), device=scores.device, dtype=torch.int32)
    _lib.check(lib().tw_topk_pages(_ptr(scores), rows, n, k, _ptr(out), _stream(scores.device)),
               "topk_pages")
    return out


def int4_qk(q: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, minimum: torch.Tensor,
            pages: torch.Tensor, *, block_size: int, sink: int,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """q [G,R,D]; packed [G, cap, D/2]; scale/minimum [G, cap, ng]; pages [G,R,b0] int32
    -> logits [G,R,b0*block] fp32 (hi/twilight_fused_qk.py:13-55, /sqrt(D) :1261)."""
    _cuda(q, packed, scale, minimum, pages)
    G, R, D = q.shape
    b0 = pages.shape[-1]
    group = D // scale.shape[-1]
    if out is None:
        out = torch.empty((G, R, b0 * block_size), device=q.device, dtype=torch.float32)
    _lib.check(lib().tw_int4_qk(_ptr(q), _ptr(packed), _ptr(scale), _ptr(minimum), packed.shape[1],
                                _ptr(pages), G, R, b0, block_size, sink, D, group,
                                _kv_code(scale.dtype), _ptr(out), _stream(q.device)), "int4_qk")
    return out


def top_p_union(logits: torch.Tensor, pages: torch.Tensor, *, block_size: int, sink: int,
                top_p: float, old_length: int, sink_end: int, recent_start: int,
                union_pos: torch.Tensor, union_count: torch.Tensor, head_count: torch.Tensor,
                head_pos: torch.Tensor | None = None,
                error_flag: torch.Tensor | None = None) -> None:
    """Top-p counts per row and the sorted GQA union per group (device outputs)."""
    _cuda(logits, pages, union_pos, union_count, head_count, head_pos, error_flag)
    G, R, n = logits.shape
    b0 = pages.shape[-1]
    _lib.check(lib().tw_top_p_union(
        _ptr(logits), _ptr(pages), G, R, b0, block_size, sink, float(top_p), old_length, sink_end,
        recent_start, _ptr(union_pos), union_pos.shape[-1], _ptr(union_count), _ptr(head_count),
        _ptr(head_pos), _ptr(error_flag), _stream(logits.device)), "top_p_union")


def select_layer(q: torch.Tensor, page_min: torch.Tensor, page_max: torch.Tensor, n_pages: int,
                 packed: torch.Tensor, scale: torch.Tensor, minimum: torch.Tensor, *, b0_pages: int,
                 block_size: int, sink: int, top_p: float, old_length: int, sink_end: int,
                 recent_start: int, union_pos: torch.Tensor, union_count: torch.Tensor,
                 head_count: torch.Tensor, head_pos: torch.Tensor | None = None,
                 error_flag: torch.Tensor | None = None,
                 pages: torch.Tensor | None = None) -> torch.Tensor:
    """Both Twilight selection stages of one layer (tw_select_layer: Quest score,
    top-k pages, INT4 estimate, top-p + GQA union; one fused launch where the
    shape allows).  q [G,R,D] fp32, metadata / codes as quest_score / int4_qk.
    Returns the B0 pages [G,R,b0] int32; the union and counts go to the outputs."""
    _cuda(q, page_min, page_max, packed, scale, minimum, union_pos, union_count, head_count,
          head_pos, error_flag, pages)
    G, R, D = q.shape
    if q.dtype != torch.float32:
        raise ValueError("select_layer expects fp32 q [G,R,D]")
    if pages is None:
        pages = torch.empty((G, R, b0_pages), device=q.device, dtype=torch.int32)
    ws_bytes = select_layer_workspace_bytes(G, R, n_pages, b0_pages, block_size)
    ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=q.device)  # merge region zero
    _lib.check(lib().tw_select_layer(
        _ptr(q), _ptr(page_min), _ptr(page_max), page_min.shape[1] * D, n_pages, _ptr(packed),
        _ptr(scale), _ptr(minimum), packed.shape[1], G, R, b0_pages, block_size, sink, D,
        D // scale.shape[-1], _kv_code(scale.dtype), float(top_p), old_length, sink_end,
        recent_start, _ptr(pages), _ptr(union_pos), union_pos.shape[-1], _ptr(union_count),
        _ptr(head_count), _ptr(head_pos), _ptr(error_flag), _ptr(ws), ws.numel(),
        _stream(q.device)), "select_layer")
    return pages


def select_layer_workspace_bytes(groups: int, heads: int, n_pages: int, b0_pages: int,
                                 block_size: int) -> int:
    return int(lib().tw_select_layer_workspace_size(groups, heads, n_pages, b0_pages, block_size))


# ------------------------------------------------------------------ gather --

def gather_kv(k: torch.Tensor, v: torch.Tensor, rows: torch.Tensor, out_k: torch.Tensor,
              out_v: torch.Tensor, error_flag: torch.Tensor) -> None:
    """out[i] = src[rows[i]] (hi/cpu_kv_gather.cpp:3-16 contract) on the GPU.  k/v may be
    CUDA tensors or mapped-host views given as (tensor, device_pointer) pairs."""
    kp, k_rows, row_bytes = _source(k)
    vp, v_rows, _ = _source(v)
    _cuda(rows, out_k, out_v, error_flag)
    if rows.dtype != torch.int64:
        raise ValueError("int64 row indices required")
    _lib.check(lib().tw_gather_kv(kp, vp, _ptr(out_k), _ptr(out_v), _ptr(rows), rows.numel(),
                                  k_rows, row_bytes, _ptr(error_flag), _stream(rows.device)),
               "gather_kv")


def _source(x):
    if isinstance(x, tuple):
        t, dev = x
        return dev, t.shape[0], t.shape[-1] * t.element_size()
    _cuda(x)
    return x.data_ptr(), x.shape[0], x.shape[-1] * x.element_size()


def decode_attention_workspace_bytes(segments: int, heads: int, max_seqlen_k: int) -> int:
    return int(lib().tw_decode_attention_workspace_size(segments, heads, max_seqlen_k, HEAD_DIM))


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_k: torch.Tensor,
                     max_seqlen_k: int, *, workspace: torch.Tensor, out: torch.Tensor | None = None,
                     out_dtype: torch.dtype | None = None, lse: torch.Tensor | None = None,
                     softmax_scale: float | None = None) -> torch.Tensor:
    """q [S,R,D]; k/v [rows,(1,)D]; cu_seqlens_k [S+1] int32 -> out [S,R,D].
    Replaces flash_attn_varlen_func at hi/mp.py:258-279."""
    _cuda(q, k, v, cu_seqlens_k, workspace, out, lse)
    S, R, D = q.shape
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k and v must share a dtype")
    if cu_seqlens_k.dtype != torch.int32 or cu_seqlens_k.numel() != S + 1:
        raise ValueError("cu_seqlens_k must be int32 [segments + 1]")
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty((S, R, D), device=q.device, dtype=out_dtype)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    _lib.check(lib().tw_decode_attention(
        _ptr(q), _ptr(k), _ptr(v), _ptr(cu_seqlens_k), S, R, int(max_seqlen_k), D,
        _kv_code(q.dtype), ctypes.c_float(scale), _ptr(out), DTYPE_CODES[out.dtype], _ptr(lse),
        _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(q.device)),
        "decode_attention")
    return out


def attend_union(slab, first_entry: int, old_length: int, union_pos: torch.Tensor,
                 union_count: torch.Tensor, cur_k: torch.Tensor, cur_v: torch.Tensor,
                 q: torch.Tensor, max_rows_per_group: int, *, workspace: torch.Tensor,
                 error_flag: torch.Tensor, out: torch.Tensor | None = None,
                 out_dtype: torch.dtype | None = None, lse: torch.Tensor | None = None,
                 softmax_scale: float | None = None,
                 entry_dirs: torch.Tensor | None = None,
                 reuse: "_lib.RowReuse | None" = None) -> torch.Tensor:
    """Fused union gather + decode attention straight from the mapped slab (or,
    with entry_dirs [2, E] int64 row-0 addresses, from each entry's placement).
    q [G,R,D] (K/V dtype), cur_k/cur_v [G,D], union_pos [G, stride] int32,
    union_count [G] int32 -> out [G,R,D].  reuse (row_reuse()): read rows of
    the previous step from device memory and keep this step's rows."""
    _cuda(union_pos, union_count, cur_k, cur_v, q, workspace, error_flag, out, lse)
    G, R, D = q.shape
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty((G, R, D), device=q.device, dtype=out_dtype)
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    _lib.check(lib().tw_attend_union(
        slab.key_device_ptr, slab.value_device_ptr, _ptr(entry_dirs),
        entry_dirs.shape[-1] if entry_dirs is not None else 0, slab.geometry.max_cache_len, first_entry, G,
        old_length, _ptr(union_pos), union_pos.shape[-1], _ptr(union_count), _ptr(cur_k),
        _ptr(cur_v), _ptr(q), R, int(max_rows_per_group), D, _kv_code(q.dtype),
        ctypes.c_float(scale), _ptr(out), DTYPE_CODES[out.dtype], _ptr(lse), _ptr(error_flag),
        _ptr(workspace), workspace.numel() * workspace.element_size(),
        ctypes.byref(reuse) if reuse is not None else None, _stream(q.device)),
        "attend_union")
    return out


def row_reuse(row_map: torch.Tensor, next_tag: int, *, next_k: torch.Tensor | None = None,
              next_v: torch.Tensor | None = None, prev_tag: int = 0,
              prev_k: torch.Tensor | None = None, prev_v: torch.Tensor | None = None,
              row_counts: torch.Tensor | None = None) -> "_lib.RowReuse":
    """tw_row_reuse for attend_union / decode_layer (next_k / next_v
    [G, S, D] receive this step's rows) or tw_gather_union (no next rows: its
    output is kept).  row_map [G, stride] int64 (zeroed before first use) maps
    positions to (tag << 32) | row of the kept rows; prev_k / prev_v [rows, D]
    (any leading shape) are the rows kept under prev_tag (0: none).
    row_counts [G, 2] int32 accumulates (hit rows, miss rows)."""
    _cuda(row_map, next_k, next_v, prev_k, prev_v, row_counts)
    if row_map.dtype != torch.int64 or row_map.dim() != 2:
        raise ValueError("row_map must be int64 [G, stride]")
    r = _lib.RowReuse()
    r.row_map, r.map_stride = row_map.data_ptr(), row_map.shape[1]
    r.next_tag, r.prev_tag = int(next_tag), int(prev_tag)
    if next_k is not None or next_v is not None:
        if next_k is None or next_v is None or next_k.dim() != 3 or next_k.shape != next_v.shape:
            raise ValueError("next_k / next_v must be [G, S, D]")
        r.next_k, r.next_v = next_k.data_ptr(), next_v.data_ptr()
        r.rows_stride = next_k.shape[1]
    if prev_tag:
        if prev_k is None or prev_v is None or prev_k.shape != prev_v.shape:
            raise ValueError("prev_tag needs prev_k and prev_v of one shape")
        r.prev_k, r.prev_v = prev_k.data_ptr(), prev_v.data_ptr()
        r.prev_rows = prev_k.numel() // prev_k.shape[-1]
    if row_counts is not None:
        if row_counts.dtype != torch.int32 or row_counts.shape != (row_map.shape[0], 2):
            raise ValueError("row_counts must be int32 [G, 2]")
        r.row_counts = row_counts.data_ptr()
    return r


def qkv_rope(hidden: torch.Tensor, w_q: torch.Tensor, w_k: torch.Tensor, w_v: torch.Tensor,
             cos: torch.Tensor, sin: torch.Tensor, *, q_out: torch.Tensor | None = None,
             k_out: torch.Tensor | None = None, v_out: torch.Tensor | None = None):
    """Decode-layer front end (tw_qkv_rope): hidden [H] and the nn.Linear weights
    w_q [n_q*128, H], w_k / w_v [n_kv*128, H] -> q [n_q, 128] (rotated), k
    [n_kv, 128] (rotated), v [n_kv, 128]; cos / sin [128] of the token's position."""
    _cuda(hidden, w_q, w_k, w_v, cos, sin, q_out, k_out, v_out)
    dt = hidden.dtype
    if any(t.dtype != dt for t in (w_q, w_k, w_v, cos, sin)):
        raise ValueError("hidden, weights and cos / sin must share one dtype")
    H = hidden.numel()
    if w_q.shape[1] != H or w_k.shape != w_v.shape or w_k.shape[1] != H or \
            w_q.shape[0] % HEAD_DIM or w_k.shape[0] % HEAD_DIM or cos.numel() != HEAD_DIM or \
            sin.numel() != HEAD_DIM:
        raise ValueError("weights must be [heads*128, hidden], cos / sin [128]")
    n_q, n_kv = w_q.shape[0] // HEAD_DIM, w_k.shape[0] // HEAD_DIM
    q_out = q_out if q_out is not None else torch.empty((n_q, HEAD_DIM), dtype=dt, device=hidden.device)
    k_out = k_out if k_out is not None else torch.empty((n_kv, HEAD_DIM), dtype=dt, device=hidden.device)
    v_out = v_out if v_out is not None else torch.empty((n_kv, HEAD_DIM), dtype=dt, device=hidden.device)
    _lib.check(lib().tw_qkv_rope(
        _ptr(hidden), _ptr(w_q), _ptr(w_k), _ptr(w_v), H, n_q, n_kv, HEAD_DIM, _ptr(cos), _ptr(sin),
        _kv_code(dt), _ptr(q_out), _ptr(k_out), _ptr(v_out), _stream(hidden.device)), "qkv_rope")
    return q_out, k_out, v_out
