"""ctypes binding of the C ABI (include/twilight_b200.h).

The library is the only compute path: there is no CPU fallback.  Loading
fails loudly when libtwilight_b200.so is absent.  Status codes map to the
exception types the reference raises: ValueError for bad shapes/arguments and
invalid row indices (hi/cpu_kv_gather.py:35-36), RuntimeError for CUDA and
capacity errors (hi/quest_offload_cache.py:104-106).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtwilight_b200.so"

TW_OK = 0
TW_ERR_INVALID_INDEX = 1
TW_ERR_BAD_ARG = 2
TW_ERR_CAPACITY = 3
TW_ERR_ORDER = 4
TW_ERR_CUDA = 5
TW_ERR_TIMEOUT = 6
TW_ERR_UNSUPPORTED = 7

TW_F16 = 0
TW_BF16 = 1
TW_F32 = 2

P = ctypes.c_void_p
I32 = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t
DBL = ctypes.c_double
FLT = ctypes.c_float

I32T = ctypes.c_int32


class DecodeLayerArgs(ctypes.Structure):
    """tw_decode_layer_args of include/twilight_b200.h (same field order and types)."""

    _fields_ = [
        ("slab_k", P), ("slab_v", P), ("entry_dirs", P), ("n_entries", I64), ("max_len", I64), ("first_entry", I32T), ("groups", I32T),
        ("heads_per_group", I32T), ("dtype", I32T), ("page_min", P), ("page_max", P),
        ("page_capacity", I64), ("n_pages", I32T), ("packed", P), ("scale", P), ("minimum", P),
        ("int4_group_size", I32T), ("sink", I32T), ("block_size", I32T), ("b0_pages", I32T),
        ("top_p", DBL), ("old_length", I64), ("sink_end", I64), ("recent_start", I64), ("q", P),
        ("k_new", P), ("v_new", P), ("out", P), ("out_dtype", I32T), ("append", I32T),
        ("pages", P), ("union_pos", P), ("pos_stride", I64), ("union_count", P),
        ("head_count", P), ("head_pos", P), ("error_flag", P), ("select_workspace", P),
        ("select_workspace_bytes", SZ), ("attn_workspace", P), ("attn_workspace_bytes", SZ),
        ("max_rows_per_group", I32T), ("reuse", P), ("stage_k", P), ("stage_v", P),
        ("stage_rows", I64),
    ]


class RowReuse(ctypes.Structure):
    """tw_row_reuse of include/twilight_b200.h (previous-token row reuse)."""

    _fields_ = [
        ("row_map", P), ("map_stride", I64), ("prev_tag", ctypes.c_uint32),
        ("next_tag", ctypes.c_uint32), ("prev_k", P), ("prev_v", P), ("prev_rows", I64),
        ("next_k", P), ("next_v", P), ("rows_stride", I64), ("row_counts", P),
    ]


# name -> (restype, argtypes); mirrors include/twilight_b200.h
SIGNATURES = {
    "tw_status_string": (ctypes.c_char_p, [I32]),
    "tw_last_cuda_error": (I32, []),
    "tw_abi_version": (I32, []),
    "tw_host_alloc_mapped": (I32, [SZ, ctypes.POINTER(P), ctypes.POINTER(P)]),
    "tw_host_alloc_mapped_numa": (I32, [SZ, I32, ctypes.POINTER(P), ctypes.POINTER(P),
                                        ctypes.POINTER(I32T)]),
    "tw_host_numa_node": (I32, [P, ctypes.POINTER(I32T)]),
    "tw_host_free": (I32, [P]),
    "tw_slab_write_rows": (I32, [P, I64, P, I64, I32, I64, I64, P]),
    "tw_host_device_pointer": (I32, [P, ctypes.POINTER(P)]),
    "tw_quest_page_metadata": (I32, [P, I64, I32, I32, I32, I32, I32, I32, I32, P, P, I64, P]),
    "tw_int4_pack": (I32, [P, I64, I32, I64, I32, I32, I32, P, P, P, I64, I64, P]),
    "tw_int4_pack_ex": (I32, [P, I64, I32, I64, I32, I32, I32, P, P, P, I64, I64, I32, P]),
    "tw_quest_score": (I32, [P, P, P, I32, I32, I32, I64, I32, I32, P, P]),
    "tw_topk_pages": (I32, [P, I32, I32, I32, P, P]),
    "tw_int4_qk": (I32, [P, P, P, P, I64, P, I32, I32, I32, I32, I32, I32, I32, I32, P, P]),
    "tw_top_p_union": (I32, [P, P, I32, I32, I32, I32, I32, DBL, I64, I64, I64, P, I64, P, P, P,
                             P, P]),
    "tw_select_layer_workspace_size": (SZ, [I32, I32, I32, I32, I32]),
    "tw_select_layer": (I32, [P, P, P, I64, I32, P, P, P, I64, I32, I32, I32, I32, I32, I32, I32,
                              I32, DBL, I64, I64, I64, P, P, I64, P, P, P, P, P, SZ, P]),
    "tw_gather_kv": (I32, [P, P, P, P, P, I64, I64, I64, P, P]),
    "tw_gather_union": (I32, [P, P, P, I64, I64, I32, I32, I64, P, I64, P, P, P, I32, I32, P, P, I64, P,
                              P, ctypes.POINTER(RowReuse), P]),
    "tw_gather_quest_heads": (I32, [P, P, P, I64, I64, I32, I32, I32, I64, I64, I64, I32, I32, P, I32, P,
                                    P, I32, I32, P, P, P, P]),
    "tw_append_token": (I32, [P, P, P, I64, I64, I32, I32, I64, P, P, I32, I32, I32, I32, P, P, I64, P, P,
                              P, I32, P]),
    "tw_decode_attention_workspace_size": (SZ, [I32, I32, I32, I32]),
    "tw_decode_attention": (I32, [P, P, P, P, I32, I32, I32, I32, I32, FLT, P, I32, P, P, SZ, P]),
    "tw_attend_union": (I32, [P, P, P, I64, I64, I32, I32, I64, P, I64, P, P, P, P, I32, I32, I32, I32, FLT,
                              P, I32, P, P, P, SZ, ctypes.POINTER(RowReuse), P]),
    "tw_twilight_decode_layer": (I32, [ctypes.POINTER(DecodeLayerArgs), P]),
    "tw_decode_layer_args_size": (SZ, []),
    "tw_row_reuse_size": (SZ, []),
    "tw_qkv_rope": (I32, [P, P, P, P, I32, I32, I32, I32, P, P, I32, P, P, P, P]),
    "tw_decode_attention_noalloc": (I32, [P, P, P, P, I32, I32, I32, I32, I32, FLT, P, I32, P, P]),
}

_lib = None


class TwilightError(RuntimeError):
    pass


def load():
    """Load the extension or raise (no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is missing: build it with "
            "`python twilight-cpu-gpu-offloading_b200/build.py` (there is no CPU fallback)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().tw_status_string(status).decode()


def check(status: int, what: str = "") -> None:
    if status == TW_OK:
        return
    msg = f"{what}: {status_string(status)}" if what else status_string(status)
    if status == TW_ERR_CUDA:
        msg += f" (cudaError {load().tw_last_cuda_error()})"
        raise TwilightError(msg)
    if status in (TW_ERR_INVALID_INDEX, TW_ERR_BAD_ARG, TW_ERR_ORDER, TW_ERR_UNSUPPORTED):
        raise ValueError(msg)
    if status == TW_ERR_TIMEOUT:
        raise TimeoutError(msg)
    raise RuntimeError(msg)


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
