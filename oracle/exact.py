"""ctypes bindings of oracle/exact.c.  TEST INFRASTRUCTURE ONLY.

numpy in, numpy out.  16-bit K/V values travel as their int16/uint16 bit patterns
(dtype code 0 = fp16, 1 = bf16).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "_build/liboracle.so"], cwd=HERE, check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        P = ctypes.c_void_p
        i64 = ctypes.c_int64
        i32 = ctypes.c_int
        L.orc_quest_page_metadata.argtypes = [P, i64, i32, i32, i32, i32, P, P]
        L.orc_quest_page_metadata.restype = i32
        L.orc_int4_pack.argtypes = [P, i64, i32, i32, i32, i32, P, P, P]
        L.orc_int4_pack.restype = None
        L.orc_quest_score.argtypes = [P, P, P, i32, i32, i32, i64, i32, P]
        L.orc_quest_score.restype = None
        L.orc_topk_pages.argtypes = [P, i32, i32, i32, P]
        L.orc_topk_pages.restype = None
        L.orc_int4_qk.argtypes = [P, P, P, P, i64, P, i32, i32, i32, i32, i32, i32, i32, P]
        L.orc_int4_qk.restype = None
        L.orc_top_p_union.argtypes = [P, P, i32, i32, i32, i32, i32, ctypes.c_double, i64, i64,
                                      i64, P, i64, P, P, P]
        L.orc_top_p_union.restype = i32
        L.orc_det_exp.argtypes = [ctypes.c_double]
        L.orc_det_exp.restype = ctypes.c_double
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _u16(a) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype.itemsize != 2:
        raise ValueError("expected 16-bit K/V bit patterns")
    return a.view(np.uint16)


def quest_page_metadata(keys, sink: int, block: int, dtype: int):
    """keys [L, D] bits -> (page_min, page_max) [(L-sink)//block, D] bits."""
    keys = _u16(keys)
    L, D = keys.shape
    pages = max(0, (L - sink) // block) if L > sink else 0
    pmin = np.zeros((pages, D), np.uint16)
    pmax = np.zeros((pages, D), np.uint16)
    lib().orc_quest_page_metadata(_p(keys), L, D, sink, block, dtype, _p(pmin), _p(pmax))
    return pmin, pmax


def int4_pack(keys, group: int, dtype: int, scale_div: int):
    """keys [N, 128] bits -> packed [N, 64] u8, scale/minimum [N, 128/group] bits."""
    keys = _u16(keys)
    n, d = keys.shape
    packed = np.zeros((n, d // 2), np.uint8)
    scale = np.zeros((n, d // group), np.uint16)
    minimum = np.zeros((n, d // group), np.uint16)
    lib().orc_int4_pack(_p(keys), n, d, group, dtype, scale_div, _p(packed), _p(scale), _p(minimum))
    return packed, scale, minimum


def quest_score(q, pmin, pmax, dtype: int):
    """q [G,R,128] f32; pmin/pmax [G,P,128] bits -> scores [G,R,P] f32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    pmin, pmax = _u16(pmin), _u16(pmax)
    G, R, _ = q.shape
    P = pmin.shape[1]
    out = np.zeros((G, R, P), np.float32)
    lib().orc_quest_score(_p(q), _p(pmin), _p(pmax), G, R, P, P * 128, dtype, _p(out))
    return out


def topk_pages(scores, k: int):
    scores = np.ascontiguousarray(scores, dtype=np.float32)
    shape = scores.shape
    rows = int(np.prod(shape[:-1]))
    out = np.zeros((rows, k), np.int32)
    lib().orc_topk_pages(_p(scores), rows, shape[-1], k, _p(out))
    return out.reshape(*shape[:-1], k)


def int4_qk(q, packed, scale, minimum, pages, block: int, sink: int, group: int, dtype: int):
    """q [G,R,128]; packed [G,S,64]; scale/minimum [G,S,ng] bits; pages [G,R,b0] -> [G,R,b0*block]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scale, minimum = _u16(scale), _u16(minimum)
    pages = np.ascontiguousarray(pages, dtype=np.int32)
    G, R, _ = q.shape
    b0 = pages.shape[-1]
    out = np.zeros((G, R, b0 * block), np.float32)
    lib().orc_int4_qk(_p(q), _p(packed), _p(scale), _p(minimum), packed.shape[1], _p(pages), G, R,
                      b0, block, sink, group, dtype, _p(out))
    return out


def top_p_union(logits, pages, block: int, sink: int, top_p: float, old_length: int,
                sink_end: int, recent_start: int):
    """-> (unions list[G] int32 ascending, head_count [G,R], head_pos list[G][R])."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    pages = np.ascontiguousarray(pages, dtype=np.int32)
    G, R, n = logits.shape
    b0 = pages.shape[-1]
    stride = max(1, old_length)
    union_pos = np.zeros((G, stride), np.int32)
    union_count = np.zeros(G, np.int32)
    head_count = np.zeros((G, R), np.int32)
    head_pos = np.zeros((G, R, n), np.int32)
    bad = lib().orc_top_p_union(_p(logits), _p(pages), G, R, b0, block, sink, float(top_p),
                                old_length, sink_end, recent_start, _p(union_pos), stride,
                                _p(union_count), _p(head_count), _p(head_pos))
    unions = [union_pos[g, : union_count[g]].copy() for g in range(G)]
    heads = [[head_pos[g, r, : head_count[g, r]].copy() for r in range(R)] for g in range(G)]
    return unions, head_count, heads, bad


def det_exp(x: float) -> float:
    return lib().orc_det_exp(float(x))
