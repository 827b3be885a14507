"""Previous-token row reuse: the hit/miss mapping.  TEST INFRASTRUCTURE ONLY.

Restates map_rows (hi/resident_mapping.cpp:6-53), which the GPU bitmap path
(hi/resident_gpu_mapping.py:14-127) computes identically: for each group, a
current union position that is also in the previous step's union is a hit
whose source is its rank there (offset by the previous groups' rows, plus one
current-token row per group in the attention layout); every other position is
a miss read from the host slab at entry * capacity + position.  Destinations
are attention rows: group g's rows start at sum_{h<g}(|current_h| + 1).

`previous_length` adds the sm_100a path's extension: the previous step's own
token (position previous_length, kept on the device after its union rows) is
also a hit, at source previous_offset + |previous_g|.

`reference_map_rows` calls the reference's compiled map_resident_rows
(oracle/_ref/libref_resident_mapping.so, built from its sources by
oracle/Makefile) so the restatement is pinned against it.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

REF_LIB = Path(__file__).resolve().parent / "_ref" / "libref_resident_mapping.so"


def resident_map(previous, current, entries, capacity: int, *, attention_layout: bool = False,
                 previous_length: int | None = None):
    """(hit_sources, hit_destinations, miss_rows, miss_destinations,
    history_destinations) as int64 arrays; ValueError for invalid positions
    (the reference's nonzero status)."""
    if capacity <= 0 or not entries:
        raise ValueError("invalid capacity or groups")
    if previous_length is not None and not attention_layout:
        raise ValueError("the previous token's row exists only in the attention layout")
    hit_src, hit_dst, miss_rows, miss_dst, hist_dst = [], [], [], [], []
    prev_off = att_off = 0
    for g, entry in enumerate(entries):
        prev = np.asarray(previous[g], dtype=np.int64)
        cur = np.asarray(current[g], dtype=np.int64)
        if entry < 0 or ((prev < 0) | (prev >= capacity)).any() or \
                ((cur < 0) | (cur >= capacity)).any():
            raise ValueError("invalid resident positions")
        rank = {int(p): r for r, p in enumerate(prev)}
        for row, pos in enumerate(cur.tolist()):
            dst = att_off + row
            hist_dst.append(dst)
            src = rank.get(pos, -1)
            if src < 0 and previous_length is not None and pos == previous_length:
                src = len(prev)
            if src >= 0:
                hit_src.append(prev_off + src)
                hit_dst.append(dst)
            else:
                miss_rows.append(entry * capacity + pos)
                miss_dst.append(dst)
        prev_off += len(prev) + (1 if attention_layout else 0)
        att_off += len(cur) + 1
    as64 = lambda x: np.asarray(x, dtype=np.int64)
    return as64(hit_src), as64(hit_dst), as64(miss_rows), as64(miss_dst), as64(hist_dst)


def group_hit_miss(previous, current, previous_length: int | None = None) -> np.ndarray:
    """[G, 2] (hit rows, miss rows) per group, as the device counters report."""
    out = np.zeros((len(current), 2), dtype=np.int64)
    for g in range(len(current)):
        prev = set(int(p) for p in np.asarray(previous[g]).tolist())
        if previous_length is not None:
            prev.add(int(previous_length))
        hits = sum(1 for p in np.asarray(current[g]).tolist() if int(p) in prev)
        out[g] = (hits, len(current[g]) - hits)
    return out


def reference_map_rows(previous, current, entries, capacity: int, *,
                       attention_layout: bool = False):
    """The reference's own map_resident_rows / ..._compact_attention_layout."""
    lib = ctypes.CDLL(str(REF_LIB))
    fn = (lib.map_resident_rows_compact_attention_layout if attention_layout
          else lib.map_resident_rows)
    fn.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 2 + [ctypes.c_void_p] * 7
    fn.restype = ctypes.c_int
    groups = len(entries)
    prev = [np.ascontiguousarray(p, dtype=np.int64) for p in previous]
    cur = [np.ascontiguousarray(c, dtype=np.int64) for c in current]
    total = sum(c.size for c in cur)
    hit_t = np.int32 if attention_layout else np.int64
    outs = [np.zeros(max(total, 1), dtype=hit_t), np.zeros(max(total, 1), dtype=hit_t)]
    outs += [np.zeros(max(total, 1), dtype=np.int64) for _ in range(3)]
    ptrs = ctypes.c_void_p * groups
    lens = ctypes.c_int64 * groups
    hits = ctypes.c_int64()
    misses = ctypes.c_int64()
    code = fn(ptrs(*(p.ctypes.data for p in prev)), ptrs(*(c.ctypes.data for c in cur)),
              lens(*(p.size for p in prev)), lens(*(c.size for c in cur)),
              lens(*(int(e) for e in entries)), groups, capacity,
              *(o.ctypes.data for o in outs), ctypes.byref(hits), ctypes.byref(misses))
    if code:
        raise ValueError(f"invalid resident positions (native error {code})")
    h, m = hits.value, misses.value
    return (outs[0][:h].astype(np.int64), outs[1][:h].astype(np.int64), outs[2][:m],
            outs[3][:m], outs[4][:total])
