"""The reuse oracle (oracle/reuse.py) pinned against the reference's own CPU
hit/miss mapping (map_resident_rows and its attention-layout variant,
hi/resident_mapping.cpp:6-95, compiled into oracle/_ref by oracle/Makefile),
plus the cache options' validation (hi/twilight_offload_cache.py:215-262)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import reuse

needs_ref = pytest.mark.skipif(not reuse.REF_LIB.exists(),
                               reason="oracle/_ref/libref_resident_mapping.so not built")


def _case(seed, groups, capacity, sizes):
    rng = np.random.default_rng(seed)
    prev, cur = [], []
    for g in range(groups):
        p = np.sort(rng.choice(capacity - 1, size=sizes[g][0], replace=False))
        shared = rng.choice(p, size=min(len(p), sizes[g][1] // 2), replace=False) if len(p) else p
        c = np.unique(np.concatenate((shared, rng.choice(capacity, size=sizes[g][1], replace=False))))
        cur.append(np.sort(c[: sizes[g][1]]).astype(np.int64))
        prev.append(p.astype(np.int64))
    return prev, cur


@needs_ref
@pytest.mark.parametrize("attention_layout", [False, True])
@pytest.mark.parametrize("seed", range(6))
def test_resident_map_matches_reference(seed, attention_layout):
    groups = 1 + seed % 8
    capacity = 50 + 997 * seed
    sizes = [((seed + g) * 37 % (capacity // 2), (seed * 7 + g * 13) % (capacity // 2))
             for g in range(groups)]
    sizes[0] = (0, sizes[0][1])  # an empty previous union
    prev, cur = _case(seed, groups, capacity, sizes)
    entries = [3 * g + seed for g in range(groups)]
    ours = reuse.resident_map(prev, cur, entries, capacity, attention_layout=attention_layout)
    ref = reuse.reference_map_rows(prev, cur, entries, capacity, attention_layout=attention_layout)
    for a, b in zip(ours, ref):
        np.testing.assert_array_equal(a, b)
    hits = reuse.group_hit_miss(prev, cur)
    assert hits[:, 0].sum() == len(ours[0]) and hits[:, 1].sum() == len(ours[2])


@needs_ref
def test_resident_map_errors_match_reference():
    prev = [np.array([1, 5], dtype=np.int64)]
    for cur in ([np.array([9], dtype=np.int64)], [np.array([-1], dtype=np.int64)]):
        with pytest.raises(ValueError):
            reuse.resident_map(prev, cur, [0], 8)
        with pytest.raises(ValueError):
            reuse.reference_map_rows(prev, cur, [0], 8)
    empty = reuse.resident_map([np.zeros(0, np.int64)], [np.zeros(0, np.int64)], [0], 8)
    assert all(a.size == 0 for a in empty[:4])


def test_previous_token_extension():
    """The previous step's token (position previous_length) is a hit on the row
    after the previous union in the attention layout."""
    prev = [np.array([0, 4, 7], dtype=np.int64), np.array([2], dtype=np.int64)]
    cur = [np.array([0, 5, 9], dtype=np.int64), np.array([2, 9], dtype=np.int64)]
    hs, hd, mr, md, _ = reuse.resident_map(prev, cur, [0, 1], 16, attention_layout=True,
                                           previous_length=9)
    assert hs.tolist() == [0, 3, 4, 5] and hd.tolist() == [0, 2, 4, 5]
    assert mr.tolist() == [5] and md.tolist() == [1]
    np.testing.assert_array_equal(reuse.group_hit_miss(prev, cur, 9), [[2, 1], [2, 0]])
    with pytest.raises(ValueError):
        reuse.resident_map(prev, cur, [0, 1], 16, previous_length=9)


def test_resident_option_validation(tw):
    from importlib import import_module

    cache_mod = import_module("twilight-cpu-gpu-offloading_b200.cache")
    check = cache_mod._check_resident_options
    check(True, {"resident_zero_copy": True, "resident_mapping_backend": "gpu_bitmap",
                 "resident_hit_copy_backend": "triton"})
    check(False, {})
    with pytest.raises(ValueError, match="resident zero-copy requires resident cache"):
        check(False, {"resident_zero_copy": True})
    with pytest.raises(ValueError, match="unknown"):
        check(True, {"resident_mapping_backend": "bogus"})
    with pytest.raises(ValueError, match="requires the previous-token resident cache"):
        check(False, {"resident_hit_copy_backend": "triton"})
    with pytest.raises(ValueError, match="compact hit indices"):
        check(True, {"resident_mapping_backend": "native_compact"})
    with pytest.raises(ValueError, match="contiguous snapshot"):
        check(True, {"resident_snapshot_backend": "contiguous"})
