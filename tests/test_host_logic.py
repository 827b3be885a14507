"""Host-side logic that needs no GPU: slab geometry, strict entry order, window
arithmetic and constructor validation (hi/slab_cache.py:37-120,
hi/twilight_offload_cache.py:1018-1071, hi/quest_offload_cache.py:46-86)."""

from __future__ import annotations

import math

import pytest
import torch

from oracle import torch_ref


def test_slab_geometry(tw):
    g = tw.SlabGeometry(num_entries=4, batch_size=1, max_cache_len=32, head_dim=128)
    assert g.elements_per_entry == 32 * 128
    assert g.total_elements == 2 * 4 * 32 * 128
    assert g.bounds("key", 0) == (0, 4096)
    assert g.bounds("value", 0) == (4 * 4096, 5 * 4096)
    assert g.bounds("value", 3) == (7 * 4096, 8 * 4096)
    assert g.tensor_shape() == (1, 1, 32, 128)
    with pytest.raises(ValueError):
        g.bounds("query", 0)
    with pytest.raises(IndexError):
        g.bounds("key", 4)
    with pytest.raises(ValueError):
        tw.SlabGeometry(num_entries=0, batch_size=1, max_cache_len=1, head_dim=1)


def test_sequential_state_order_and_capacity(tw):
    s = tw.SequentialCacheState(3, 10)
    assert s.advance(0, 4) == (0, 4) and s.seen_tokens == 4
    with pytest.raises(ValueError, match="strict sequential"):
        s.advance(2, 4)
    s.advance(1, 4)
    s.advance(2, 4)
    assert s.uniform and s.expected_next_entry == 0
    s.advance(0, 6)
    with pytest.raises(RuntimeError, match="capacity"):
        s.advance(1, 7)
    with pytest.raises(ValueError):
        s.preview(1, 0)


@pytest.mark.parametrize("L", [0, 1, 16, 63, 64, 65, 200, 319, 320, 336, 4096, 32768])
def test_window_arithmetic(L):
    w = torch_ref.window(L, sink=64, recent=256, block=16, candidate_token_budget=4096)
    sink_end = min(64, L)
    recent_start = max(sink_end, L - 255)
    assert w.sink_end == sink_end and w.recent_start == recent_start
    assert w.candidate_pages == max(0, recent_start - sink_end) // 16
    assert w.b0_pages == min(w.candidate_pages, max(1, math.ceil(4096 / 16)))
    protected = sink_end + (L - recent_start)
    assert protected <= L


def test_constructor_requires_cuda_without_gpu(tw):
    if torch.cuda.is_available():
        pytest.skip("CUDA present")
    with pytest.raises(ValueError, match="CUDA"):
        tw.TwilightMatchedBudgetOffloadedCache(
            num_cache_entries=2, max_cache_len=64, head_dim=128, num_query_heads_per_kv=4,
            dtype=torch.float16, device="cuda", layer_batched_selection=True,
            gqa_groupwise_execution=True, budget_mode="dynamic")


def test_twilight_kwarg_validation_is_host_side(tw):
    base = dict(num_cache_entries=2, max_cache_len=64, head_dim=128, num_query_heads_per_kv=4,
                dtype=torch.float16, device="cuda")
    cls = tw.TwilightMatchedBudgetOffloadedCache
    for bad, msg in ((dict(candidate_token_budget=0), "candidate_token_budget"),
                     (dict(top_p=0.0), "top_p"), (dict(top_p=1.5), "top_p"),
                     (dict(budget_mode="x"), "budget_mode"),
                     (dict(budget_mode="matched"), "matched"),
                     (dict(qk_backend="x"), "backend"),
                     (dict(qk_backend="triton"), "layer-batched"),
                     (dict(gqa_groupwise_execution=True), "layer-batched"),
                     (dict(int4_group_size=16), "int4_group_size")):
        with pytest.raises(ValueError, match=msg):
            cls(**base, **bad)
