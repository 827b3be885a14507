"""Runs the reference's own CPU code for the sparse decode layer-step.
TEST / BASELINE INFRASTRUCTURE ONLY: used by tests/golden/make_golden.py (to
dump golden vectors) and by bench.py's CPU baseline leg and reference arm (to
time the reference), never by the product.

The reference's caches need CUDA in their constructors, so instances are made
with __new__ and given the attributes their selection path reads; then the
reference's own _build_metadata (hi/twilight_offload_cache.py:925-936) and
prepare_layer_selection (hi/twilight_offload_cache.py:996-1843) run on
device='cpu' with qk_backend='pytorch' and the GPU-compact union semantics
(gpu_compact_gqa_union=True), as the reference's CPU execution of that code.

The reference package (a directory holding ``headinfer/``) is looked up in
this order: $TW_REFERENCE_PKG, then ``baseline/_ref`` beside this repository
(the pip --target install of the reference).  ``source/headinfer`` under a
reference checkout named by $TW_REFERENCE_ROOT also works.
"""

from __future__ import annotations

import importlib
import os
import sys
from collections import defaultdict
from pathlib import Path
from typing import Optional

import torch

REPO = Path(__file__).resolve().parents[1]


def reference_package_dir() -> Optional[Path]:
    cands = []
    if os.environ.get("TW_REFERENCE_PKG"):
        cands.append(Path(os.environ["TW_REFERENCE_PKG"]))
    cands.append(REPO / "baseline" / "_ref")
    if os.environ.get("TW_REFERENCE_ROOT"):
        cands.append(Path(os.environ["TW_REFERENCE_ROOT"]) / "source" / "headinfer")
    for c in cands:
        if (c / "headinfer" / "twilight_offload_cache.py").exists():
            return c
    return None


def import_reference(module: str = "twilight_offload_cache"):
    """The reference module headinfer.<module>, or None when the package is absent."""
    d = reference_package_dir()
    if d is None:
        return None
    if str(d) not in sys.path:
        sys.path.insert(0, str(d))
    try:
        return importlib.import_module(f"headinfer.{module}")
    except Exception:
        return None


def make_ref_cache(mod, cls_name: str, *, entries: int, max_len: int, heads: int, dtype, sink: int,
                   recent: int, block: int, **extra):
    """A reference cache instance on device='cpu' with the attributes its
    selection path reads (hi/quest_offload_cache.py:55-160 sets them in the
    CUDA-only constructor)."""
    from headinfer.slab_cache import SequentialCacheState, SlabGeometry

    cls = getattr(mod, cls_name)
    c = cls.__new__(cls)
    c.geometry = SlabGeometry(num_entries=entries, batch_size=1, max_cache_len=max_len, head_dim=128)
    c.dtype = dtype
    c.device = torch.device("cpu")
    c.allocated_capacity = max_len
    c.num_query_heads_per_kv = heads
    c.sink_tokens = sink
    c.recent_tokens = recent
    c.block_size = block
    c.selection_interval = 1
    c.layer_batched_selection = True
    c._bookkeeping = SequentialCacheState(entries, max_len)
    c._logical_lengths = c._bookkeeping.logical_lengths
    c._page_min = [None] * entries
    c._page_max = [None] * entries
    c._prompt_length = None
    c._cached_selected_pages = [None] * entries
    c._layer_prepared_entries = set()
    c._capture_selection_trace = False
    c._selection_trace = []
    c.metrics_enabled = False
    c.metrics = defaultdict(float)
    c._timing_events = []
    for k, v in extra.items():
        setattr(c, k, v)
    return c


def make_twilight_cache(mod, *, groups: int, heads: int, max_len: int, dtype, sink: int, recent: int,
                        block: int, b0_tokens: int, top_p: float, budget_trace: bool = False):
    """TwilightMatchedBudgetOffloadedCache in dynamic-budget mode, pytorch QK
    backend, GPU-compact GQA union semantics, every CUDA-only option off."""
    G = groups
    return make_ref_cache(
        mod, "TwilightMatchedBudgetOffloadedCache", entries=G, max_len=max_len, heads=heads,
        dtype=dtype, sink=sink, recent=recent, block=block, candidate_token_budget=b0_tokens,
        top_p=top_p, matched_budget_fraction=0.05, budget_mode="dynamic",
        gqa_groupwise_execution=True, detailed_selection_profile=False, qk_backend="pytorch",
        exact_scan_graph=False, exact_top_p_graph=False, fused_quest_score=False,
        reuse_quant_metadata=False, _layer_quant_metadata={}, fused_final_indices=False,
        gpu_compact_gqa_union=True, gpu_union_validate_cpu=False, cpu_bitmap_union=False,
        post_selection_pipeline=False, resident_zero_copy=False,
        resident_precompute_gpu_mapping=False, _resident_zero_copy_placeholder_active=False,
        _capture_budget_trace=budget_trace, _budget_trace=[],
        _quant_key_packed=[None] * G, _quant_key_scale=[None] * G, _quant_key_minimum=[None] * G,
        _cached_twilight_positions=[None] * G, _cached_twilight_group_positions=[None] * G,
        _cached_twilight_per_q_lengths=[None] * G, _gpu_group_membership=None,
        _post_selection_pending={}, _post_selection_host_starts={})


class ReferenceLayerStep:
    """One layer's sparse decode step run by the reference's own CPU code:
    prepare_layer_selection (Quest score, top-k, per-token INT4 estimate,
    top-p, GQA union), then the flat host-row gather and the reference's
    SDPA-math decode attention (hi/decode_reference_attention.py:18-69) once
    per KV group over its union and the current token.

    keys / values: [G, L, D] host tensors (the prompt).  The reference cache
    quantises keys per token (INT4 scale over all 128 channels,
    hi/twilight_offload_cache.py:25-37); it has no group-wise mode."""

    def __init__(self, keys: torch.Tensor, values: torch.Tensor, *, heads: int, sink: int,
                 recent: int, block: int, b0_tokens: int, top_p: float) -> None:
        mod = import_reference("twilight_offload_cache")
        if mod is None:
            raise RuntimeError("the reference package is not available")
        from headinfer.decode_reference_attention import sdpa_math_decode_attention

        self._attention = sdpa_math_decode_attention
        G, L, D = keys.shape
        self.G, self.R, self.L = G, heads, L
        self.cache = make_twilight_cache(mod, groups=G, heads=heads, max_len=L + 8,
                                         dtype=keys.dtype, sink=sink, recent=recent, block=block,
                                         b0_tokens=b0_tokens, top_p=top_p)
        self.cache._prompt_length = L
        for e in range(G):
            self.cache._logical_lengths[e] = L
            self.cache._build_metadata(e, keys[e].view(1, 1, L, D))
        self.k_rows = keys.reshape(G * L, D).contiguous()
        self.v_rows = values.reshape(G * L, D).contiguous()

    def select(self, q: torch.Tensor) -> list[torch.Tensor]:
        """q [G, R, D] -> the G sorted union position lists (int64)."""
        R = self.R
        self.cache.prepare_layer_selection(entries=list(range(self.G)),
                                           queries=[q[g].view(1, R, 1, 128) for g in range(self.G)])
        return [self.cache._cached_twilight_group_positions[g] for g in range(self.G)]

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, gather_fn=None):
        """One layer-step: q [G,R,D], new K/V [G,D] -> (attention [G,R,D] fp32, unions).
        gather_fn(rows) -> (K rows, V rows) defaults to torch.index_select over
        the flat host rows (hi/twilight_offload_cache.py:3017-3020)."""
        unions = self.select(q)
        rows = torch.cat([u + g * self.L for g, u in enumerate(unions)])
        if gather_fn is None:
            k, v = self.k_rows.index_select(0, rows), self.v_rows.index_select(0, rows)
        else:
            k, v = gather_fn(rows)
        outs, off = [], 0
        for g, u in enumerate(unions):
            n = u.numel()
            kk = torch.cat((k[off:off + n], k_new[g:g + 1])).float()
            vv = torch.cat((v[off:off + n], v_new[g:g + 1])).float()
            o = self._attention(q[g].float().view(1, 1, self.R, 128), kk.view(1, -1, 1, 128),
                                vv.view(1, -1, 1, 128), None, 1)
            outs.append(o[0, 0])
            off += n
        return torch.stack(outs), unions
