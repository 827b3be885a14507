"""Drop-in offload caches: the reference's operator API over the sm_100a kernels.

QuestTopKOffloadedCache mirrors hi/quest_offload_cache.py:23 (per-query-head
Quest pages) and TwilightMatchedBudgetOffloadedCache mirrors
hi/twilight_offload_cache.py:133 (Quest B0 -> INT4 QK -> top-p -> GQA union,
dynamic budget).  Same constructor keywords, method names, return tuples and
exception types; the full K/V history lives in a pinned, device-mapped host
slab and every selection, gather and attention step runs as CUDA kernels of
libtwilight_b200.so on the caller's current stream.  Selections stay on the
device: the only host synchronisation on the reference-compatible path is
the read of the G union lengths that update_layer_gqa_group_ragged must
return as Python ints; attend_layer needs none.
"""

from __future__ import annotations

import ctypes
import hashlib
import math
from collections import defaultdict
from typing import Any, Optional

import torch

from . import _lib, ops
from .slab import MappedHostSlab, SequentialCacheState, SlabGeometry

HEAD_DIM = ops.HEAD_DIM


def _contiguous_entries(entries: list[int]) -> int:
    first = entries[0]
    if list(entries) != list(range(first, first + len(entries))):
        raise ValueError("layer entries must be contiguous (layer * kv_heads + kv_head)")
    return first


class QuestTopKOffloadedCache:
    """Pinned-host full cache with per-query-head Quest top-k pages.

    hi/quest_offload_cache.py:23-1055.  Extra keywords (not in the reference):
    ``incremental_page_metadata`` (default False = the reference's candidate
    window capped at the prompt's pages, hi/twilight_offload_cache.py:1062-1069;
    True = pages completed by appended tokens become candidates) and
    ``resident_entries`` (entries whose K/V stay in GPU memory, HeadInfer's
    GPU-resident heads; all other entries live in the pinned, mapped host slab).
    Kernels find each entry's rows through a device directory [2, E] of row-0
    addresses, so resident and offloaded heads share one code path.
    ``host_numa_node`` ("auto" or a node id) pins the slab on that host NUMA
    node ("auto": the node closest to the cache's GPU) instead of the default
    cudaHostAlloc placement.
    """

    def __init__(self, *, num_cache_entries: int, max_cache_len: int, head_dim: int,
                 num_query_heads_per_kv: int, dtype: torch.dtype, device: torch.device | str,
                 sink_tokens: int = 64, recent_tokens: int = 256, block_size: int = 16,
                 budget_fraction: float = 0.05, selection_interval: int = 1,
                 max_selected_history_fraction: Optional[float] = None,
                 layer_batched_selection: bool = False, layer_flat_ragged_execution: bool = False,
                 sparse_gather_stabilized: bool = False,
                 per_head_varlen_attention_reference: bool = False,
                 incremental_page_metadata: bool = False,
                 resident_entries: Optional[Any] = None,
                 host_numa_node: Optional[Any] = None, **ignored: Any) -> None:
        device = torch.device(device)
        if device.type != "cuda" or not torch.cuda.is_available():
            raise ValueError("an operational CUDA device is required")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if sink_tokens < 0 or recent_tokens <= 0 or block_size <= 0:
            raise ValueError("invalid sink/recent/block configuration")
        if not 0.0 < budget_fraction <= 1.0:
            raise ValueError("budget_fraction must be in (0, 1]")
        if selection_interval <= 0:
            raise ValueError("selection_interval must be positive")
        if max_selected_history_fraction is None:
            max_selected_history_fraction = budget_fraction
        if not 0.0 < max_selected_history_fraction <= 1.0:
            raise ValueError("max_selected_history_fraction must be in (0, 1]")
        if num_query_heads_per_kv <= 0:
            raise ValueError("num_query_heads_per_kv must be positive")
        if head_dim != HEAD_DIM:
            raise ValueError(f"head_dim must be {HEAD_DIM} (the sm_100a kernels' tile)")
        if num_query_heads_per_kv > 8:
            raise ValueError("at most 8 query heads per KV head are supported")
        if dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("K/V dtype must be float16 or bfloat16")
        if layer_flat_ragged_execution and not layer_batched_selection:
            raise ValueError("layer-flat ragged execution requires layer-batched selection")
        if sparse_gather_stabilized and not layer_flat_ragged_execution:
            raise ValueError("stabilized sparse gather requires layer-flat ragged execution")
        _lib.load()  # fail loudly without the extension
        self.geometry = SlabGeometry(num_entries=num_cache_entries, batch_size=1,
                                     max_cache_len=max_cache_len, head_dim=head_dim)
        self.dtype = dtype
        self.device = device
        self._device_index = device.index
        self.allocated_capacity = max_cache_len
        self.num_query_heads_per_kv = num_query_heads_per_kv
        self.sink_tokens = sink_tokens
        self.recent_tokens = recent_tokens
        self.block_size = block_size
        self.budget_fraction = budget_fraction
        self.selection_interval = int(selection_interval)
        self.layer_batched_selection = bool(layer_batched_selection)
        self.layer_flat_ragged_execution = bool(layer_flat_ragged_execution)
        self.sparse_gather_stabilized = bool(sparse_gather_stabilized)
        self.per_head_varlen_attention_reference = bool(per_head_varlen_attention_reference)
        self.max_selected_history_fraction = max_selected_history_fraction
        self.incremental_page_metadata = bool(incremental_page_metadata)
        self.ignored_options = dict(ignored)
        self._bookkeeping = SequentialCacheState(num_cache_entries, max_cache_len)
        self._logical_lengths = self._bookkeeping.logical_lengths
        self._initialized = [False] * num_cache_entries
        self._seen_tokens = 0
        self._prompt_length: Optional[int] = None

        self._slab = MappedHostSlab(self.geometry, dtype, numa_node=host_numa_node)
        res = sorted(set(int(e) for e in (resident_entries or ())))
        if any(not 0 <= e < num_cache_entries for e in res):
            raise ValueError("resident_entries outside [0, num_cache_entries)")
        self.resident_entries = tuple(res)
        self._resident_index = {e: i for i, e in enumerate(res)}
        self._resident_kv = (torch.empty((2, len(res), max_cache_len, head_dim), dtype=dtype,
                                         device=device) if res else None)
        itemsize = torch.tensor([], dtype=dtype).element_size()
        entry_bytes = max_cache_len * head_dim * itemsize
        dirs = []
        for plane, base in ((0, self._slab.key_device_ptr), (1, self._slab.value_device_ptr)):
            for e in range(num_cache_entries):
                if e in self._resident_index:
                    dirs.append(self._resident_kv[plane, self._resident_index[e]].data_ptr())
                else:
                    dirs.append(base + e * entry_bytes)
        self._dirs = torch.tensor(dirs, dtype=torch.int64).view(2, num_cache_entries).to(device)
        self.page_capacity = max(1, math.ceil(max(0, max_cache_len - sink_tokens) / block_size))
        E, D = num_cache_entries, head_dim
        self._page_min = torch.empty((E, self.page_capacity, D), dtype=dtype, device=device)
        self._page_max = torch.empty_like(self._page_min)
        self._meta_pages = [0] * E  # prompt pages with metadata per entry
        self._meta_version = 0      # bumped whenever _meta_pages changes
        max_pages = math.ceil(max(0, max_cache_len - sink_tokens) / block_size)
        self.max_selected_tokens_per_query_head = min(
            max_cache_len,
            sink_tokens + recent_tokens
            + max(1, math.ceil(max_selected_history_fraction * max_pages)) * block_size)
        self._error_flag = torch.zeros(1, dtype=torch.int32, device=device)
        self._quest_pages: dict[int, tuple[Optional[torch.Tensor], int, int]] = {}
        self._quest_prepared: set[int] = set()
        self._last_query_head_lengths: list[Optional[tuple[int, ...]]] = [None] * E
        self._quest_pack: Optional[torch.Tensor] = None
        self._layer_bufs: dict[int, dict[str, Any]] = {}
        self._capture_selection_trace = False
        self._selection_trace: list[dict[str, Any]] = []
        self.metrics_enabled = False
        self.metrics: dict[str, float] = defaultdict(float)
        self._timing_events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []

    # ------------------------------------------------------------ construction --
    @classmethod
    def from_llama_model(cls, model: torch.nn.Module, **kwargs: Any):
        """hi/quest_offload_cache.py:175-190."""
        config = model.config
        parameter = next(model.parameters())
        return cls(
            num_cache_entries=config.num_hidden_layers * config.num_key_value_heads,
            head_dim=getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads,
            num_query_heads_per_kv=config.num_attention_heads // config.num_key_value_heads,
            dtype=parameter.dtype, device=parameter.device, **kwargs)

    # ------------------------------------------------------------------ views --
    def _host_tensor(self, kind: str, entry: int) -> torch.Tensor:
        return self._slab.entry(kind, entry)

    @property
    def _host_key_rows(self) -> torch.Tensor:
        return self._slab.rows[0].reshape(-1, self.geometry.head_dim)

    @property
    def _host_value_rows(self) -> torch.Tensor:
        return self._slab.rows[1].reshape(-1, self.geometry.head_dim)

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    # ---------------------------------------------------------------- metrics --
    def reset_metrics(self) -> None:
        self.metrics = defaultdict(float)
        self._timing_events = []

    def enable_metrics(self, enabled: bool = True) -> None:
        self.metrics_enabled = enabled
        if enabled:
            self.reset_metrics()

    def _phase_start(self) -> Optional[torch.cuda.Event]:
        if not self.metrics_enabled:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record(torch.cuda.current_stream(self.device))
        return ev

    def _phase_end(self, name: str, start: Optional[torch.cuda.Event]) -> None:
        if start is None:
            return
        end = torch.cuda.Event(enable_timing=True)
        end.record(torch.cuda.current_stream(self.device))
        self._timing_events.append((name, start, end))

    def resolve_metrics(self) -> dict[str, float]:
        self.synchronize()
        for name, start, end in self._timing_events:
            self.metrics[f"{name}_cuda_seconds"] += start.elapsed_time(end) / 1000.0
            self.metrics[f"{name}_event_intervals"] += 1
        self._timing_events = []
        return dict(self.metrics)

    def enable_selection_trace(self, enabled: bool = True) -> None:
        self._capture_selection_trace = bool(enabled)
        self._selection_trace = []

    def selection_trace(self) -> list[dict[str, Any]]:
        return list(self._selection_trace)

    # ------------------------------------------------------------ bookkeeping --
    def _check_error_flag(self) -> None:
        flag = int(self._error_flag.item())
        if flag:
            self._error_flag.zero_()
            _lib.check(flag, "device-side check")

    def _window(self, old_length: int) -> dict[str, int]:
        sink_end = min(self.sink_tokens, old_length)
        recent_start = max(sink_end, old_length - max(0, self.recent_tokens - 1))
        eligible = max(0, recent_start - sink_end)
        return dict(sink_end=sink_end, recent_start=recent_start, eligible=eligible,
                    candidate_pages=eligible // self.block_size)

    def _metadata_pages(self, entries: list[int], old_length: int) -> int:
        if self.incremental_page_metadata:
            return max(0, old_length - self.sink_tokens) // self.block_size if old_length > self.sink_tokens else 0
        return min(self._meta_pages[e] for e in entries)

    def _build_metadata(self, entry: int, key_states: torch.Tensor) -> None:
        """Quest page min/max of the prompt (hi/quest_offload_cache.py:276-289) plus
        the running min/max of the trailing partial page, continued on append."""
        self._build_metadata_entries(entry, key_states[0, 0].unsqueeze(0))

    def _build_metadata_entries(self, first: int, keys: torch.Tensor) -> None:
        """_build_metadata for entries first .. first + G - 1 at once; keys [G, S, D]."""
        keys = keys.contiguous()
        G, S = int(keys.shape[0]), int(keys.shape[1])
        complete = max(0, S - self.sink_tokens) // self.block_size if S > self.sink_tokens else 0
        if complete:
            _lib.check(_lib.load().tw_quest_page_metadata(
                keys.data_ptr(), S * HEAD_DIM, G, self.sink_tokens, self.block_size, HEAD_DIM,
                ops._kv_code(self.dtype), 0, complete,
                self._page_min[first].data_ptr(), self._page_max[first].data_ptr(),
                self.page_capacity * HEAD_DIM, self._stream()), "quest_page_metadata")
        partial = S - self.sink_tokens - complete * self.block_size if S > self.sink_tokens else 0
        if partial > 0 and complete < self.page_capacity:
            off = complete * HEAD_DIM * keys.element_size()
            _lib.check(_lib.load().tw_quest_page_metadata(
                keys.data_ptr(), S * HEAD_DIM, G, self.sink_tokens + complete * self.block_size,
                partial, HEAD_DIM, ops._kv_code(self.dtype), 0, 1,
                self._page_min[first].data_ptr() + off, self._page_max[first].data_ptr() + off,
                self.page_capacity * HEAD_DIM, self._stream()), "quest_page_metadata")
        for e in range(first, first + G):
            self._meta_pages[e] = complete
        self._meta_version += 1

    def prefill_layer(self, *, key_states: torch.Tensor, value_states: torch.Tensor,
                      entries: list[int]) -> None:
        """Prefill of one layer's KV heads at once: the per-entry update() of every
        entry in `entries` (same results), with the Quest metadata (and INT4
        codes) of all entries in one launch each, and the K / V rows written to
        the slab by one pitched copy per plane on a side stream, so that the copy
        engine runs while the metadata kernels do.  key_states / value_states
        [1, G, S, D] or [G, S, D] on the cache device, in the cache dtype."""
        keys = key_states.reshape(-1, *key_states.shape[-2:])
        vals = value_states.reshape(-1, *value_states.shape[-2:])
        G = len(entries)
        if keys.shape != vals.shape or keys.shape[0] != G or keys.shape[-1] != HEAD_DIM:
            raise ValueError("expected [1, G, S, D] K/V for the G entries")
        if keys.device != self.device or keys.dtype != self.dtype or vals.dtype != self.dtype:
            raise ValueError("K/V must be on the cache device in the cache dtype")
        S = int(keys.shape[1])
        if S <= 1:
            raise ValueError("prefill needs more than one token")
        first = _contiguous_entries(entries)
        self._bookkeeping.preview(first, S)  # strict entry order and capacity
        if any(self._logical_lengths[e] != 0 for e in entries):
            raise ValueError("chunked/multiple prefill updates are unsupported")
        if self._prompt_length is not None and self._prompt_length != S:
            raise RuntimeError("cache entries received unequal prompt lengths")
        keys, vals = keys.contiguous(), vals.contiguous()
        main = torch.cuda.current_stream(self.device)
        side = getattr(self, "_prefill_stream", None)
        if side is None:
            side = self._prefill_stream = torch.cuda.Stream(device=self.device)
        side.wait_stream(main)
        lib = _lib.load()
        item = keys.element_size()
        row = HEAD_DIM * item
        L = self.geometry.max_cache_len
        with torch.cuda.stream(side):
            g = 0
            while g < G:
                e = first + g
                if e in self._resident_index:
                    idx = self._resident_index[e]
                    self._resident_kv[0, idx, :S].copy_(keys[g], non_blocking=True)
                    self._resident_kv[1, idx, :S].copy_(vals[g], non_blocking=True)
                    g += 1
                    continue
                run = 1
                while g + run < G and (first + g + run) not in self._resident_index:
                    run += 1
                for plane, src in ((0, keys), (1, vals)):
                    dst = self._slab._host_ptr + plane * (self._slab.nbytes // 2) + e * L * row
                    _lib.check(lib.tw_slab_write_rows(src[g].data_ptr(), S, dst, L, run, S, row,
                                                      side.cuda_stream), "slab_write_rows")
                g += run
        keys.record_stream(side)
        vals.record_stream(side)
        for e in entries:
            self._bookkeeping.advance(e, S)
            self._initialized[e] = True
        self._seen_tokens = self._bookkeeping.seen_tokens
        if self._prompt_length is None:
            self._prompt_length = S
        self._build_metadata_entries(first, keys)
        main.wait_stream(side)

    def _schedule_d2h(self, entry: int, start: int, key_states, value_states) -> None:
        n = int(key_states.shape[-2])
        self.entry_kv("key", entry)[start:start + n].copy_(key_states[0, 0], non_blocking=True)
        self.entry_kv("value", entry)[start:start + n].copy_(value_states[0, 0], non_blocking=True)

    def entry_kv(self, kind: str, entry: int) -> torch.Tensor:
        """[max_len, D] rows of one entry where they live: a device view for a
        resident entry, the pinned host slab view otherwise."""
        idx = self._resident_index.get(entry)
        if idx is not None:
            return self._resident_kv[0 if kind == "key" else 1, idx]
        return self._host_tensor(kind, entry)[0, 0]

    def _append_rows(self, first_entry: int, groups: int, position: int, k_new: torch.Tensor,
                     v_new: torch.Tensor) -> None:
        """Current token -> slab row `position`, running page min/max, INT4 codes."""
        packed = getattr(self, "_packed", None)
        lib = _lib.load()
        _lib.check(lib.tw_append_token(
            self._slab.key_device_ptr, self._slab.value_device_ptr, self._dirs.data_ptr(),
            self.geometry.num_entries, self.geometry.max_cache_len,
            first_entry, groups, position, k_new.data_ptr(), v_new.data_ptr(), HEAD_DIM,
            ops._kv_code(self.dtype), self.sink_tokens, self.block_size,
            self._page_min.data_ptr(), self._page_max.data_ptr(), self.page_capacity * HEAD_DIM,
            None if packed is None else packed.data_ptr(),
            None if packed is None else self._scale.data_ptr(),
            None if packed is None else self._minimum.data_ptr(),
            getattr(self, "int4_group_size", 128), self._stream()), "append_token")

    # ---------------------------------------------------------------- prefill --
    def _prefill(self, key_states, value_states, layer_idx: int, append_length: int,
                 old_length: int) -> None:
        if old_length != 0:
            raise ValueError("chunked/multiple prefill updates are unsupported")
        if self._prompt_length is None:
            self._prompt_length = append_length
        elif self._prompt_length != append_length:
            raise RuntimeError("cache entries received unequal prompt lengths")
        self._build_metadata(layer_idx, key_states)
        self._schedule_d2h(layer_idx, 0, key_states, value_states)

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[dict[str, Any]] = None):
        """hi/quest_offload_cache.py:513-665.  Prefill: metadata + slab copy, returns the
        inputs.  Decode: per-query-head pack [1, R, T, D] for K and V."""
        if key_states.shape != value_states.shape or key_states.shape[:2] != (1, 1):
            raise ValueError("expected identical head-wise [1, 1, seq, dim] K/V")
        if not key_states.is_cuda or key_states.device != self.device:
            raise ValueError("K/V must be on the cache device")
        append_length = int(key_states.shape[-2])
        old_length, _ = self._bookkeeping.preview(layer_idx, append_length)
        if append_length > 1:
            self._bookkeeping.advance(layer_idx, append_length)
            self._seen_tokens = self._bookkeeping.seen_tokens
            self._initialized[layer_idx] = True
            self._prefill(key_states, value_states, layer_idx, append_length, old_length)
            return key_states, value_states
        query = None if cache_kwargs is None else cache_kwargs.get("query_states")
        R = self.num_query_heads_per_kv
        if query is None or tuple(query.shape) != (1, R, 1, HEAD_DIM):
            raise ValueError("decode requires post-RoPE query_states")
        self._bookkeeping.advance(layer_idx, 1)
        self._seen_tokens = self._bookkeeping.seen_tokens
        self._initialized[layer_idx] = True
        return self._quest_decode_entry(layer_idx, query, key_states, value_states, old_length)

    # ---------------------------------------------------------- Quest per-Q path --
    def _quest_select(self, entries: list[int], queries: list[torch.Tensor], old_length: int):
        w = self._window(old_length)
        budget = min(w["candidate_pages"],
                     max(1, math.ceil(self.budget_fraction * w["eligible"] / self.block_size)))
        candidate_pages = min(w["candidate_pages"], self._metadata_pages(entries, old_length))
        budget = min(budget, candidate_pages)
        first = _contiguous_entries(entries)
        if budget == 0:
            return None, 0, w
        G = len(entries)
        # [1, R, 1, D] each (validated) -> [G, R, D] fp32
        q = torch.cat(queries, dim=0).view(G, self.num_query_heads_per_kv, HEAD_DIM).float()
        start = self._phase_start()
        scores = ops.quest_score(q, self._page_min[first:first + G], self._page_max[first:first + G],
                                 candidate_pages)
        pages = ops.topk_pages(scores, budget)
        self._phase_end("selector", start)
        if self._capture_selection_trace:
            decode_step = old_length - (self._prompt_length or 0) + 1
            cpu = pages.cpu()
            for g, entry in enumerate(entries):
                for r in range(self.num_query_heads_per_kv):
                    self._selection_trace.append({
                        "decode_step": decode_step, "entry": entry, "query_head_in_group": r,
                        "selected_page_indices": tuple(int(v) for v in cpu[g, r].tolist())})
        return pages, budget, w

    def prepare_layer_selection(self, *, entries: list[int], queries: list[torch.Tensor]) -> None:
        """hi/quest_offload_cache.py:299-401 (pages stay on the device).  With
        selection_interval > 1 the cached pages are reused between refreshes."""
        if not self.layer_batched_selection:
            return
        self._validate_layer(entries, queries)
        old_length = self._layer_old_length(entries)
        if self._prompt_length is None:
            raise RuntimeError("prompt length is missing")
        if not self._refresh_due(entries, old_length):
            self._quest_prepared.update(entries)
            return
        pages, budget, _ = self._quest_select(entries, queries, old_length)
        for g, entry in enumerate(entries):
            self._quest_pages[entry] = (pages, g, budget)
        self._quest_prepared.update(entries)

    def _refresh_due(self, entries, old_length: int) -> bool:
        decode_step = old_length - (self._prompt_length or 0) + 1
        return (any(e not in self._quest_pages for e in entries)
                or (decode_step - 1) % self.selection_interval == 0)

    def _quest_pages_for(self, entries: list[int], queries, old_length: int):
        """Pages [G,R,k] for the entries: prepared or cached, else selected now."""
        prepared = all(e in self._quest_prepared for e in entries)
        for e in entries:
            self._quest_prepared.discard(e)
        if not prepared and self._refresh_due(entries, old_length):
            pages, budget, w = self._quest_select(entries, queries, old_length)
            for g, entry in enumerate(entries):
                self._quest_pages[entry] = (pages, g, budget)
            return pages, budget, w
        items = [self._quest_pages[e] for e in entries]
        budget = items[0][2]
        w = self._window(old_length)
        if budget == 0:
            return None, 0, w
        base = items[0][0]
        if all(it[0] is base for it in items) and [it[1] for it in items] == list(
                range(items[0][1], items[0][1] + len(entries))):
            g0 = items[0][1]
            return base[g0:g0 + len(entries)], budget, w
        return torch.cat([it[0][it[1]:it[1] + 1] for it in items], dim=0), budget, w

    def _validate_layer(self, entries, queries) -> None:
        if len(entries) != len(queries) or not entries:
            raise ValueError("entries and queries must be non-empty and aligned")
        if len(set(entries)) != len(entries):
            raise ValueError("layer entries must be unique")
        shape = (1, self.num_query_heads_per_kv, 1, HEAD_DIM)
        if any(tuple(q.shape) != shape for q in queries):
            raise ValueError("unexpected layer Query shape")
        _contiguous_entries(entries)

    def _layer_old_length(self, entries) -> int:
        lengths = [self._logical_lengths[e] for e in entries]
        if len(set(lengths)) != 1:
            raise AssertionError("layer KV entries have unequal logical lengths")
        return lengths[0]

    def _quest_pack_buffers(self, rows: int) -> tuple[torch.Tensor, torch.Tensor]:
        if self._quest_pack is None or self._quest_pack.shape[1] < rows:
            self._quest_pack = torch.empty((2, rows, HEAD_DIM), dtype=self.dtype, device=self.device)
        return self._quest_pack[0, :rows], self._quest_pack[1, :rows]

    def _quest_gather(self, first: int, groups: int, pages, k_pages: int, w, old_length: int,
                      k_new: torch.Tensor, v_new: torch.Tensor):
        R = self.num_query_heads_per_kv
        seg_len = w["sink_end"] + k_pages * self.block_size + (old_length - w["recent_start"]) + 1
        total = seg_len * groups * R
        out_k, out_v = self._quest_pack_buffers(total)
        start = self._phase_start()
        _lib.check(_lib.load().tw_gather_quest_heads(
            self._slab.key_device_ptr, self._slab.value_device_ptr, self._dirs.data_ptr(),
            self.geometry.num_entries, self.geometry.max_cache_len,
            first, groups, R, old_length, w["sink_end"], w["recent_start"], self.sink_tokens,
            self.block_size, None if pages is None else pages.data_ptr(), k_pages,
            k_new.data_ptr(), v_new.data_ptr(), HEAD_DIM, ops._kv_code(self.dtype),
            out_k.data_ptr(), out_v.data_ptr(), self._error_flag.data_ptr(), self._stream()),
            "gather_quest_heads")
        self._phase_end("h2d", start)
        if self.metrics_enabled:
            self.metrics["h2d_bytes"] += 2 * (seg_len - 1) * groups * R * HEAD_DIM * k_new.element_size()
            self.metrics["h2d_copy_calls"] += 1
        return out_k, out_v, seg_len

    def _quest_decode_entry(self, entry: int, query, key_states, value_states, old_length: int):
        pages, budget, w = self._quest_pages_for([entry], [query], old_length)
        k_new = key_states[0, 0].contiguous()
        v_new = value_states[0, 0].contiguous()
        out_k, out_v, seg_len = self._quest_gather(entry, 1, pages, budget, w, old_length, k_new, v_new)
        self._append_rows(entry, 1, old_length, k_new, v_new)
        R = self.num_query_heads_per_kv
        self._last_query_head_lengths[entry] = tuple([seg_len] * R)
        return out_k.view(1, R, seg_len, HEAD_DIM), out_v.view(1, R, seg_len, HEAD_DIM)

    def update_layer_flat_ragged(self, *, key_states: list[torch.Tensor],
                                 value_states: list[torch.Tensor], queries: list[torch.Tensor],
                                 entries: list[int]):
        """hi/quest_offload_cache.py:724-987: per-query-head segments of one layer in
        one flat ragged batch.  Returns (K [sum_T,1,D], V, cu_seqlens int32, max, lengths)."""
        if not self.layer_flat_ragged_execution:
            raise RuntimeError("layer-flat ragged execution is disabled")
        if not (len(entries) == len(key_states) == len(value_states) == len(queries) and entries):
            raise ValueError("layer entries, K/V, and Queries must be aligned")
        self._validate_layer(entries, queries)
        for k, v in zip(key_states, value_states):
            if k.shape != v.shape or tuple(k.shape) != (1, 1, 1, HEAD_DIM):
                raise ValueError("layer-flat decode expects [1, 1, 1, dim] K/V")
        old_length = self._advance_layer(entries)
        first = entries[0]
        G = len(entries)
        pages, budget, w = self._quest_pages_for(entries, queries, old_length)
        k_new = torch.cat(key_states, dim=0).view(G, HEAD_DIM)
        v_new = torch.cat(value_states, dim=0).view(G, HEAD_DIM)
        out_k, out_v, seg_len = self._quest_gather(first, G, pages, budget, w, old_length, k_new, v_new)
        self._append_rows(first, G, old_length, k_new, v_new)
        R = self.num_query_heads_per_kv
        total = seg_len * G * R
        cu = self._equal_cu_seqlens(G * R, seg_len)
        lengths = tuple([seg_len] * (G * R))
        for g, entry in enumerate(entries):
            self._last_query_head_lengths[entry] = tuple([seg_len] * R)
        return out_k.view(total, 1, HEAD_DIM), out_v.view(total, 1, HEAD_DIM), cu, seg_len, lengths

    def _equal_cu_seqlens(self, segments: int, seg_len: int) -> torch.Tensor:
        """arange(segments + 1) * seg_len as int32 on the device.  The values are
        kept for the next call with the same shape (segment lengths stay fixed
        once the recent window is full); each call returns its own copy."""
        key = (segments, seg_len)
        cached = getattr(self, "_cu_cache", None)
        if cached is None or cached[0] != key:
            cu = torch.arange(0, segments + 1, dtype=torch.int32, device=self.device) * seg_len
            self._cu_cache = (key, cu)
        return self._cu_cache[1].clone()

    def _advance_layer(self, entries: list[int]) -> int:
        olds = []
        for entry in entries:
            self._bookkeeping.preview(entry, 1)
            old, _ = self._bookkeeping.advance(entry, 1)
            self._initialized[entry] = True
            olds.append(old)
        self._seen_tokens = self._bookkeeping.seen_tokens
        if len(set(olds)) != 1:
            raise AssertionError("layer KV entries have unequal logical lengths")
        return olds[0]

    # ------------------------------------------------------------------- misc --
    def get_last_query_head_lengths(self, entry: int) -> Optional[tuple[int, ...]]:
        return self._last_query_head_lengths[entry]

    def synchronize(self) -> None:
        torch.cuda.current_stream(self.device).synchronize()
        self._check_error_flag()

    def get_seq_length(self, layer_idx: Optional[int] = 0) -> int:
        return self._logical_lengths[0 if layer_idx is None else layer_idx]

    def get_max_length(self) -> Optional[int]:
        return self.allocated_capacity

    def reorder_cache(self, beam_idx: torch.LongTensor) -> None:
        del beam_idx
        raise NotImplementedError("batch-size-1 cache does not support reordering")

    def _device_bytes(self) -> int:
        tensors = [self._page_min, self._page_max, self._error_flag]
        if self._quest_pack is not None:
            tensors.append(self._quest_pack)
        for bufs in self._layer_bufs.values():
            tensors.extend(t for t in bufs.values() if isinstance(t, torch.Tensor))
        return sum(t.numel() * t.element_size() for t in tensors)

    def state_snapshot(self) -> dict[str, Any]:
        return {
            "logical_length": self.get_seq_length(),
            "allocated_capacity": self.allocated_capacity,
            "initialized_entries": sum(self._initialized),
            "host_slab_bytes": self._slab.nbytes,
            "host_slab_numa_node": self._slab.numa_node,
            "host_slab_pinned": True,
            "host_slab_device_mapped": True,
            "metadata_gpu_bytes": 2 * self._page_min.numel() * self._page_min.element_size(),
            "execution_buffer_gpu_bytes": self._device_bytes(),
            "block_size": self.block_size,
            "budget_fraction": self.budget_fraction,
            "selection_interval": self.selection_interval,
            "layer_batched_selection": self.layer_batched_selection,
            "layer_flat_ragged_execution": self.layer_flat_ragged_execution,
            "sparse_gather_stabilized": self.sparse_gather_stabilized,
            "max_selected_history_fraction": self.max_selected_history_fraction,
            "sink_tokens": self.sink_tokens,
            "recent_tokens": self.recent_tokens,
            "num_query_heads_per_kv": self.num_query_heads_per_kv,
            "incremental_page_metadata": self.incremental_page_metadata,
            "resident_entries": list(self.resident_entries),
            "resident_kv_gpu_bytes": 0 if self._resident_kv is None else
            self._resident_kv.numel() * self._resident_kv.element_size(),
            "backend": "sm_100a",
        }

    def close(self) -> None:
        self._slab.close()


_RESIDENT_OPTIONS = {
    # option: (default, allowed values); hi/twilight_offload_cache.py:163-175, :215-262
    "resident_mapping_backend": ("torch", {"torch", "native", "native_compact", "gpu_bitmap"}),
    "resident_hit_copy_backend": ("torch", {"torch", "triton"}),
    "resident_snapshot_backend": ("torch", {"torch", "triton", "contiguous"}),
    "resident_position_snapshot_backend": ("clone", {"clone", "reference"}),
}


def _check_resident_options(enabled: bool, options: dict[str, Any]) -> None:
    """The reference's validation of its resident-cache implementation options
    (hi/twilight_offload_cache.py:215-262).  They select among the reference's
    own mapping / copy / snapshot implementations; here one CUDA path serves
    them all, so valid values are accepted and otherwise unused."""
    for name, (default, allowed) in _RESIDENT_OPTIONS.items():
        value = options.get(name, default)
        if value not in allowed:
            raise ValueError(f"unknown {name.replace('_', ' ')}")
        if value != default and not enabled:
            raise ValueError(f"{name} requires the previous-token resident cache")
    if options.get("resident_zero_copy", False) and not enabled:
        raise ValueError("resident zero-copy requires resident cache")
    if options.get("resident_precompute_gpu_mapping", False) and not options.get(
            "resident_zero_copy", False):
        raise ValueError("precomputed GPU mapping requires mapped resident fast path")
    mapping = options.get("resident_mapping_backend", "torch")
    hit_copy = options.get("resident_hit_copy_backend", "torch")
    snapshot = options.get("resident_snapshot_backend", "torch")
    if mapping in {"native_compact", "gpu_bitmap"} and hit_copy != "triton":
        raise ValueError("compact hit indices require Triton hit copy")
    if snapshot == "contiguous" and (mapping not in {"native_compact", "gpu_bitmap"}
                                     or hit_copy != "triton"):
        raise ValueError("contiguous snapshot requires native_compact mapping and Triton hit copy")


class _RowReusePool:
    """Previous-token row reuse state of one GQA group count: per layer, the
    K/V rows of the previous decode step (union rows, then the current token)
    stay in device memory, and the next step reads every row it shares with
    them from there instead of over the host link
    (hi/twilight_offload_cache.py:2457-2608 and :3323-3470 keep the same
    per-layer state; hi/resident_gpu_mapping.py:103-144 maps hits/misses).
    Which previous row holds a position is recorded in the cache's row map
    under the step's tag.

    A slot holds one layer-step's rows kv [2, G * rows_per_group, D] and, for
    the staged gather, its cu_seqlens [G + 1].  A step writes a free slot and
    releases its layer's old one, so layers stepping in turn hold layers + 1
    slots."""

    def __init__(self, groups: int, rows_per_group: int, dtype: torch.dtype,
                 device: torch.device) -> None:
        self.groups = groups
        self.rows_per_group = rows_per_group
        self.dtype = dtype
        self.device = device
        self.slots: list[dict[str, torch.Tensor]] = []
        self.free: list[int] = []
        self.layers: dict[int, tuple[int, int]] = {}  # first entry -> (slot, tag)
        self.tag = 0
        self.log_chunks: list[torch.Tensor] = []
        self.log_used = 0
        self.slot_ptrs: list[tuple[int, int]] = []  # (K rows, V rows) device addresses

    def log_row_ptr(self) -> tuple[int, int]:
        """log_row as a device address: (address of the [G, 2] counter, log index)."""
        chunk, row = divmod(self.log_used, 1024)
        if chunk == len(self.log_chunks):
            self.log_chunks.append(torch.zeros((1024, self.groups, 2), dtype=torch.int32,
                                               device=self.device))
        self.log_used += 1
        return self.log_chunks[chunk].data_ptr() + row * self.groups * 8, self.log_used - 1

    def begin(self, first: int) -> tuple[Optional[tuple[torch.Tensor, int]], int, int]:
        """(previous (kv, tag) of the layer or None, reserved slot, its tag)."""
        if self.free:
            idx = self.free.pop()
        else:
            G = self.groups
            kv = torch.empty((2, G * self.rows_per_group, HEAD_DIM), dtype=self.dtype,
                             device=self.device)
            self.slots.append({
                "kv": kv,
                "cu": torch.zeros(G + 1, dtype=torch.int32, device=self.device),
            })
            self.slot_ptrs.append((kv[0].data_ptr(), kv[1].data_ptr()))
            idx = len(self.slots) - 1
        self.tag = self.tag + 1 if self.tag < 0xFFFFFFFF else 1
        state = self.layers.get(first)
        prev = None if state is None else (self.slots[state[0]]["kv"], state[1])
        if prev is not None and prev[1] == self.tag:  # after 2^32 steps: skip one reuse
            prev = None
        return prev, idx, self.tag

    def commit(self, first: int, idx: int, tag: int) -> None:
        state = self.layers.get(first)
        if state is not None:
            self.free.append(state[0])
        self.layers[first] = (idx, tag)

    def abort(self, idx: int) -> None:
        self.free.append(idx)

    def log_row(self) -> tuple[torch.Tensor, int]:
        """A zeroed [G, 2] (hit rows, miss rows) counter for one step."""
        chunk, row = divmod(self.log_used, 1024)
        if chunk == len(self.log_chunks):
            self.log_chunks.append(torch.zeros((1024, self.groups, 2), dtype=torch.int32,
                                               device=self.device))
        self.log_used += 1
        return self.log_chunks[chunk][row], self.log_used - 1

    def log_counts(self) -> torch.Tensor:
        if not self.log_chunks:
            return torch.zeros((0, self.groups, 2), dtype=torch.int32)
        return torch.cat(self.log_chunks).cpu()[: self.log_used]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for slot in self.slots for t in slot.values()) + \
            sum(t.numel() * t.element_size() for t in self.log_chunks)


class TwilightMatchedBudgetOffloadedCache(QuestTopKOffloadedCache):
    """Quest B0 + INT4 QK + top-p with the dynamic budget, GQA-group execution.

    hi/twilight_offload_cache.py:133-3743.  budget_mode must be 'dynamic' (the
    deployed profile); 'matched' raises ValueError.  qk_backend values of the
    reference are accepted and all run the CUDA INT4 estimator.  Extra keywords:
    ``int4_group_size`` (128 = the reference's per-token scale, or 32/64);
    ``protected_row_staging`` (default True): decode_layer's selection launch
    copies each group's sink and recent rows into device memory while it
    selects, and the attention reads them from there (same results; unused
    with the previous-token resident cache, whose kept rows serve them).
    """

    def __init__(self, *, candidate_token_budget: int = 8192, top_p: float = 0.95,
                 matched_budget_fraction: float = 0.05, budget_mode: str = "dynamic",
                 gqa_groupwise_execution: bool = False, qk_backend: str = "pytorch",
                 int4_group_size: int = 128, previous_token_resident_cache: bool = False,
                 protected_row_staging: bool = True, **kwargs: Any) -> None:
        if candidate_token_budget <= 0:
            raise ValueError("candidate_token_budget must be positive")
        if not 0.0 < top_p <= 1.0:
            raise ValueError("top_p must be in (0, 1]")
        if not 0.0 < matched_budget_fraction <= 1.0:
            raise ValueError("matched_budget_fraction must be in (0, 1]")
        if budget_mode not in {"matched", "dynamic"}:
            raise ValueError("budget_mode must be 'matched' or 'dynamic'")
        if budget_mode == "matched":
            raise ValueError("budget_mode='matched' is not implemented by the sm_100a path; "
                             "use budget_mode='dynamic'")
        if qk_backend not in {"pytorch", "triton", "triton_prepare", "cuda"}:
            raise ValueError("unknown Twilight QK backend")
        layer_batched = bool(kwargs.get("layer_batched_selection", False))
        if qk_backend != "pytorch" and not layer_batched:
            raise ValueError("fused QK requires layer-batched selection")
        if gqa_groupwise_execution and not layer_batched:
            raise ValueError("GQA group-wise execution requires layer-batched selection")
        if gqa_groupwise_execution and kwargs.get("layer_flat_ragged_execution", False):
            raise ValueError("GQA group-wise and per-Query-head flat execution are exclusive")
        if int4_group_size not in (32, 64, 128):
            raise ValueError("int4_group_size must be 32, 64 or 128")
        _check_resident_options(bool(previous_token_resident_cache), kwargs)
        if previous_token_resident_cache and not gqa_groupwise_execution:
            raise ValueError("previous-token resident cache requires GQA group-wise execution")
        max_cache_len = int(kwargs["max_cache_len"])
        sink = int(kwargs.get("sink_tokens", 64))
        block = int(kwargs.get("block_size", 16))
        max_pages = math.ceil(max(0, max_cache_len - sink) / block)
        required = min(max_pages, math.ceil(candidate_token_budget / block))
        kwargs["budget_fraction"] = matched_budget_fraction
        kwargs["max_selected_history_fraction"] = required / max_pages if max_pages else 1.0
        super().__init__(**kwargs)
        self.candidate_token_budget = int(candidate_token_budget)
        self.top_p = float(top_p)
        self.matched_budget_fraction = float(matched_budget_fraction)
        self.budget_mode = budget_mode
        self.gqa_groupwise_execution = bool(gqa_groupwise_execution)
        self.qk_backend = qk_backend
        self.int4_group_size = int(int4_group_size)
        E, L = self.geometry.num_entries, self.geometry.max_cache_len
        ng = HEAD_DIM // self.int4_group_size
        self._packed = torch.empty((E, L, HEAD_DIM // 2), dtype=torch.uint8, device=self.device)
        self._scale = torch.empty((E, L, ng), dtype=self.dtype, device=self.device)
        self._minimum = torch.empty_like(self._scale)
        self.b0_page_capacity = max(1, min(self.page_capacity, math.ceil(candidate_token_budget / block)))
        self._prepared: dict[int, dict[str, Any]] = {}
        self._capture_budget_trace = False
        self._budget_trace: list[dict[str, Any]] = []
        self._group_union_trace: list[dict[str, Any]] = []
        self._cached_group_positions: dict[int, torch.Tensor] = {}
        self._cached_per_q_positions: dict[int, tuple[torch.Tensor, ...]] = {}
        self.previous_token_resident_cache = bool(previous_token_resident_cache)
        self.protected_row_staging = bool(protected_row_staging)
        self._reuse_pools: dict[int, _RowReusePool] = {}
        self._reuse_trace_enabled = self.previous_token_resident_cache
        self._reuse_trace: list[dict[str, Any]] = []
        self._reuse_pending: list[tuple[dict[str, Any], int, int]] = []  # (row, G, log row)
        self._row_map: Optional[torch.Tensor] = None  # [E, L] int64 (tag << 32) | kept row
        self._plans: dict[tuple[int, ...], dict[str, Any]] = {}

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[dict[str, Any]] = None):
        """Prefill as the reference (metadata + INT4 codes + slab copy).  Decode runs
        through update_layer_gqa_group_ragged / attend_layer (the GQA group path)."""
        if int(key_states.shape[-2]) == 1:
            raise NotImplementedError(
                "Twilight decode runs per layer: use update_layer_gqa_group_ragged or attend_layer")
        return super().update(key_states, value_states, layer_idx, cache_kwargs)

    # --------------------------------------------------------------- metadata --
    def _build_metadata_entries(self, first: int, keys: torch.Tensor) -> None:
        """Quest metadata + INT4 codes of the prompt (hi/twilight_offload_cache.py:925-936)
        for entries first .. first + G - 1; keys [G, S, D]."""
        keys = keys.contiguous()
        super()._build_metadata_entries(first, keys)
        G, S = int(keys.shape[0]), int(keys.shape[1])
        _lib.check(_lib.load().tw_int4_pack(  # key entry stride in rows
            keys.data_ptr(), S, G, S, HEAD_DIM, self.int4_group_size,
            ops._kv_code(self.dtype), self._packed[first].data_ptr(), self._scale[first].data_ptr(),
            self._minimum[first].data_ptr(), self.geometry.max_cache_len, 0, self._stream()),
            "int4_pack")

    # ---------------------------------------------------------------- buffers --
    def _buffers(self, first: int, groups: int) -> dict[str, Any]:
        bufs = self._layer_bufs.get(groups)
        if bufs is not None:
            return bufs
        R = self.num_query_heads_per_kv
        L = self.geometry.max_cache_len
        dev = self.device
        n_cap = self.b0_page_capacity * self.block_size
        per_group = min(L, self.sink_tokens + self.recent_tokens + R * n_cap) + 1
        rows_cap = groups * per_group
        ws = ops.select_layer_workspace_bytes(groups, R, self.page_capacity, self.b0_page_capacity,
                                              self.block_size)
        attn_ws = ops.decode_attention_workspace_bytes(groups, R, per_group)
        bufs = {
            "pages": torch.empty((groups, R, self.b0_page_capacity), dtype=torch.int32, device=dev),
            "union_pos": torch.empty((groups, L), dtype=torch.int32, device=dev),
            # union_count [G] | error flag slot is separate
            "union_count": torch.zeros(groups, dtype=torch.int32, device=dev),
            "head_count": torch.zeros((groups, R), dtype=torch.int32, device=dev),
            "head_pos": torch.empty((groups, R, n_cap), dtype=torch.int32, device=dev),
            # zero: the fused selection keeps its union merge state here, left zero
            "workspace": torch.zeros(max(ws, 256), dtype=torch.uint8, device=dev),
            "attn_workspace": torch.zeros(max(attn_ws, 256), dtype=torch.uint8, device=dev),
            "flat": torch.empty((2, 2, rows_cap, HEAD_DIM), dtype=self.dtype, device=dev),
            "cu": torch.zeros((2, groups + 1), dtype=torch.int32, device=dev),
            "rows_cap": rows_cap,
            "per_group_cap": per_group,
            "slot": 0,
            "stage": None,
        }
        if self.protected_row_staging and not self.previous_token_resident_cache:
            # sink rows + recent rows of every group (decode_layer's staging)
            stage_rows = self.sink_tokens + max(1, self.recent_tokens)
            bufs["stage"] = torch.empty((2, groups, stage_rows, HEAD_DIM), dtype=self.dtype,
                                        device=dev)
        self._layer_bufs[groups] = bufs
        return bufs

    # ------------------------------------------------------------ row reuse --
    def _reuse_pool(self, groups: int) -> _RowReusePool:
        pool = self._reuse_pools.get(groups)
        if pool is None:
            per_group = self._buffers(0, groups)["per_group_cap"]
            pool = _RowReusePool(groups, per_group, self.dtype, self.device)
            self._reuse_pools[groups] = pool
            if self._row_map is None:
                self._row_map = torch.zeros((self.geometry.num_entries, self.geometry.max_cache_len),
                                            dtype=torch.int64, device=self.device)
        return pool

    def _reuse_begin(self, first: int, G: int, old_length: int, staged: bool):
        """Reserve this layer-step's kept rows: (RowReuse or None, slot or None)."""
        if not self.previous_token_resident_cache:
            return None, None
        pool = self._reuse_pool(G)
        prev, idx, tag = pool.begin(first)
        counts = None
        if self._reuse_trace_enabled:
            counts, log_idx = pool.log_row()
            self._reuse_pending.append(({
                "decode_step": old_length - (self._prompt_length or 0) + 1,
                "layer": first // G, "reuse_active": prev is not None}, G, log_idx))
        kv = pool.slots[idx]["kv"]
        rows = self._row_map[first: first + G]
        kw = {} if prev is None else dict(prev_tag=prev[1], prev_k=prev[0][0], prev_v=prev[0][1])
        if staged:
            r = ops.row_reuse(rows, tag, row_counts=counts, **kw)
        else:
            per = pool.rows_per_group
            r = ops.row_reuse(rows, tag, next_k=kv[0].view(G, per, HEAD_DIM),
                              next_v=kv[1].view(G, per, HEAD_DIM), row_counts=counts, **kw)
        return r, (idx, tag)

    def _reuse_end(self, first: int, G: int, slot, ok: bool) -> None:
        if slot is None:
            return
        pool = self._reuse_pools[G]
        if ok:
            pool.commit(first, *slot)
        else:
            pool.abort(slot[0])

    def enable_resident_reuse_trace(self, enabled: bool = True) -> None:
        """Record per-layer-step hit / miss row counts (on by default with the
        previous-token resident cache; each recorded step adds two counter
        atomics per warp, no host synchronisation)."""
        self._reuse_trace_enabled = bool(enabled) and self.previous_token_resident_cache

    def resident_reuse_trace(self) -> list[dict[str, Any]]:
        """Per-layer-step hit / miss rows of the previous-token resident cache
        (hi/twilight_offload_cache.py:803-823 and its trace rows at :2545-2557,
        :3447-3470).  hit_rows counts the union rows read from the previous
        step's device rows; the previous step's own token counts as a hit (the
        reference reads it from the host).  Reading synchronises."""
        if self._reuse_pending:
            logs = {G: pool.log_counts() for G, pool in self._reuse_pools.items()}
            item = torch.tensor([], dtype=self.dtype).element_size()
            for row, G, idx in self._reuse_pending:
                hits = int(logs[G][idx, :, 0].sum())
                misses = int(logs[G][idx, :, 1].sum())
                history = hits + misses
                miss_bytes = 2 * misses * HEAD_DIM * item
                row.update({
                    "history_rows": history, "hit_rows": hits, "miss_rows": misses,
                    "hit_ratio": hits / history if history else 0.0,
                    "selected_kv_h2d_bytes": miss_bytes, "mapped_cpu_kv_read_bytes": miss_bytes,
                    "resident_logical_bytes": 2 * history * HEAD_DIM * item})
                self._reuse_trace.append(row)
            self._reuse_pending.clear()
        return list(self._reuse_trace)

    # -------------------------------------------------------------- selection --
    def prepare_layer_selection(self, *, entries: list[int], queries: list[torch.Tensor]) -> None:
        """Both Twilight selection stages for one layer on the device
        (hi/twilight_offload_cache.py:996-1843, gpu_compact_gqa_union semantics)."""
        if not self.layer_batched_selection:
            return
        self._validate_layer(entries, queries)
        old_length = self._layer_old_length(entries)
        if self._prompt_length is None:
            raise RuntimeError("Twilight prompt metadata is missing")
        q = torch.stack([query[0, :, 0] for query in queries], dim=0).float().contiguous()
        self._select(entries, q, old_length)

    def _select(self, entries: list[int], q: torch.Tensor, old_length: int) -> None:
        first = entries[0]
        G = len(entries)
        R = self.num_query_heads_per_kv
        bufs = self._buffers(first, G)
        w = self._window(old_length)
        candidate_pages = min(w["candidate_pages"], self._metadata_pages(entries, old_length))
        b0_pages = min(candidate_pages, max(1, math.ceil(self.candidate_token_budget / self.block_size)),
                       self.b0_page_capacity)
        start = self._phase_start()
        if candidate_pages == 0 or b0_pages == 0:
            protected = torch.cat((torch.arange(w["sink_end"], device=self.device, dtype=torch.int32),
                                   torch.arange(w["recent_start"], old_length, device=self.device,
                                                dtype=torch.int32)))
            bufs["union_pos"][:, : protected.numel()] = protected
            bufs["union_count"].fill_(protected.numel())
            bufs["head_count"].zero_()
        else:
            lib = _lib.load()
            _lib.check(lib.tw_select_layer(
                q.data_ptr(), self._page_min[first].data_ptr(), self._page_max[first].data_ptr(),
                self.page_capacity * HEAD_DIM, candidate_pages, self._packed[first].data_ptr(),
                self._scale[first].data_ptr(), self._minimum[first].data_ptr(),
                self.geometry.max_cache_len, G, R, b0_pages, self.block_size, self.sink_tokens,
                HEAD_DIM, self.int4_group_size, ops._kv_code(self.dtype), self.top_p, old_length,
                w["sink_end"], w["recent_start"], bufs["pages"].data_ptr(),
                bufs["union_pos"].data_ptr(), self.geometry.max_cache_len,
                bufs["union_count"].data_ptr(), bufs["head_count"].data_ptr(),
                bufs["head_pos"].data_ptr() if self._tracing() else None,
                self._error_flag.data_ptr(), bufs["workspace"].data_ptr(),
                bufs["workspace"].numel(), self._stream()), "select_layer")
        self._phase_end("twilight_selection_core", start)
        self._prepared[first] = dict(old_length=old_length, window=w, b0_pages=b0_pages,
                                     candidate_pages=candidate_pages, entries=list(entries))
        if self._tracing():
            self._record_traces(entries, old_length, w, b0_pages, bufs)

    def _tracing(self) -> bool:
        return self._capture_selection_trace or self._capture_budget_trace

    def _record_traces(self, entries, old_length, w, b0_pages, bufs) -> None:
        R = self.num_query_heads_per_kv
        counts = bufs["head_count"].cpu()
        head_pos = bufs["head_pos"].cpu()
        decode_step = old_length - (self._prompt_length or 0) + 1
        protected = w["sink_end"] + (old_length - w["recent_start"])
        for g, entry in enumerate(entries):
            rows = []
            for r in range(R):
                c = int(counts[g, r]) if b0_pages else 0
                sel = head_pos[g, r, :c].to(torch.int64) if b0_pages else torch.empty(0, dtype=torch.int64)
                rows.append(sel)
                if self._capture_budget_trace:
                    self._budget_trace.append({
                        "decode_step": decode_step, "entry": entry, "kv_head": g,
                        "query_head_in_group": r, "budget_mode": self.budget_mode,
                        "b0_tokens": b0_pages * self.block_size, "raw_b1_tokens": c,
                        "selected_adaptive_tokens": c, "protected_tokens": protected,
                        "selected_history_tokens": protected + c,
                        "eligible_history_tokens": w["eligible"], "full_history_tokens": old_length})
            self._cached_per_q_positions[entry] = tuple(rows)
            if self._capture_selection_trace:
                for r, sel in enumerate(rows):
                    self._selection_trace.append({
                        "decode_step": decode_step, "entry": entry, "query_head_in_group": r,
                        "selected_positions": tuple(int(v) for v in sel.tolist())})

    def enable_budget_trace(self, enabled: bool = True) -> None:
        self._capture_budget_trace = bool(enabled)
        self._budget_trace = []

    def budget_trace(self) -> list[dict[str, Any]]:
        return list(self._budget_trace)

    def group_union_trace(self) -> list[dict[str, Any]]:
        return list(self._group_union_trace)

    # --------------------------------------------------------- GQA group path --
    def _begin_group_step(self, key_states, value_states, queries, entries):
        if not self.gqa_groupwise_execution:
            raise RuntimeError("Twilight GQA group-wise execution is disabled")
        if not (len(entries) == len(key_states) == len(value_states) == len(queries) and entries):
            raise ValueError("layer entries, K/V, and Queries must be aligned")
        if len(set(entries)) != len(entries):
            raise ValueError("layer entries must be unique")
        _contiguous_entries(entries)
        for k, v in zip(key_states, value_states):
            if k.shape != v.shape or tuple(k.shape) != (1, 1, 1, HEAD_DIM):
                raise ValueError("GQA group decode expects [1, 1, 1, dim] K/V")
        prepared = self._prepared.get(entries[0])
        if prepared is None or prepared["old_length"] != self._layer_old_length(entries):
            raise AssertionError("prepared GPU GQA union is missing")
        del self._prepared[entries[0]]
        old_length = self._advance_layer(entries)
        k_new = torch.cat([k[0, 0] for k in key_states], dim=0)
        v_new = torch.cat([v[0, 0] for v in value_states], dim=0)
        return old_length, k_new, v_new

    def _gather_union(self, first: int, G: int, old_length: int, k_new, v_new):
        bufs = self._buffers(first, G)
        reuse, slot = self._reuse_begin(first, G, old_length, staged=True)
        if slot is None:
            cur = bufs["slot"]
            bufs["slot"] = 1 - cur
            out_k = bufs["flat"][cur, 0]
            out_v = bufs["flat"][cur, 1]
            cu = bufs["cu"][cur]
        else:
            kept = self._reuse_pools[G].slots[slot[0]]
            out_k, out_v, cu = kept["kv"][0], kept["kv"][1], kept["cu"]
        start = self._phase_start()
        status = _lib.load().tw_gather_union(
            self._slab.key_device_ptr, self._slab.value_device_ptr, self._dirs.data_ptr(),
            self.geometry.num_entries, self.geometry.max_cache_len,
            first, G, old_length, bufs["union_pos"].data_ptr(), self.geometry.max_cache_len,
            bufs["union_count"].data_ptr(), k_new.data_ptr(), v_new.data_ptr(), HEAD_DIM,
            ops._kv_code(self.dtype), out_k.data_ptr(), out_v.data_ptr(), bufs["rows_cap"],
            cu.data_ptr(), self._error_flag.data_ptr(),
            ctypes.byref(reuse) if reuse is not None else None, self._stream())
        self._reuse_end(first, G, slot, status == _lib.TW_OK)
        _lib.check(status, "gather_union")
        self._phase_end("h2d", start)
        return bufs, out_k, out_v, cu

    def update_layer_gqa_group_ragged(self, *, key_states: list[torch.Tensor],
                                      value_states: list[torch.Tensor],
                                      queries: list[torch.Tensor], entries: list[int]):
        """hi/twilight_offload_cache.py:2610-3602.  Returns (K [sum_T,1,D], V, cu_seqlens_k
        int32 [G+1] (device), max_seqlen_k, group_total_lengths); group g's rows are its
        sorted union followed by its current token.  K/V are views into cache-owned
        double-buffered storage, valid until the next layer reuses the slot."""
        old_length, k_new, v_new = self._begin_group_step(key_states, value_states, queries, entries)
        first, G = entries[0], len(entries)
        bufs, out_k, out_v, cu = self._gather_union(first, G, old_length, k_new, v_new)
        self._append_rows(first, G, old_length, k_new, v_new)
        host = torch.cat((bufs["union_count"], self._error_flag)).cpu()
        flag = int(host[-1])
        if flag:
            self._error_flag.zero_()
            _lib.check(flag, "device-side check")
        counts = [int(c) for c in host[:-1].tolist()]
        lengths = tuple(c + 1 for c in counts)
        total = sum(lengths)
        for g, entry in enumerate(entries):
            self._last_query_head_lengths[entry] = tuple([lengths[g]] * self.num_query_heads_per_kv)
        self._record_group_step(entries, old_length, counts, bufs["union_pos"])
        return (out_k[:total].view(total, 1, HEAD_DIM), out_v[:total].view(total, 1, HEAD_DIM), cu,
                max(lengths), lengths)

    def _record_group_step(self, entries, old_length, counts, union_pos) -> None:
        decode_step = old_length - (self._prompt_length or 0) + 1
        if self._capture_selection_trace:
            for g, entry in enumerate(entries):
                union = union_pos[g, : counts[g]].to(torch.int64).cpu()
                self._cached_group_positions[entry] = union
                self._group_union_trace.append({
                    "decode_step": decode_step, "entry": entry, "kv_head": g,
                    "group_union_history_tokens": counts[g],
                    "positions_sha256": hashlib.sha256(union.numpy().tobytes()).hexdigest()})
        if self.metrics_enabled:
            self.metrics["h2d_bytes"] += 2 * sum(counts) * HEAD_DIM * torch.tensor([], dtype=self.dtype).element_size()
            self.metrics["h2d_copy_calls"] += 1
            self.metrics["group_union_history_tokens_total"] += sum(counts)
            self.metrics["cache_update_calls"] += len(entries)

    def attend_layer(self, *, key_states, value_states, queries, entries,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Fused extension of the GQA group step: the split-K attention reads each
        group's union rows straight from the mapped host slab (no staged copy),
        then the new token is appended; no host synchronisation.  Returns the
        attention output [G, R, D] in the K/V dtype (what hi/mp.py:258-279 feeds
        to o_proj)."""
        old_length, k_new, v_new = self._begin_group_step(key_states, value_states, queries, entries)
        first, G = entries[0], len(entries)
        bufs = self._buffers(first, G)
        q = torch.stack([query[0, :, 0] for query in queries], dim=0).to(self.dtype).contiguous()
        reuse, slot = self._reuse_begin(first, G, old_length, staged=False)
        start = self._phase_start()
        try:
            out = ops.attend_union(self._slab, first, old_length, bufs["union_pos"],
                                   bufs["union_count"], k_new, v_new, q,
                                   min(bufs["per_group_cap"], old_length + 1),
                                   workspace=bufs["attn_workspace"], error_flag=self._error_flag,
                                   out=out, entry_dirs=self._dirs, reuse=reuse)
        except Exception:
            self._reuse_end(first, G, slot, False)
            raise
        self._reuse_end(first, G, slot, True)
        self._phase_end("attention", start)
        self._append_rows(first, G, old_length, k_new, v_new)
        return out

    def decode_layer(self, *, queries, key_states, value_states, entries,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One whole layer-step in one library call (tw_twilight_decode_layer):
        selection, fused union gather + attention and the new-token append, no
        host synchronisation.  Equivalent to prepare_layer_selection followed by
        attend_layer.  queries may be the reference's list of [1, R, 1, D]
        tensors or one [G, R, D] tensor; key_states / value_states lists of
        [1, 1, 1, D] or [G, D] tensors."""
        key = tuple(entries)
        plan = self._plans.get(key)
        if plan is None:
            plan = self._make_plan(entries)
        G, first = plan["G"], plan["first"]
        R = self.num_query_heads_per_kv
        if isinstance(queries, torch.Tensor):
            q = queries
        else:
            self._validate_layer(entries, queries)
            q = torch.stack([query[0, :, 0] for query in queries], dim=0)
        k_new = key_states if isinstance(key_states, torch.Tensor) else torch.cat(
            [k.reshape(1, HEAD_DIM) for k in key_states], dim=0)
        v_new = value_states if isinstance(value_states, torch.Tensor) else torch.cat(
            [v.reshape(1, HEAD_DIM) for v in value_states], dim=0)
        dt = self.dtype
        if (q.shape != plan["q_shape"] or k_new.shape != plan["kv_shape"]
                or v_new.shape != plan["kv_shape"]):
            raise ValueError("queries must be [G, R, D] and new K/V [G, D]")
        if (q.dtype != dt or k_new.dtype != dt or v_new.dtype != dt
                or not (q.is_cuda and k_new.is_cuda and v_new.is_cuda)
                or not (q.is_contiguous() and k_new.is_contiguous() and v_new.is_contiguous())):
            raise ValueError("queries and new K/V must be contiguous CUDA tensors of the K/V dtype")
        old_length = self._bookkeeping.check_block(first, G)
        if self._prompt_length is None:
            raise RuntimeError("Twilight prompt metadata is missing")
        sink_end = min(self.sink_tokens, old_length)
        recent_start = max(sink_end, old_length - max(0, self.recent_tokens - 1))
        if self.incremental_page_metadata:
            meta = max(0, old_length - self.sink_tokens) // self.block_size
        else:
            if plan["meta_version"] != self._meta_version:
                plan["meta_pages"] = min(self._meta_pages[e] for e in entries)
                plan["meta_version"] = self._meta_version
            meta = plan["meta_pages"]
        candidate_pages = min((recent_start - sink_end) // self.block_size, meta)
        b0_pages = min(candidate_pages, plan["b0_budget"])
        if candidate_pages <= 0 or b0_pages <= 0 or self._tracing():
            # protected-only windows and traced runs take the two-call path
            self.prepare_layer_selection(entries=entries, queries=[q[g].view(1, R, 1, HEAD_DIM) for g in range(G)])
            return self.attend_layer(key_states=[k_new[g].view(1, 1, 1, HEAD_DIM) for g in range(G)],
                                     value_states=[v_new[g].view(1, 1, 1, HEAD_DIM) for g in range(G)],
                                     queries=[q[g].view(1, R, 1, HEAD_DIM) for g in range(G)],
                                     entries=entries, out=out)
        if out is None:
            out = torch.empty(plan["q_shape"], dtype=dt, device=self.device)
        elif out.shape != plan["q_shape"] or not out.is_cuda or not out.is_contiguous():
            raise ValueError("out must be a contiguous CUDA tensor [G, R, D]")
        args = plan["args"]
        args.n_pages = candidate_pages
        args.b0_pages = b0_pages
        args.old_length = old_length
        args.sink_end = sink_end
        args.recent_start = recent_start
        args.q = q.data_ptr()
        args.k_new = k_new.data_ptr()
        args.v_new = v_new.data_ptr()
        args.out = out.data_ptr()
        args.out_dtype = ops.DTYPE_CODES[out.dtype]
        args.max_rows_per_group = min(plan["per_group_cap"], old_length + 1)
        pool = plan["pool"]
        if pool is not None:
            reuse = plan["reuse"]
            prev, idx, tag = pool.begin(first)
            reuse.next_tag = tag
            reuse.next_k, reuse.next_v = pool.slot_ptrs[idx]
            if prev is None:
                reuse.prev_tag = 0
                reuse.prev_k = reuse.prev_v = None
            else:
                reuse.prev_tag = prev[1]
                reuse.prev_k, reuse.prev_v = pool.slot_ptrs[pool.layers[first][0]]
            if self._reuse_trace_enabled:
                counts, log_idx = pool.log_row_ptr()
                reuse.row_counts = counts
                self._reuse_pending.append(({
                    "decode_step": old_length - (self._prompt_length or 0) + 1,
                    "layer": first // G, "reuse_active": prev is not None}, G, log_idx))
            else:
                reuse.row_counts = None
        start = self._phase_start() if self.metrics_enabled else None
        status = plan["fn"](plan["args_ref"], torch._C._cuda_getCurrentRawStream(self._device_index))
        if pool is not None:
            if status == _lib.TW_OK:
                pool.commit(first, idx, tag)
            else:
                pool.abort(idx)
        if status != _lib.TW_OK:
            _lib.check(status, "twilight_decode_layer")
        if start is not None:
            self._phase_end("decode_layer", start)
        self._bookkeeping.commit_block(first, G, old_length)
        self._initialized[first:first + G] = plan["initialized"]
        self._seen_tokens = self._bookkeeping.seen_tokens
        return out

    def _make_plan(self, entries: list[int]) -> dict[str, Any]:
        """Per-layer constants of decode_layer: the argument struct with its fixed
        fields, buffer addresses, shapes and the library entry point."""
        G = len(entries)
        if G == 0 or len(set(entries)) != G:
            raise ValueError("layer entries must be non-empty and unique")
        first = _contiguous_entries(entries)
        if first + G > self.geometry.num_entries:
            raise ValueError("layer entries outside the cache")
        R = self.num_query_heads_per_kv
        bufs = self._buffers(first, G)
        args = _lib.DecodeLayerArgs()
        args.slab_k = self._slab.key_device_ptr
        args.slab_v = self._slab.value_device_ptr
        args.entry_dirs = self._dirs.data_ptr()
        args.n_entries = self.geometry.num_entries
        args.max_len = self.geometry.max_cache_len
        args.first_entry = first
        args.groups = G
        args.heads_per_group = R
        args.dtype = ops._kv_code(self.dtype)
        args.page_min = self._page_min.data_ptr()
        args.page_max = self._page_max.data_ptr()
        args.page_capacity = self.page_capacity
        args.packed = self._packed.data_ptr()
        args.scale = self._scale.data_ptr()
        args.minimum = self._minimum.data_ptr()
        args.int4_group_size = self.int4_group_size
        args.sink = self.sink_tokens
        args.block_size = self.block_size
        args.top_p = self.top_p
        args.append = 1
        args.pages = bufs["pages"].data_ptr()
        args.union_pos = bufs["union_pos"].data_ptr()
        args.pos_stride = self.geometry.max_cache_len
        args.union_count = bufs["union_count"].data_ptr()
        args.head_count = bufs["head_count"].data_ptr()
        args.head_pos = None
        args.error_flag = self._error_flag.data_ptr()
        args.select_workspace = bufs["workspace"].data_ptr()
        args.select_workspace_bytes = bufs["workspace"].numel()
        args.attn_workspace = bufs["attn_workspace"].data_ptr()
        args.attn_workspace_bytes = bufs["attn_workspace"].numel()
        pool = reuse = None
        if self.previous_token_resident_cache:
            pool = self._reuse_pool(G)
            reuse = _lib.RowReuse()
            reuse.row_map = self._row_map[first].data_ptr()
            reuse.map_stride = self.geometry.max_cache_len
            reuse.prev_rows = G * pool.rows_per_group
            reuse.rows_stride = pool.rows_per_group
            args.reuse = ctypes.addressof(reuse)
        elif bufs["stage"] is not None:
            args.stage_k = bufs["stage"][0].data_ptr()
            args.stage_v = bufs["stage"][1].data_ptr()
            args.stage_rows = bufs["stage"].shape[2]
        plan = {
            "G": G, "first": first, "args": args, "args_ref": ctypes.byref(args),
            "fn": _lib.load().tw_twilight_decode_layer, "bufs": bufs,
            "q_shape": torch.Size((G, R, HEAD_DIM)), "kv_shape": torch.Size((G, HEAD_DIM)),
            "per_group_cap": bufs["per_group_cap"],
            "b0_budget": min(max(1, math.ceil(self.candidate_token_budget / self.block_size)),
                             self.b0_page_capacity),
            "meta_version": -1, "meta_pages": 0, "pool": pool, "reuse": reuse,
            "initialized": [True] * G,
        }
        self._plans[tuple(entries)] = plan
        return plan

    # ------------------------------------------------------------- hashes ----
    def selected_positions_sha256(self) -> str:
        digest = hashlib.sha256()
        for entry in sorted(self._cached_per_q_positions):
            positions = self._cached_per_q_positions[entry]
            digest.update(entry.to_bytes(4, byteorder="little", signed=False))
            digest.update(len(positions).to_bytes(4, byteorder="little", signed=False))
            for selected in positions:
                arr = selected.to(torch.int64).contiguous()
                digest.update(arr.numel().to_bytes(8, byteorder="little", signed=False))
                digest.update(arr.numpy().tobytes())
        return digest.hexdigest()

    def group_positions_sha256(self) -> Optional[str]:
        digest = hashlib.sha256()
        for entry in sorted(self._cached_group_positions):
            arr = self._cached_group_positions[entry].to(torch.int64).contiguous()
            digest.update(entry.to_bytes(4, byteorder="little", signed=False))
            digest.update(arr.numel().to_bytes(8, byteorder="little", signed=False))
            digest.update(arr.numpy().tobytes())
        return digest.hexdigest()

    def state_snapshot(self) -> dict[str, Any]:
        snap = super().state_snapshot()
        quant = sum(t.numel() * t.element_size() for t in (self._packed, self._scale, self._minimum))
        snap.update({
            "policy": "twilight_inspired_int4_top_p_dynamic",
            "candidate_token_budget": self.candidate_token_budget,
            "top_p": self.top_p,
            "matched_budget_fraction": self.matched_budget_fraction,
            "budget_mode": self.budget_mode,
            "quantized_key_metadata_gpu_bytes": quant,
            "int4_group_size": self.int4_group_size,
            "qk_backend": self.qk_backend,
            "twilight_gqa_groupwise_execution": self.gqa_groupwise_execution,
            "twilight_gqa_group_semantics": "exact union of the original per-Query-head selected token sets",
            "selection_boundary": "device-resident union; host reads only the union lengths",
            "previous_token_resident_cache": self.previous_token_resident_cache,
            "resident_cache_allocated_bytes": sum(p.nbytes() for p in self._reuse_pools.values())
            + (self._row_map.numel() * 8 if self._row_map is not None else 0),
        })
        return snap

    def _device_bytes(self) -> int:
        extra = sum(p.nbytes() for p in self._reuse_pools.values())
        if self._row_map is not None:
            extra += self._row_map.numel() * self._row_map.element_size()
        return super()._device_bytes() + extra
