"""The exact-order oracle pipeline for one layer (checker for the GPU path)."""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from oracle import exact, torch_ref

DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1}


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@dataclass
class OracleSelection:
    window: torch_ref.Window
    pmin: np.ndarray
    pmax: np.ndarray
    packed: np.ndarray
    scale: np.ndarray
    minimum: np.ndarray
    scores: np.ndarray
    pages: np.ndarray
    logits: np.ndarray
    head_count: np.ndarray
    head_pos: list
    unions: list


def twilight_oracle(keys: torch.Tensor, queries: torch.Tensor, *, old_length: int, sink: int,
                    recent: int, block: int, b0_tokens: int, top_p: float, group: int = 128,
                    scale_div: int = 0, meta_pages: int | None = None) -> OracleSelection:
    """keys [G, S, D] (S >= old_length rows; metadata/codes from rows < meta_len), queries [G,R,D]."""
    G, S, D = keys.shape
    code = DTYPE_CODE[keys.dtype]
    kb = bits(keys)
    if meta_pages is None:
        meta_pages = max(0, old_length - sink) // block if old_length > sink else 0
    meta_len = sink + meta_pages * block
    w = torch_ref.window(old_length, sink=sink, recent=recent, block=block,
                         candidate_token_budget=b0_tokens, metadata_pages=meta_pages)
    pm, px = [], []
    for g in range(G):
        a, b = exact.quest_page_metadata(kb[g, :max(meta_len, 0)], sink, block, code)
        pm.append(a)
        px.append(b)
    pmin = np.stack(pm) if meta_pages else np.zeros((G, 0, D), np.uint16)
    pmax = np.stack(px) if meta_pages else np.zeros((G, 0, D), np.uint16)
    packs = [exact.int4_pack(kb[g, :S], group, code, scale_div) for g in range(G)]
    packed = np.stack([p[0] for p in packs])
    scale = np.stack([p[1] for p in packs])
    minimum = np.stack([p[2] for p in packs])
    q = queries.float().numpy()
    P, b0 = w.candidate_pages, w.b0_pages
    R = q.shape[1]
    if P == 0 or b0 == 0:
        protected = np.concatenate([np.arange(w.sink_end), np.arange(w.recent_start, old_length)]).astype(np.int32)
        return OracleSelection(w, pmin, pmax, packed, scale, minimum, np.zeros((G, R, 0), np.float32),
                               np.zeros((G, R, 0), np.int32), np.zeros((G, R, 0), np.float32),
                               np.zeros((G, R), np.int32), [[np.zeros(0, np.int32)] * R] * G,
                               [protected.copy() for _ in range(G)])
    scores = exact.quest_score(q, np.ascontiguousarray(pmin[:, :P]), np.ascontiguousarray(pmax[:, :P]), code)
    pages = exact.topk_pages(scores, b0)
    logits = exact.int4_qk(q, packed, scale, minimum, pages, block, sink, group, code)
    unions, hc, hp, bad = exact.top_p_union(logits, pages, block, sink, top_p, old_length,
                                            w.sink_end, w.recent_start)
    assert bad == 0
    return OracleSelection(w, pmin, pmax, packed, scale, minimum, scores, pages, logits, hc, hp, unions)


def attention_f64(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return torch_ref.decode_attention(q, k, v)


def gather_rows(host_keys: torch.Tensor, positions) -> torch.Tensor:
    return host_keys.index_select(0, torch.as_tensor(np.asarray(positions), dtype=torch.long))


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


__all__ = ["twilight_oracle", "attention_f64", "bits", "DTYPE_CODE", "ceil_div", "math"]
