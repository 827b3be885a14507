"""Comparison rules shared by the parity tests.

* Index sets chosen by a top-k over float scores must match exactly, except
  that an element may be swapped for one whose reference score is within
  REL_TIE (1e-6) relative of the selection boundary (a tie).
* Top-p counts may differ only where the exact cumulative softmax mass at the
  boundary lies within the fp32 accumulation error of the reference's
  sequential cumsum, n * 2^-24 (n = number of candidates).
* Attention outputs: 1e-3 absolute in fp32 mode, 2e-2 absolute in bf16/fp16.
"""

from __future__ import annotations

import numpy as np

REL_TIE = 1e-6
ATTN_TOL_FP32 = 1e-3
ATTN_TOL_16BIT = 2e-2


def _tie_tol(x: float) -> float:
    return REL_TIE * max(abs(x), 1e-30)


def assert_topset_consistent(ref_scores: np.ndarray, chosen: np.ndarray, k: int, what: str = ""):
    """`chosen` (k indices) is a top-k of ref_scores up to ties within REL_TIE."""
    ref_scores = np.asarray(ref_scores, dtype=np.float64)
    chosen = np.asarray(chosen, dtype=np.int64)
    assert len(chosen) == k and len(np.unique(chosen)) == k, f"{what}: {len(chosen)} vs {k}"
    if k == 0:
        return
    order = np.sort(ref_scores)[::-1]
    kth = order[k - 1]
    nxt = order[k] if k < len(order) else -np.inf
    mask = np.zeros(len(ref_scores), bool)
    mask[chosen] = True
    inside_min = ref_scores[mask].min()
    outside_max = ref_scores[~mask].max() if (~mask).any() else -np.inf
    assert inside_min >= kth - _tie_tol(kth), f"{what}: chosen score {inside_min} below k-th {kth}"
    if np.isfinite(nxt):
        assert outside_max <= nxt + _tie_tol(nxt), f"{what}: unchosen {outside_max} above {nxt}"


def count_window(ref_logits: np.ndarray, top_p: float):
    """Counts acceptable for top-p over these logits: [lo, hi] such that every c
    in it crosses p within the fp32 cumsum error bound."""
    x = np.sort(np.asarray(ref_logits, dtype=np.float64))[::-1]
    e = np.exp(x - x[0])
    cum = np.cumsum(e) / e.sum()
    n = len(x)
    delta = n * 2.0 ** -24
    ok = [c for c in range(1, n + 1) if cum[c - 1] >= top_p - delta and (c == 1 or cum[c - 2] < top_p + delta)]
    return (min(ok), max(ok)) if ok else (n, n)


def assert_top_p_consistent(ref_logits: np.ndarray, selected_idx: np.ndarray, count: int,
                            top_p: float, what: str = ""):
    lo, hi = count_window(ref_logits, top_p)
    assert lo <= count <= hi, f"{what}: count {count} outside acceptable [{lo}, {hi}]"
    assert_topset_consistent(ref_logits, selected_idx, count, what)
