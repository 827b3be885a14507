"""Pin the oracle (oracle/exact.c, oracle/torch_ref.py) to the reference itself.

Golden vectors come from the reference's own code run on CPU
(tests/golden/make_golden.py); inputs are regenerated from oracle/synth.py
and checked against the recorded input checksums.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import exact, synth, torch_ref
from pipeline import DTYPE_CODE, bits, twilight_oracle
from tolerance import REL_TIE, assert_top_p_consistent, assert_topset_consistent, count_window

GOLDEN = Path(__file__).resolve().parent / "golden"

TWILIGHT = {
    "twilight_outliers": dict(groups=2, heads=4, length=2048, dtype="float16", seed=11,
                              workload="outliers", sink=64, recent=256, block=16, b0_tokens=512,
                              top_p=0.95, n_needles=0),
    "twilight_needles": dict(groups=2, heads=4, length=1536, dtype="bfloat16", seed=12,
                             workload="needles", sink=64, recent=256, block=16, b0_tokens=256,
                             top_p=0.9, n_needles=8),
    "twilight_tiny": dict(groups=2, heads=3, length=16, dtype="bfloat16", seed=13,
                          workload="outliers", sink=1, recent=2, block=1, b0_tokens=8, top_p=0.85,
                          n_needles=0),
}
QUEST = dict(groups=2, heads=4, length=1024, dtype="float16", seed=14, workload="needles", sink=64,
             recent=256, block=16, budget_fraction=0.36, n_needles=8)


def _sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def _layer(cfg):
    layer = synth.make_layer(groups=cfg["groups"], heads_per_group=cfg["heads"],
                             length=cfg["length"], dtype=cfg["dtype"], seed=cfg["seed"],
                             workload=cfg["workload"], sink=cfg["sink"], recent=cfg["recent"],
                             block=cfg["block"], n_needles=cfg["n_needles"])
    return layer


def _load(name, layer):
    g = np.load(GOLDEN / f"{name}.npz")
    assert list(g["inputs_sha256"]) == [_sha(layer.keys), _sha(layer.values), _sha(layer.queries)], \
        "synthetic generator drifted from the golden inputs"
    return g


def _vals(bits_i16: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(bits_i16).view(np.int16)).view(dtype).float().numpy()


@pytest.mark.parametrize("name", list(TWILIGHT))
def test_metadata_and_int4_match_reference(name):
    cfg = TWILIGHT[name]
    layer = _layer(cfg)
    g = _load(name, layer)
    dt = synth.TORCH_DTYPES[cfg["dtype"]]
    code = DTYPE_CODE[dt]
    kb = bits(layer.keys)
    for e in range(cfg["groups"]):
        pmin, pmax = exact.quest_page_metadata(kb[e], cfg["sink"], cfg["block"], code)
        np.testing.assert_array_equal(_vals(pmin, dt), _vals(g["page_min"][e], dt))
        np.testing.assert_array_equal(_vals(pmax, dt), _vals(g["page_max"][e], dt))
        # The reference's cache packs on CPU here (IEEE divide by 15): scale_div=1.
        packed, scale, minimum = exact.int4_pack(kb[e], 128, code, 1)
        np.testing.assert_array_equal(packed, g["packed"][e])
        np.testing.assert_array_equal(_vals(scale[:, 0], dt), _vals(g["scale"][e], dt))
        np.testing.assert_array_equal(_vals(minimum[:, 0], dt), _vals(g["minimum"][e], dt))


def test_int4_group32_and_special_rows_match_reference():
    g = np.load(GOLDEN / "int4_pack.npz")
    layer = synth.make_layer(groups=2, heads_per_group=4, length=1024, dtype="float16", seed=21,
                             workload="outliers")
    assert g["inputs_sha256"][0] == _sha(layer.keys)
    for dname, code in (("float16", 0), ("bfloat16", 1)):
        dt = synth.TORCH_DTYPES[dname]
        keys = layer.keys.float().to(dt).reshape(-1, 128)
        for group, suffix in ((32, ""), (128, "128")):
            packed, scale, minimum = exact.int4_pack(bits(keys), group, code, 1)
            np.testing.assert_array_equal(packed, g[f"{dname}_packed{suffix}"])
            ref_s = g[f"{dname}_scale{suffix}"].reshape(scale.shape)
            ref_m = g[f"{dname}_minimum{suffix}"].reshape(minimum.shape)
            np.testing.assert_array_equal(_vals(scale, dt), _vals(ref_s, dt))
            np.testing.assert_array_equal(_vals(minimum, dt), _vals(ref_m, dt))
    packed, scale, minimum = exact.int4_pack(g["special_keys"].view(np.uint16), 128, 0, 1)
    np.testing.assert_array_equal(packed, g["special_packed"])
    np.testing.assert_array_equal(_vals(scale[:, 0], torch.float16), _vals(g["special_scale"], torch.float16))


@pytest.mark.parametrize("name", list(TWILIGHT))
def test_quest_scores_and_b0_pages_match_reference(name):
    cfg = TWILIGHT[name]
    layer = _layer(cfg)
    g = _load(name, layer)
    dt = synth.TORCH_DTYPES[cfg["dtype"]]
    ref_scores = g["page_scores"]
    P = ref_scores.shape[-1]
    q = layer.queries.float().numpy()
    pmin = np.ascontiguousarray(g["page_min"][:, :P]).view(np.uint16)
    pmax = np.ascontiguousarray(g["page_max"][:, :P]).view(np.uint16)
    scores = exact.quest_score(q, pmin, pmax, DTYPE_CODE[dt])
    scale = np.abs(ref_scores).max()
    assert np.max(np.abs(scores - ref_scores)) <= 8 * REL_TIE * scale
    w = torch_ref.window(cfg["length"], sink=cfg["sink"], recent=cfg["recent"], block=cfg["block"],
                         candidate_token_budget=cfg["b0_tokens"], metadata_pages=g["page_min"].shape[1])
    pages = exact.topk_pages(scores, w.b0_pages)
    for gi in range(cfg["groups"]):
        for r in range(cfg["heads"]):
            assert_topset_consistent(ref_scores[gi, r], pages[gi, r], w.b0_pages, f"{name} {gi} {r}")


@pytest.mark.parametrize("name", list(TWILIGHT))
def test_twilight_selection_matches_reference(name):
    cfg = TWILIGHT[name]
    layer = _layer(cfg)
    g = _load(name, layer)
    L = cfg["length"]
    sel = twilight_oracle(layer.keys, layer.queries, old_length=L, sink=cfg["sink"],
                          recent=cfg["recent"], block=cfg["block"], b0_tokens=cfg["b0_tokens"],
                          top_p=cfg["top_p"], group=128, scale_div=1)
    ref_counts = g["desired"]
    exact_match = np.array_equal(sel.head_count, ref_counts) and all(
        np.array_equal(sel.unions[gi], g["unions"][gi][: g["union_counts"][gi]])
        for gi in range(cfg["groups"]))
    if exact_match:
        for gi in range(cfg["groups"]):
            for r in range(cfg["heads"]):
                ref_row = g["per_head"][gi, r][g["per_head"][gi, r] >= 0]
                np.testing.assert_array_equal(np.sort(sel.head_pos[gi][r]), ref_row)
        return
    # Differences must be explained by ties / the fp32 cumsum boundary of the reference.
    ref = torch_ref.twilight_select(
        layer.queries.float(), torch.from_numpy(g["page_min"]).view(layer.keys.dtype),
        torch.from_numpy(g["page_max"]).view(layer.keys.dtype), torch.from_numpy(g["packed"]),
        torch.from_numpy(g["scale"]).view(layer.keys.dtype),
        torch.from_numpy(g["minimum"]).view(layer.keys.dtype), old_length=L, sink=cfg["sink"],
        recent=cfg["recent"], block=cfg["block"], candidate_token_budget=cfg["b0_tokens"],
        top_p=cfg["top_p"])
    for gi in range(cfg["groups"]):
        for r in range(cfg["heads"]):
            cand = ref.candidate_positions[gi, r].numpy()
            idx = np.nonzero(np.isin(cand, sel.head_pos[gi][r]))[0]
            assert_top_p_consistent(ref.logits[gi, r].numpy(), idx, int(sel.head_count[gi, r]),
                                    cfg["top_p"], f"{name} {gi} {r}")


@pytest.mark.parametrize("name", list(TWILIGHT))
def test_torch_ref_reproduces_reference(name):
    """oracle/torch_ref.py on CPU == the reference's own CPU run, bit for bit."""
    cfg = TWILIGHT[name]
    layer = _layer(cfg)
    g = _load(name, layer)
    dt = layer.keys.dtype
    pmin, pmax, packed, scale, minimum = [], [], [], [], []
    for e in range(cfg["groups"]):
        a, b = torch_ref.quest_page_metadata(layer.keys[e], cfg["sink"], cfg["block"])
        p, s, m = torch_ref.affine_int4_pack(layer.keys[e])
        pmin.append(a); pmax.append(b); packed.append(p); scale.append(s); minimum.append(m)
    np.testing.assert_array_equal(torch.stack(pmin).view(torch.int16).numpy(), g["page_min"])
    np.testing.assert_array_equal(torch.stack(packed).numpy(), g["packed"])
    sel = torch_ref.twilight_select(layer.queries.float(), torch.stack(pmin), torch.stack(pmax),
                                    torch.stack(packed), torch.stack(scale), torch.stack(minimum),
                                    old_length=cfg["length"], sink=cfg["sink"],
                                    recent=cfg["recent"], block=cfg["block"],
                                    candidate_token_budget=cfg["b0_tokens"], top_p=cfg["top_p"])
    np.testing.assert_array_equal(sel.desired.numpy(), g["desired"])
    for gi in range(cfg["groups"]):
        np.testing.assert_array_equal(sel.unions[gi].numpy(), g["unions"][gi][: g["union_counts"][gi]])
    assert dt in (torch.float16, torch.bfloat16)


@pytest.mark.parametrize("name", list(TWILIGHT))
def test_attention_oracle_matches_reference(name):
    cfg = TWILIGHT[name]
    layer = _layer(cfg)
    g = _load(name, layer)
    for gi in range(cfg["groups"]):
        u = torch.from_numpy(g["unions"][gi][: g["union_counts"][gi]])
        k = torch.cat((layer.keys[gi].index_select(0, u), layer.key_new[gi:gi + 1]))
        v = torch.cat((layer.values[gi].index_select(0, u), layer.value_new[gi:gi + 1]))
        out = torch_ref.decode_attention(layer.queries[gi], k, v)
        np.testing.assert_allclose(out.numpy(), g["attention"][gi], atol=1e-5, rtol=0)


def test_quest_pages_match_reference():
    cfg = QUEST
    layer = _layer(cfg)
    g = _load("quest_needles", layer)
    dt = layer.keys.dtype
    code = DTYPE_CODE[dt]
    kb = bits(layer.keys)
    P = g["page_scores"].shape[-1]
    pm = np.stack([exact.quest_page_metadata(kb[e], cfg["sink"], cfg["block"], code)[0] for e in range(2)])
    px = np.stack([exact.quest_page_metadata(kb[e], cfg["sink"], cfg["block"], code)[1] for e in range(2)])
    scores = exact.quest_score(layer.queries.float().numpy(), np.ascontiguousarray(pm[:, :P]),
                               np.ascontiguousarray(px[:, :P]), code)
    k = g["pages"].shape[-1]
    pages = exact.topk_pages(scores, k)
    for gi in range(2):
        for r in range(cfg["heads"]):
            assert_topset_consistent(g["page_scores"][gi, r], pages[gi, r], k, f"quest {gi} {r}")
            assert np.all(np.diff(pages[gi, r]) > 0)
    # torch_ref reproduces the reference's positions exactly
    chosen, positions, _ = torch_ref.quest_select(
        layer.queries.float(), torch.from_numpy(g["page_min"]).view(dt),
        torch.from_numpy(g["page_max"]).view(dt), old_length=cfg["length"], sink=cfg["sink"],
        recent=cfg["recent"], block=cfg["block"], budget_fraction=cfg["budget_fraction"])
    np.testing.assert_array_equal(chosen.numpy(), g["pages"])
    for gi in range(2):
        for r in range(cfg["heads"]):
            np.testing.assert_array_equal(positions[gi][r].numpy(), g["positions"][gi, r])


@pytest.mark.parametrize("kind", ["uniform", "ties", "peaked", "p_one", "single"])
def test_top_p_edge_cases_against_reference_ops(kind):
    """Top-p counts of the oracle vs the reference's own operator sequence
    (argsort / softmax / cumsum / searchsorted + 1) on constructed logits."""
    rng = np.random.default_rng(5)
    n, top_p = 256, 0.95
    if kind == "uniform":
        logits = np.zeros(n, np.float32)
    elif kind == "ties":
        logits = np.repeat(rng.standard_normal(16).astype(np.float32), n // 16)
    elif kind == "peaked":
        logits = (rng.standard_normal(n) * 8).astype(np.float32)
    elif kind == "p_one":
        logits = rng.standard_normal(n).astype(np.float32)
        top_p = 1.0
    else:
        logits = np.full(n, -1e4, np.float32)
        logits[7] = 0.0
    pages = np.arange(n // 16, dtype=np.int32).reshape(1, 1, -1)
    L = 64 + n + 300
    unions, hc, hp, bad = exact.top_p_union(logits.reshape(1, 1, n), pages, 16, 64, top_p, L, 64, L - 255)
    count = int(hc[0, 0])
    t = torch.from_numpy(logits).view(1, 1, n)
    order = torch.argsort(t, dim=-1, descending=True)
    probs = torch.softmax(torch.gather(t, -1, order), dim=-1)
    cum = probs[0, 0].cumsum(0)
    desired = int(torch.searchsorted(cum, torch.tensor([top_p]), right=False)) + 1
    desired = min(desired, n)
    lo, hi = count_window(logits, top_p)
    if kind == "p_one":
        assert count >= lo and desired >= lo  # both keep (almost) everything
    else:
        assert lo <= count <= hi and lo <= desired <= hi, (count, desired, lo, hi)
    sel_idx = (hp[0][0] - 64)
    assert_topset_consistent(logits, sel_idx, count, kind)
