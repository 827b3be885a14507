"""Generate golden vectors from the reference itself (run in a container that
holds the reference tree; the GPU box does not need it).

    python tests/golden/make_golden.py --reference /path/to/reference-checkout

(or with $TW_REFERENCE_ROOT set to the checkout).

It imports the reference's own modules (source/headinfer/headinfer/), builds a
TwilightMatchedBudgetOffloadedCache / QuestTopKOffloadedCache on device='cpu'
(the constructors require CUDA, so instances are made with __new__ and the
attributes the selection path reads), runs _build_metadata and
prepare_layer_selection exactly as the reference does, and saves inputs'
checksums and outputs as .npz next to this script.  Inputs are regenerated
from oracle/synth.py seeds at test time.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from oracle import synth  # noqa: E402
from oracle.ref_harness import make_ref_cache, make_twilight_cache  # noqa: E402

CASES = {
    # Twilight (Quest B0 -> INT4 per-token QK -> top-p -> GQA union), outliers.
    "twilight_outliers": dict(kind="twilight", groups=2, heads=4, length=2048, dtype="float16",
                              seed=11, workload="outliers", sink=64, recent=256, block=16,
                              b0_tokens=512, top_p=0.95, n_needles=0),
    # Same path with needles and bf16.
    "twilight_needles": dict(kind="twilight", groups=2, heads=4, length=1536, dtype="bfloat16",
                             seed=12, workload="needles", sink=64, recent=256, block=16,
                             b0_tokens=256, top_p=0.9, n_needles=8),
    # The reference unit-test geometry (sink 1, recent 2, block 1, B0 8, prompt 16), D=128.
    "twilight_tiny": dict(kind="twilight", groups=2, heads=3, length=16, dtype="bfloat16",
                          seed=13, workload="outliers", sink=1, recent=2, block=1, b0_tokens=8,
                          top_p=0.85, n_needles=0),
    # Quest per-query-head pages (budget 16 pages of 16) with needles, fp16.
    "quest_needles": dict(kind="quest", groups=2, heads=4, length=1024, dtype="float16",
                          seed=14, workload="needles", sink=64, recent=256, block=16,
                          budget_fraction=0.36, n_needles=8),
}


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def twilight_case(ref_twilight, ref_root, name, cfg):
    G, R, L = cfg["groups"], cfg["heads"], cfg["length"]
    tdt = synth.TORCH_DTYPES[cfg["dtype"]]
    layer = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype=cfg["dtype"],
                             seed=cfg["seed"], workload=cfg["workload"], sink=cfg["sink"],
                             recent=cfg["recent"], block=cfg["block"], n_needles=cfg["n_needles"])
    c = make_twilight_cache(ref_twilight, groups=G, heads=R, max_len=L + 8, dtype=tdt,
                            sink=cfg["sink"], recent=cfg["recent"], block=cfg["block"],
                            b0_tokens=cfg["b0_tokens"], top_p=cfg["top_p"], budget_trace=True)
    c._capture_selection_trace = True
    c._prompt_length = L
    for e in range(G):
        c._logical_lengths[e] = L
        c._build_metadata(e, layer.keys[e].view(1, 1, L, 128))
    queries = [layer.queries[g].view(1, R, 1, 128) for g in range(G)]
    c.prepare_layer_selection(entries=list(range(G)), queries=queries)

    out = {}
    out["page_min"] = torch.stack(c._page_min).view(torch.int16).numpy()
    out["page_max"] = torch.stack(c._page_max).view(torch.int16).numpy()
    out["packed"] = torch.stack(c._quant_key_packed).numpy()
    out["scale"] = torch.stack(c._quant_key_scale).view(torch.int16).numpy()
    out["minimum"] = torch.stack(c._quant_key_minimum).view(torch.int16).numpy()
    rows = c.budget_trace()
    desired = np.zeros((G, R), dtype=np.int64)
    for row in rows:
        desired[row["kv_head"], row["query_head_in_group"]] = row["raw_b1_tokens"]
    out["desired"] = desired
    per_head = [[c._cached_twilight_positions[g][r].numpy() for r in range(R)] for g in range(G)]
    n_max = max(len(x) for rr in per_head for x in rr)
    ph = np.full((G, R, n_max), -1, dtype=np.int64)
    for g in range(G):
        for r in range(R):
            ph[g, r, : len(per_head[g][r])] = per_head[g][r]
    out["per_head"] = ph
    unions = [c._cached_twilight_group_positions[g].numpy() for g in range(G)]
    u_max = max(len(u) for u in unions)
    un = np.full((G, u_max), -1, dtype=np.int64)
    for g in range(G):
        un[g, : len(unions[g])] = unions[g]
    out["unions"] = un
    out["union_counts"] = np.array([len(u) for u in unions], dtype=np.int64)
    # The stage intermediates (scores, chosen pages, logits) are recomputed here
    # with the reference's own expressions on the same inputs, for tolerance checks.
    q = torch.stack([x[0, :, 0] for x in queries]).float()
    w_pages = min(min(int(p.shape[0]) for p in c._page_min),
                  max(0, max(min(cfg["sink"], L), L - (cfg["recent"] - 1)) - min(cfg["sink"], L))
                  // cfg["block"])
    pmin = torch.stack([p[:w_pages] for p in c._page_min])
    pmax = torch.stack([p[:w_pages] for p in c._page_max])
    extrema = torch.where(q.unsqueeze(2) > 0, pmax.unsqueeze(1), pmin.unsqueeze(1))
    out["page_scores"] = (extrema.float() * q.unsqueeze(2)).sum(dim=-1).numpy()
    # attention over each union + the current token with the reference's SDPA-math helper
    from headinfer.decode_reference_attention import sdpa_math_decode_attention
    att = []
    for g in range(G):
        u = torch.from_numpy(unions[g])
        kk = torch.cat((layer.keys[g].index_select(0, u), layer.key_new[g:g + 1])).float()
        vv = torch.cat((layer.values[g].index_select(0, u), layer.value_new[g:g + 1])).float()
        o = sdpa_math_decode_attention(layer.queries[g].float().view(1, 1, R, 128),
                                       kk.view(1, -1, 1, 128), vv.view(1, -1, 1, 128), None, 1)
        att.append(o[0, 0])
    out["attention"] = torch.stack(att).numpy()
    out["inputs_sha256"] = np.array([sha(layer.keys), sha(layer.values), sha(layer.queries)])
    return out


def quest_case(ref_quest, name, cfg):
    G, R, L = cfg["groups"], cfg["heads"], cfg["length"]
    tdt = synth.TORCH_DTYPES[cfg["dtype"]]
    layer = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype=cfg["dtype"],
                             seed=cfg["seed"], workload=cfg["workload"], sink=cfg["sink"],
                             recent=cfg["recent"], block=cfg["block"], n_needles=cfg["n_needles"])
    c = make_ref_cache(ref_quest, "QuestTopKOffloadedCache", entries=G, max_len=L + 8, heads=R,
                       dtype=tdt, sink=cfg["sink"], recent=cfg["recent"], block=cfg["block"],
                       budget_fraction=cfg["budget_fraction"])
    c._prompt_length = L
    for e in range(G):
        c._logical_lengths[e] = L
        c._build_metadata(e, layer.keys[e].view(1, 1, L, 128))
    c._capture_selection_trace = True
    queries = [layer.queries[g].view(1, R, 1, 128) for g in range(G)]
    # prepare_layer_selection moves the chosen pages to CPU; _selected_positions
    # expands them (hi/quest_offload_cache.py:299-511).
    c.prepare_layer_selection(entries=list(range(G)), queries=queries)
    positions = [c._selected_positions(query=queries[g], entry=g, old_length=L) for g in range(G)]
    trace = c.selection_trace()
    k = len(trace[0]["selected_page_indices"])
    pages = np.zeros((G, R, k), dtype=np.int64)
    for row in trace:
        pages[row["entry"], row["query_head_in_group"]] = row["selected_page_indices"]
    out = {"pages": pages,
           "positions": np.stack([np.stack([p.numpy() for p in positions[g]]) for g in range(G)])}
    q = torch.stack([x[0, :, 0] for x in queries]).float()
    pmin = torch.stack(c._page_min)
    pmax = torch.stack(c._page_max)
    extrema = torch.where(q.unsqueeze(2) > 0, pmax.unsqueeze(1), pmin.unsqueeze(1))
    out["page_scores"] = (extrema.float() * q.unsqueeze(2)).sum(dim=-1).numpy()
    out["page_min"] = pmin.view(torch.int16).numpy()
    out["page_max"] = pmax.view(torch.int16).numpy()
    out["needle_pages"] = layer.needle_pages
    out["inputs_sha256"] = np.array([sha(layer.keys), sha(layer.values), sha(layer.queries)])
    return out


def int4_group32_case(ref_twilight):
    layer = synth.make_layer(groups=2, heads_per_group=4, length=1024, dtype="float16", seed=21,
                             workload="outliers")
    out = {}
    for dname in ("float16", "bfloat16"):
        keys = layer.keys.float().to(synth.TORCH_DTYPES[dname]).reshape(-1, 128)
        packed, scale, minimum = ref_twilight.affine_int4_pack(keys.reshape(-1, 32))
        out[f"{dname}_packed"] = packed.reshape(-1, 64).numpy()
        out[f"{dname}_scale"] = scale.reshape(-1, 4).view(torch.int16).numpy()
        out[f"{dname}_minimum"] = minimum.reshape(-1, 4).view(torch.int16).numpy()
        p128, s128, m128 = ref_twilight.affine_int4_pack(keys)
        out[f"{dname}_packed128"] = p128.numpy()
        out[f"{dname}_scale128"] = s128.view(torch.int16).numpy()
        out[f"{dname}_minimum128"] = m128.view(torch.int16).numpy()
    # constant rows (scale underflow in fp16) and ties to even
    special = torch.zeros(4, 128, dtype=torch.float16)
    special[1] = 1.0
    special[2, :64] = -3.0
    special[2, 64:] = 5.0
    special[3] = torch.arange(128, dtype=torch.float32).to(torch.float16) / 8
    sp, ss, sm = ref_twilight.affine_int4_pack(special)
    out["special_keys"] = special.view(torch.int16).numpy()
    out["special_packed"] = sp.numpy()
    out["special_scale"] = ss.view(torch.int16).numpy()
    out["special_minimum"] = sm.view(torch.int16).numpy()
    out["inputs_sha256"] = np.array([sha(layer.keys)])
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TW_REFERENCE_ROOT"),
                    help="the reference checkout (holds source/headinfer/headinfer/)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("--reference (or $TW_REFERENCE_ROOT) is required")
    sys.path.insert(0, str(Path(args.reference) / "source" / "headinfer"))
    torch.set_num_threads(1)
    from headinfer import quest_offload_cache, twilight_offload_cache

    for name, cfg in CASES.items():
        if cfg["kind"] == "twilight":
            out = twilight_case(twilight_offload_cache, args.reference, name, cfg)
        else:
            out = quest_case(quest_offload_cache, name, cfg)
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print("wrote", name, {k: getattr(v, "shape", None) for k, v in out.items()})
    out = int4_group32_case(twilight_offload_cache)
    np.savez_compressed(HERE / "int4_pack.npz", **out)
    print("wrote int4_pack")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
