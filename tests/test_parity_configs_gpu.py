"""GPU parity at the benchmark's own shapes.

* Twilight layer-step at the timed configuration: one layer of 8 KV heads x 4
  query heads, D 128, 32768 tokens of K/V, K with 4 lognormal outlier channels
  per KV head, INT4 group 32, Quest B0 4096 tokens (256 pages of 16), dynamic
  top-p 0.95, sink 64, recent 256.  The fp16 case is bench.py's own layer
  (seed 0) and its first queries (torch.Generator seed 17).  Checked, through
  the one-call decode_layer path and through tw_select_layer:
  - unions and per-head counts equal the exact-order oracle (oracle/exact.c)
    bit for bit;
  - the per-head selections and counts lie within the tie rule of the
    reference's own fp32 operator sequence (oracle/torch_ref.twilight_select =
    hi/twilight_offload_cache.py:1128-1310: topk, argsort, softmax, cumsum,
    searchsorted);
  - attention matches the float64 oracle within 1e-3 with fp32 output and
    within 2e-2 with 16-bit output, over two consecutive decode steps (the
    second step sees the token the first one appended).
* Per-query-head Quest at 4096 tokens (hi/quest_offload_cache.py:330-338,
  373-374, 403-511): 8 KV x 4 query heads, top-64 pages of 16 per query head,
  8 needle pages per KV head, all KV in the host slab.  Selected page ids equal
  the exact oracle (and are tie-consistent with the reference's torch.topk),
  and each query head's attention over sink U pages U recent U current
  (hi/mp.py:420-473) matches the float64 oracle within 1e-3 (fp32 output).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import exact, synth, torch_ref
from pipeline import DTYPE_CODE, bits, twilight_oracle
from tolerance import (ATTN_TOL_16BIT, ATTN_TOL_FP32, assert_top_p_consistent,
                       assert_topset_consistent)

pytestmark = pytest.mark.gpu

CFG2 = dict(groups=8, heads=4, length=32768, sink=64, recent=256, block=16, b0_tokens=4096,
            top_p=0.95, int4_group=32, n_outlier_channels=4)


def _cfg2_layer(dtype: str):
    c = CFG2
    layer = synth.make_layer(groups=c["groups"], heads_per_group=c["heads"], length=c["length"],
                             dtype=dtype, seed=0, workload="outliers", sink=c["sink"],
                             recent=c["recent"], block=c["block"],
                             n_outlier_channels=c["n_outlier_channels"])
    gq = torch.Generator().manual_seed(17)  # bench.py's query stream of rank 0
    queries = torch.randn(2, c["groups"], c["heads"], 128, generator=gq).to(synth.TORCH_DTYPES[dtype])
    gn = torch.Generator().manual_seed(99)
    k2 = torch.randn(c["groups"], 128, generator=gn).to(synth.TORCH_DTYPES[dtype])
    v2 = torch.randn(c["groups"], 128, generator=gn).to(synth.TORCH_DTYPES[dtype])
    return layer, queries, (layer.key_new, layer.value_new), (k2, v2)


def _torch_reference(keys: torch.Tensor, q: torch.Tensor, old_length: int):
    """The reference's fp32 operator sequence on the prompt metadata / codes."""
    c = CFG2
    pm, px, pk, sc, mn = [], [], [], [], []
    prompt = keys[:, :c["length"]]
    for g in range(keys.shape[0]):
        a, b = torch_ref.quest_page_metadata(prompt[g], c["sink"], c["block"])
        p, s, m = torch_ref.affine_int4_pack_grouped(keys[g], c["int4_group"])
        pm.append(a); px.append(b); pk.append(p); sc.append(s); mn.append(m)
    return torch_ref.twilight_select(
        q.float(), torch.stack(pm), torch.stack(px), torch.stack(pk), torch.stack(sc),
        torch.stack(mn), old_length=old_length, sink=c["sink"], recent=c["recent"],
        block=c["block"], candidate_token_budget=c["b0_tokens"], top_p=c["top_p"])


def _check_against_reference(sel, pages: np.ndarray, head_count: np.ndarray, head_pos, what: str):
    """pages [G,R,b0] (any order), head_count [G,R], head_pos [G][R] positions:
    within the tie rule of the reference's own selection `sel`."""
    G, R, b0 = pages.shape
    equal_sets = 0
    for g in range(G):
        for r in range(R):
            tag = f"{what} g{g} r{r}"
            scores = sel.page_scores[g, r].numpy()
            assert_topset_consistent(scores, pages[g, r], b0, tag + " B0 pages")
            ref_pages = np.sort(sel.chosen_pages[g, r].numpy())
            if not np.array_equal(np.sort(pages[g, r]), ref_pages):
                continue  # a tie at the B0 boundary: the candidate sets differ by tied pages
            equal_sets += 1
            cand = sel.candidate_positions[g, r].numpy()
            logits = sel.logits[g, r].numpy()
            index = {int(p): i for i, p in enumerate(cand)}
            idx = np.array([index[int(p)] for p in head_pos[g][r]], dtype=np.int64)
            assert len(idx) == int(head_count[g, r])
            assert_top_p_consistent(logits, idx, int(head_count[g, r]), CFG2["top_p"], tag + " top-p")
    # the B0 stage agrees with the reference on (nearly) every row
    assert equal_sets >= G * R - 1, f"{what}: only {equal_sets} of {G * R} B0 sets equal"


def _make_cache(tw, dev, dtype, max_len):
    c = CFG2
    return tw.TwilightMatchedBudgetOffloadedCache(
        num_cache_entries=c["groups"], max_cache_len=max_len, head_dim=128,
        num_query_heads_per_kv=c["heads"], dtype=dtype, device=dev, sink_tokens=c["sink"],
        recent_tokens=c["recent"], block_size=c["block"], candidate_token_budget=c["b0_tokens"],
        top_p=c["top_p"], budget_mode="dynamic", layer_batched_selection=True,
        gqa_groupwise_execution=True, qk_backend="cuda", int4_group_size=c["int4_group"])


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_twilight_layer_step_at_benchmark_shape(tw, cuda, dtype):
    c = CFG2
    G, R, L = c["groups"], c["heads"], c["length"]
    tdt = synth.TORCH_DTYPES[dtype]
    layer, queries, (k1, v1), (k2, v2) = _cfg2_layer(dtype)
    cache = _make_cache(tw, cuda, tdt, L + 8)
    cache.prefill_layer(key_states=layer.keys.to(cuda), value_states=layer.values.to(cuda),
                        entries=list(range(G)))
    meta_pages = (L - c["sink"]) // c["block"]
    okw = dict(sink=c["sink"], recent=c["recent"], block=c["block"], b0_tokens=c["b0_tokens"],
               top_p=c["top_p"], group=c["int4_group"], scale_div=0, meta_pages=meta_pages)

    # tw_select_layer on the cache's metadata and codes, with per-head positions
    q0 = queries[0]
    ref = twilight_oracle(layer.keys, q0, old_length=L, **okw)
    w = ref.window
    n_cap = w.b0_pages * c["block"]
    union_pos = torch.zeros((G, L + 8), dtype=torch.int32, device=cuda)
    union_count = torch.zeros(G, dtype=torch.int32, device=cuda)
    head_count = torch.zeros((G, R), dtype=torch.int32, device=cuda)
    head_pos = torch.zeros((G, R, n_cap), dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    pages = tw.ops.select_layer(
        q0.float().to(cuda), cache._page_min[:G], cache._page_max[:G], w.candidate_pages,
        cache._packed[:G], cache._scale[:G], cache._minimum[:G], b0_pages=w.b0_pages,
        block_size=c["block"], sink=c["sink"], top_p=c["top_p"], old_length=L,
        sink_end=w.sink_end, recent_start=w.recent_start, union_pos=union_pos,
        union_count=union_count, head_count=head_count, head_pos=head_pos, error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    pages_np = pages.cpu().numpy()
    np.testing.assert_array_equal(np.sort(pages_np, axis=-1), np.sort(ref.pages, axis=-1))
    np.testing.assert_array_equal(head_count.cpu().numpy(), ref.head_count)
    hp = head_pos.cpu().numpy()
    gpu_head_pos = [[np.sort(hp[g, r, :ref.head_count[g, r]]) for r in range(R)] for g in range(G)]
    for g in range(G):
        assert int(union_count[g]) == len(ref.unions[g])
        np.testing.assert_array_equal(union_pos[g, :len(ref.unions[g])].cpu().numpy(), ref.unions[g])
        for r in range(R):
            np.testing.assert_array_equal(gpu_head_pos[g][r], np.sort(ref.head_pos[g][r]))
    sel = _torch_reference(layer.keys, q0, L)
    _check_against_reference(sel, pages_np, head_count.cpu().numpy(), gpu_head_pos, "select_layer")

    # two consecutive decode_layer steps (fp32 output, then 16-bit output)
    keys_hist, vals_hist = layer.keys, layer.values
    bufs = None
    for step, (q, kn, vn, out_dtype, tol) in enumerate((
            (queries[0], k1, v1, torch.float32, ATTN_TOL_FP32),
            (queries[1], k2, v2, tdt, ATTN_TOL_16BIT))):
        old = L + step
        ref = twilight_oracle(keys_hist, q, old_length=old, **okw)
        out = torch.empty((G, R, 128), dtype=out_dtype, device=cuda)
        cache.decode_layer(queries=q.to(cuda), key_states=kn.to(cuda), value_states=vn.to(cuda),
                           entries=list(range(G)), out=out)
        torch.cuda.synchronize()
        cache._check_error_flag()
        bufs = cache._layer_bufs[G]
        np.testing.assert_array_equal(bufs["head_count"].cpu().numpy(), ref.head_count)
        counts = bufs["union_count"].cpu().numpy()
        for g in range(G):
            u = ref.unions[g]
            assert counts[g] == len(u), (step, g, counts[g], len(u))
            np.testing.assert_array_equal(bufs["union_pos"][g, :len(u)].cpu().numpy(), u)
            ui = torch.as_tensor(u, dtype=torch.long)
            kk = torch.cat((keys_hist[g].index_select(0, ui), kn[g:g + 1]))
            vv = torch.cat((vals_hist[g].index_select(0, ui), vn[g:g + 1]))
            expect = torch_ref.decode_attention(q[g], kk, vv)
            e = (out[g].cpu().double() - expect).abs().max().item()
            assert e < tol, (step, g, e)
            # the new token is in the host slab at position `old`
            assert torch.equal(cache._host_tensor("key", g)[0, 0, old], kn[g])
            assert torch.equal(cache._host_tensor("value", g)[0, 0, old], vn[g])
        # counts within the tie rule of the reference's own fp32 sequence
        sel = _torch_reference(keys_hist, q, old)
        _check_against_reference(sel, ref.pages, ref.head_count, ref.head_pos, f"oracle step {step}")
        keys_hist = torch.cat((keys_hist, kn[:, None]), 1)
        vals_hist = torch.cat((vals_hist, vn[:, None]), 1)
    assert cache.get_seq_length(0) == L + 2
    cache.close()


def test_quest_per_head_at_benchmark_shape(tw, cuda):
    G, R, L, sink, recent, block, k_pages = 8, 4, 4096, 64, 256, 16, 64
    d = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype="float16", seed=1,
                         workload="needles", sink=sink, recent=recent, block=block, n_needles=8)
    sink_end, recent_start = sink, L - (recent - 1)
    eligible = recent_start - sink_end
    P = eligible // block
    # budget = ceil(fraction * eligible / block) = 64 pages (hi/quest_offload_cache.py:330-338)
    fraction = 0.27
    assert int(np.ceil(fraction * eligible / block)) == k_pages
    cache = tw.QuestTopKOffloadedCache(
        num_cache_entries=G, max_cache_len=L + 8, head_dim=128, num_query_heads_per_kv=R,
        dtype=torch.float16, device=cuda, sink_tokens=sink, recent_tokens=recent, block_size=block,
        budget_fraction=fraction, layer_batched_selection=True, layer_flat_ragged_execution=True)
    cache.prefill_layer(key_states=d.keys.to(cuda), value_states=d.values.to(cuda),
                        entries=list(range(G)))
    qs = [d.queries[g].view(1, R, 1, 128).to(cuda) for g in range(G)]
    ks = [d.key_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    vs = [d.value_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    cache.enable_selection_trace()
    cache.prepare_layer_selection(entries=list(range(G)), queries=qs)
    k, v, cu, max_k, lengths = cache.update_layer_flat_ragged(key_states=ks, value_states=vs,
                                                              queries=qs, entries=list(range(G)))
    q = torch.stack([x[0, :, 0] for x in qs]).reshape(G * R, 1, 128)
    out32 = tw.sparse_gqa_decode_attention(q, k.view(-1, 128), v.view(-1, 128), cu, max_k,
                                                     out_dtype=torch.float32)
    out16 = tw.flash_attention_varlen_forward(q, k, v, torch.arange(G * R + 1, dtype=torch.int32,
                                                                    device=cuda), cu, 1, max_k)
    torch.cuda.synchronize()

    kb = bits(d.keys)
    pm = np.stack([exact.quest_page_metadata(kb[g], sink, block, 0)[0][:P] for g in range(G)])
    px = np.stack([exact.quest_page_metadata(kb[g], sink, block, 0)[1][:P] for g in range(G)])
    scores = exact.quest_score(d.queries.float().numpy(), pm, px, 0)
    pages = np.sort(exact.topk_pages(scores, k_pages), axis=-1)
    t_pages, positions, t_scores = torch_ref.quest_select(
        d.queries.float(), torch.from_numpy(pm.view(np.int16)).view(torch.float16),
        torch.from_numpy(px.view(np.int16)).view(torch.float16), old_length=L, sink=sink,
        recent=recent, block=block, budget_fraction=fraction)
    seg = sink_end + k_pages * block + (L - recent_start) + 1
    assert lengths == tuple([seg] * (G * R)) and max_k == seg
    for g in range(G):
        for r in range(R):
            s = g * R + r
            trace = [t for t in cache.selection_trace()
                     if t["entry"] == g and t["query_head_in_group"] == r]
            chosen = np.array(trace[-1]["selected_page_indices"])
            np.testing.assert_array_equal(np.sort(chosen), pages[g, r])
            assert_topset_consistent(t_scores[g, r].numpy(), chosen, k_pages, f"quest g{g} r{r}")
            pos = torch.cat((torch.arange(sink_end),
                             (sink + torch.from_numpy(pages[g, r]).long()[:, None] * block
                              + torch.arange(block)).reshape(-1),
                             torch.arange(recent_start, L)))
            assert torch.equal(pos, positions[g][r])
            kk = torch.cat((d.keys[g].index_select(0, pos), d.key_new[g:g + 1]))
            vv = torch.cat((d.values[g].index_select(0, pos), d.value_new[g:g + 1]))
            assert torch.equal(k[s * seg:(s + 1) * seg, 0].cpu(), kk)
            expect = torch_ref.decode_attention(d.queries[g, r:r + 1], kk, vv)[0]
            assert (out32[s, 0].cpu().double() - expect).abs().max().item() < ATTN_TOL_FP32
            assert (out16[s, 0].cpu().double() - expect).abs().max().item() < ATTN_TOL_16BIT
    cache.close()
