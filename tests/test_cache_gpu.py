"""The drop-in cache API on the GPU, checked against the oracle.

Mirrors the reference's own tests (scripts/test_twilight_offload_cache_v1.py):
layer-batched selection, GQA union == sorted unique of the per-query-head sets,
gathered K/V rows == host slab rows followed by the current token, attention
metadata (cu_seqlens / lengths / max), consecutive decode steps, error paths.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import exact, synth, torch_ref
from pipeline import DTYPE_CODE, bits, twilight_oracle
from tolerance import ATTN_TOL_16BIT

pytestmark = pytest.mark.gpu

KV = dict(sink=64, recent=256, block=16)


def make_twilight(tw, dev, *, layers, G, R, L, dtype, b0_tokens=256, top_p=0.95, group=32,
                  extra=0, **kw):
    return tw.TwilightMatchedBudgetOffloadedCache(
        num_cache_entries=layers * G, max_cache_len=L + extra + 8, head_dim=128,
        num_query_heads_per_kv=R, dtype=dtype, device=dev, sink_tokens=KV["sink"],
        recent_tokens=KV["recent"], block_size=KV["block"], candidate_token_budget=b0_tokens,
        top_p=top_p, budget_mode="dynamic", layer_batched_selection=True,
        gqa_groupwise_execution=True, qk_backend="cuda", int4_group_size=group, **kw)


def layer_data(layers, G, R, L, dtype, seed):
    return [synth.make_layer(groups=G, heads_per_group=R, length=L, dtype=dtype, seed=seed + i,
                             workload="outliers") for i in range(layers)]


def _step_inputs(dev, G, R, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(G, R, 128, generator=g).to(synth.TORCH_DTYPES[dtype])
    kn = torch.randn(G, 128, generator=g).to(synth.TORCH_DTYPES[dtype])
    vn = torch.randn(G, 128, generator=g).to(synth.TORCH_DTYPES[dtype])
    return q, kn, vn


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_gqa_group_steps_match_oracle(tw, cuda, dtype):
    layers, G, R, L = 2, 2, 4, 1536
    data = layer_data(layers, G, R, L, dtype, 40)
    cache = make_twilight(tw, cuda, layers=layers, G=G, R=R, L=L, dtype=synth.TORCH_DTYPES[dtype],
                          extra=4)
    for li, d in enumerate(data):
        for g in range(G):
            cache.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda),
                         li * G + g)
    history = [[d.keys.clone(), d.values.clone()] for d in data]
    for step in range(3):
        old = L + step
        for li in range(layers):
            entries = [li * G + g for g in range(G)]
            q, kn, vn = _step_inputs(cuda, G, R, dtype, 1000 * step + li)
            qs = [q[g].view(1, R, 1, 128).to(cuda) for g in range(G)]
            ks = [kn[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
            vs = [vn[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
            cache.prepare_layer_selection(entries=entries, queries=qs)
            k, v, cu, max_k, lengths = cache.update_layer_gqa_group_ragged(
                key_states=ks, value_states=vs, queries=qs, entries=entries)
            keys_hist, vals_hist = history[li]
            # prompt pages only (reference candidate window); INT4 codes as on CUDA
            ref = twilight_oracle(keys_hist, q, old_length=old, sink=KV["sink"], recent=KV["recent"],
                                  block=KV["block"], b0_tokens=256, top_p=0.95, group=32, scale_div=0,
                                  meta_pages=(L - KV["sink"]) // KV["block"])
            offs = cu.cpu().tolist()
            assert offs[0] == 0 and len(offs) == G + 1
            assert max_k == max(lengths)
            for g in range(G):
                u = torch.as_tensor(ref.unions[g], dtype=torch.long)
                assert lengths[g] == u.numel() + 1
                assert offs[g + 1] - offs[g] == lengths[g]
                exp_k = torch.cat((keys_hist[g].index_select(0, u), kn[g:g + 1]))
                exp_v = torch.cat((vals_hist[g].index_select(0, u), vn[g:g + 1]))
                assert torch.equal(k[offs[g]:offs[g + 1], 0].cpu(), exp_k)
                assert torch.equal(v[offs[g]:offs[g + 1], 0].cpu(), exp_v)
                # host slab row `old` now holds the appended token
                assert torch.equal(cache._host_tensor("key", li * G + g)[0, 0, old], kn[g])
            history[li] = [torch.cat((keys_hist, kn[:, None]), 1), torch.cat((vals_hist, vn[:, None]), 1)]
    assert cache.get_seq_length(0) == L + 3
    cache.close()


def test_union_is_sorted_unique_of_per_head_sets(tw, cuda):
    """hi/twilight_offload_cache.py GQA semantics: one exact sorted union per KV
    head of the per-query-head selections plus sink and recent tokens."""
    G, R, L = 2, 4, 2048
    d = layer_data(1, G, R, L, "float16", 7)[0]
    cache = make_twilight(tw, cuda, layers=1, G=G, R=R, L=L, dtype=torch.float16)
    for g in range(G):
        cache.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda), g)
    cache.enable_selection_trace()
    cache.enable_budget_trace()
    cache.enable_metrics()
    qs = [d.queries[g].view(1, R, 1, 128).to(cuda) for g in range(G)]
    cache.prepare_layer_selection(entries=[0, 1], queries=qs)
    ks = [d.key_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    vs = [d.value_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    k, v, cu, max_k, lengths = cache.update_layer_gqa_group_ragged(key_states=ks, value_states=vs,
                                                                   queries=qs, entries=[0, 1])
    metrics = cache.resolve_metrics()
    trace = cache.selection_trace()
    sink_end, recent_start = 64, L - 255
    total_union = 0
    for g in range(G):
        rows = [torch.tensor(t["selected_positions"], dtype=torch.long) for t in trace if t["entry"] == g]
        assert len(rows) == R
        protected = torch.cat((torch.arange(sink_end), torch.arange(recent_start, L)))
        expected = torch.unique(torch.cat(rows + [protected]), sorted=True)
        assert lengths[g] == expected.numel() + 1
        assert cache._cached_group_positions[g].numel() == expected.numel()
        assert torch.equal(cache._cached_group_positions[g], expected)
        total_union += expected.numel()
    for row in cache.budget_trace():
        assert 1 <= row["raw_b1_tokens"] <= row["b0_tokens"]
        assert row["selected_history_tokens"] == row["protected_tokens"] + row["selected_adaptive_tokens"]
    assert metrics["h2d_bytes"] == 2 * total_union * 128 * 2
    assert cache.state_snapshot()["host_slab_device_mapped"]
    cache.close()


@pytest.mark.parametrize("R", [4, 8])
def test_attend_layer_matches_ragged_path(tw, cuda, R):
    G, L = 2, 4096
    d = layer_data(1, G, R, L, "bfloat16", 21)[0]
    caches = [make_twilight(tw, cuda, layers=1, G=G, R=R, L=L, dtype=torch.bfloat16, b0_tokens=512)
              for _ in range(2)]
    for c in caches:
        for g in range(G):
            c.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda), g)
    qs = [d.queries[g].view(1, R, 1, 128).to(cuda) for g in range(G)]
    ks = [d.key_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    vs = [d.value_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    for c in caches:
        c.prepare_layer_selection(entries=[0, 1], queries=qs)
    fused = caches[0].attend_layer(key_states=ks, value_states=vs, queries=qs, entries=[0, 1])
    k, v, cu, max_k, lengths = caches[1].update_layer_gqa_group_ragged(
        key_states=ks, value_states=vs, queries=qs, entries=[0, 1])
    q = torch.stack([x[0, :, 0] for x in qs])
    flat = tw.flash_attention_varlen_forward(q, k, v, torch.arange(G + 1, dtype=torch.int32, device=cuda),
                                             cu, 1, max_k, dropout=0.0, is_causal=True)
    torch.cuda.synchronize()
    assert torch.equal(fused, flat)
    offs = cu.cpu().tolist()
    for g in range(G):
        ref = torch_ref.decode_attention(q[g].cpu(), k[offs[g]:offs[g + 1], 0].cpu(),
                                         v[offs[g]:offs[g + 1], 0].cpu())
        assert (fused[g].cpu().double() - ref).abs().max().item() < ATTN_TOL_16BIT
    for c in caches:
        c.close()


def test_quest_per_head_paths(tw, cuda):
    """QuestTopKOffloadedCache: batched selection + flat ragged layer, and the
    per-entry update pack, against the exact oracle's pages."""
    G, R, L = 2, 4, 1024
    d = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype="float16", seed=14,
                         workload="needles", n_needles=8)
    kwargs = dict(num_cache_entries=G, max_cache_len=L + 8, head_dim=128, num_query_heads_per_kv=R,
                  dtype=torch.float16, device=cuda, budget_fraction=0.36, **{
                      "sink_tokens": 64, "recent_tokens": 256, "block_size": 16})
    flat = tw.QuestTopKOffloadedCache(layer_batched_selection=True, layer_flat_ragged_execution=True,
                                      **kwargs)
    per_entry = tw.QuestTopKOffloadedCache(**kwargs)
    for c in (flat, per_entry):
        for g in range(G):
            c.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda), g)
    qs = [d.queries[g].view(1, R, 1, 128).to(cuda) for g in range(G)]
    ks = [d.key_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    vs = [d.value_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    flat.enable_selection_trace()
    flat.prepare_layer_selection(entries=[0, 1], queries=qs)
    k, v, cu, max_k, lengths = flat.update_layer_flat_ragged(key_states=ks, value_states=vs,
                                                             queries=qs, entries=[0, 1])
    kb = bits(d.keys)
    P = (L - 255 - 64) // 16
    pm = np.stack([exact.quest_page_metadata(kb[g], 64, 16, 0)[0][:P] for g in range(G)])
    px = np.stack([exact.quest_page_metadata(kb[g], 64, 16, 0)[1][:P] for g in range(G)])
    scores = exact.quest_score(d.queries.float().numpy(), pm, px, 0)
    k_pages = int(np.ceil(0.36 * (L - 255 - 64) / 16))
    pages = exact.topk_pages(scores, k_pages)
    _, positions, _ = torch_ref.quest_select(d.queries.float(), torch.from_numpy(pm.view(np.int16)).view(torch.float16),
                                             torch.from_numpy(px.view(np.int16)).view(torch.float16),
                                             old_length=L, sink=64, recent=256, block=16,
                                             budget_fraction=0.36)
    seg = lengths[0]
    assert all(x == seg for x in lengths) and max_k == seg and len(lengths) == G * R
    for g in range(G):
        for r in range(R):
            trace = [t for t in flat.selection_trace() if t["entry"] == g and t["query_head_in_group"] == r]
            assert list(trace[0]["selected_page_indices"]) == pages[g, r].tolist()
            pos = torch.cat((torch.arange(64),
                             (64 + torch.from_numpy(pages[g, r]).long()[:, None] * 16 + torch.arange(16)).reshape(-1),
                             torch.arange(L - 255, L)))
            s = g * R + r
            exp = torch.cat((d.keys[g].index_select(0, pos), d.key_new[g:g + 1]))
            assert torch.equal(k[s * seg:(s + 1) * seg, 0].cpu(), exp)
    for g in range(G):
        key_pack, val_pack = per_entry.update(ks[g], vs[g], g, {"query_states": qs[g]})
        assert key_pack.shape == (1, R, seg, 128)
        for r in range(R):
            s = g * R + r
            assert torch.equal(key_pack[0, r].cpu(), k[s * seg:(s + 1) * seg, 0].cpu())
        assert per_entry.get_last_query_head_lengths(g) == tuple([seg] * R)
    flat.close()
    per_entry.close()


def test_error_paths(tw, cuda):
    G, R, L = 2, 4, 512
    d = layer_data(1, G, R, L, "float16", 3)[0]
    cache = make_twilight(tw, cuda, layers=1, G=G, R=R, L=L, dtype=torch.float16)
    with pytest.raises(ValueError, match="strict sequential"):
        cache.update(d.keys[1].view(1, 1, L, 128).to(cuda), d.values[1].view(1, 1, L, 128).to(cuda), 1)
    for g in range(G):
        cache.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda), g)
    qs = [d.queries[g].view(1, R, 1, 128).to(cuda) for g in range(G)]
    ks = [d.key_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    vs = [d.value_new[g].view(1, 1, 1, 128).to(cuda) for g in range(G)]
    with pytest.raises(ValueError, match="Query shape"):
        cache.prepare_layer_selection(entries=[0, 1], queries=[q[:, :2] for q in qs])
    with pytest.raises(AssertionError, match="prepared"):
        cache.update_layer_gqa_group_ragged(key_states=ks, value_states=vs, queries=qs, entries=[0, 1])
    with pytest.raises(NotImplementedError):
        cache.reorder_cache(torch.zeros(1, dtype=torch.long))
    with pytest.raises(NotImplementedError):
        cache.update(ks[0], vs[0], 0, {"query_states": qs[0]})
    cache.close()
    small = make_twilight(tw, cuda, layers=1, G=1, R=R, L=64, dtype=torch.float16)
    small.update(d.keys[0, :64].reshape(1, 1, 64, 128).to(cuda), d.values[0, :64].reshape(1, 1, 64, 128).to(cuda), 0)
    with pytest.raises(RuntimeError, match="capacity"):
        small.update(d.keys[0, :64].reshape(1, 1, 64, 128).to(cuda), d.values[0, :64].reshape(1, 1, 64, 128).to(cuda), 0)
    small.close()


@pytest.mark.parametrize("R,dtype", [(4, "float16"), (8, "bfloat16"), (3, "bfloat16")])
def test_decode_layer_equals_prepare_plus_attend(tw, cuda, R, dtype):
    """The one-call layer-step (tw_twilight_decode_layer) gives the same unions
    and attention output, bit for bit, as prepare_layer_selection + attend_layer,
    over consecutive steps (its append feeds the next step)."""
    G, L = 2, 3072
    tdt = synth.TORCH_DTYPES[dtype]
    d = layer_data(1, G, R, L, dtype, 31)[0]
    caches = [make_twilight(tw, cuda, layers=1, G=G, R=R, L=L, dtype=tdt, extra=4, b0_tokens=512)
              for _ in range(2)]
    for c in caches:
        for g in range(G):
            c.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda), g)
    for step in range(3):
        q, kn, vn = _step_inputs(cuda, G, R, dtype, 500 + step)
        q, kn, vn = q.to(cuda), kn.to(cuda), vn.to(cuda)
        qs = [q[g].view(1, R, 1, 128) for g in range(G)]
        ks = [kn[g].view(1, 1, 1, 128) for g in range(G)]
        vs = [vn[g].view(1, 1, 1, 128) for g in range(G)]
        caches[0].prepare_layer_selection(entries=[0, 1], queries=qs)
        two = caches[0].attend_layer(key_states=ks, value_states=vs, queries=qs, entries=[0, 1])
        one = caches[1].decode_layer(queries=q, key_states=kn, value_states=vn, entries=[0, 1])
        torch.cuda.synchronize()
        assert torch.equal(one, two), step
        b0, b1 = caches[0]._layer_bufs[G], caches[1]._layer_bufs[G]
        assert torch.equal(b0["union_count"], b1["union_count"])
        for g in range(G):
            n = int(b0["union_count"][g])
            assert torch.equal(b0["union_pos"][g, :n], b1["union_pos"][g, :n])
    assert caches[1].get_seq_length(0) == L + 3
    for c in caches:
        c.synchronize()
        c.close()


def test_resident_heads_match_offloaded(tw, cuda):
    """GPU-resident entries (device K/V) and offloaded entries (mapped host slab)
    go through one directory: a cache with half its heads resident gives the same
    unions, gathered rows and attention, bit for bit, as a fully offloaded one,
    and the appended token lands where its entry lives."""
    layers, G, R, L = 2, 4, 4, 2048
    data = layer_data(layers, G, R, L, "bfloat16", 71)
    plain = make_twilight(tw, cuda, layers=layers, G=G, R=R, L=L, dtype=torch.bfloat16, extra=4)
    mixed = make_twilight(tw, cuda, layers=layers, G=G, R=R, L=L, dtype=torch.bfloat16, extra=4,
                          resident_entries=[0, 3, 5, 6])
    assert mixed.state_snapshot()["resident_entries"] == [0, 3, 5, 6]
    for c in (plain, mixed):
        for li, d in enumerate(data):
            for g in range(G):
                c.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda),
                         li * G + g)
    assert mixed.entry_kv("key", 3).is_cuda and not mixed.entry_kv("key", 2).is_cuda
    for step in range(2):
        for li in range(layers):
            entries = [li * G + g for g in range(G)]
            q, kn, vn = _step_inputs(cuda, G, R, "bfloat16", 900 + 10 * step + li)
            q, kn, vn = q.to(cuda), kn.to(cuda), vn.to(cuda)
            if step == 0:
                qs = [q[g].view(1, R, 1, 128) for g in range(G)]
                ks = [kn[g].view(1, 1, 1, 128) for g in range(G)]
                vs = [vn[g].view(1, 1, 1, 128) for g in range(G)]
                outs = []
                for c in (plain, mixed):
                    c.prepare_layer_selection(entries=entries, queries=qs)
                    outs.append(c.update_layer_gqa_group_ragged(key_states=ks, value_states=vs,
                                                                queries=qs, entries=entries))
                for i in range(3):
                    assert torch.equal(outs[0][i], outs[1][i])
                assert outs[0][3:] == outs[1][3:]
            else:
                a = plain.decode_layer(queries=q, key_states=kn, value_states=vn, entries=entries)
                b = mixed.decode_layer(queries=q, key_states=kn, value_states=vn, entries=entries)
                torch.cuda.synchronize()
                assert torch.equal(a, b)
            for g in range(G):
                e = li * G + g
                assert torch.equal(mixed.entry_kv("key", e)[L + step].cpu(), kn[g].cpu())
    for c in (plain, mixed):
        c.synchronize()
        c.close()


@pytest.mark.parametrize("resident", [(), (1, 2)])
def test_prefill_layer_equals_per_entry_update(tw, cuda, resident):
    """prefill_layer (one metadata / INT4 launch per layer, pitched slab copies
    on a side stream) leaves the slab, the resident K/V, the page metadata and
    the INT4 codes exactly as per-entry update() does, and decodes identically."""
    G, R, L = 4, 4, 2000
    d = layer_data(1, G, R, L, "bfloat16", 88)[0]
    caches = [make_twilight(tw, cuda, layers=1, G=G, R=R, L=L, dtype=torch.bfloat16, extra=4,
                            resident_entries=list(resident)) for _ in range(2)]
    for g in range(G):
        caches[0].update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda), g)
    caches[1].prefill_layer(key_states=d.keys.view(1, G, L, 128).to(cuda),
                            value_states=d.values.view(1, G, L, 128).to(cuda), entries=list(range(G)))
    torch.cuda.synchronize()
    a, b = caches
    for g in range(G):
        for kind in ("key", "value"):
            assert torch.equal(a.entry_kv(kind, g)[:L].cpu(), b.entry_kv(kind, g)[:L].cpu())
    # pages with metadata: the complete pages after the sink plus the partial page
    pages = -(-(L - a.sink_tokens) // a.block_size)
    for name in ("_page_min", "_page_max"):
        assert torch.equal(getattr(a, name)[:, :pages], getattr(b, name)[:, :pages]), name
    for name in ("_packed", "_scale", "_minimum"):
        assert torch.equal(getattr(a, name)[:, :L], getattr(b, name)[:, :L]), name
    assert a._meta_pages == b._meta_pages and a.get_seq_length(0) == b.get_seq_length(0) == L
    q, kn, vn = _step_inputs(cuda, G, R, "bfloat16", 5)
    q, kn, vn = q.to(cuda), kn.to(cuda), vn.to(cuda)
    outs = [c.decode_layer(queries=q, key_states=kn, value_states=vn, entries=list(range(G)))
            for c in caches]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    with pytest.raises((ValueError, RuntimeError)):
        b.prefill_layer(key_states=d.keys.view(1, G, L, 128).to(cuda),
                        value_states=d.values.view(1, G, L, 128).to(cuda), entries=list(range(G)))
    for c in caches:
        c.close()
