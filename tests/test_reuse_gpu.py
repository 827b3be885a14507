"""Previous-token row reuse on the GPU (tw_row_reuse).

Kernel level: rows whose position the previous step kept (its union rows and
its token, recorded in the row map under the previous tag) are read from the
previous rows in device memory, every other row from the mapped slab; each
step records its own kept rows under its tag.  The tests plant previous rows that
differ from the slab so that the source of every row is visible, and compare
the hit / miss counters with the oracle's mapping (oracle/reuse.py, pinned to
the reference's map_rows).

Cache level: mirrors the reference's resident-cache check
(scripts/test_twilight_offload_cache_v1.py:380-430): with the previous-token
resident cache on, unions, gathered rows and attention equal the direct path
bit for bit over consecutive steps, the first step has no hits, later steps
do, and hit + miss rows = history rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import reuse as reuse_oracle
from oracle import synth
from pipeline import DTYPE_CODE

pytestmark = pytest.mark.gpu

DTYPES = [torch.float16, torch.bfloat16]


def _slab(tw, G, max_len, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    keys = torch.randn(G, max_len, 128, generator=g).to(dtype)
    vals = torch.randn(G, max_len, 128, generator=g).to(dtype)
    geom = tw.SlabGeometry(num_entries=G, batch_size=1, max_cache_len=max_len, head_dim=128)
    slab = tw.MappedHostSlab(geom, dtype)
    slab.rows[0].copy_(keys)
    slab.rows[1].copy_(vals)
    return slab, keys, vals, g


def _unions(g, L, prev_counts, cur_counts, prev_length):
    """Previous unions over [0, prev_length) and current unions over [0, L)
    that share part of their positions (and, for some groups, the previous
    step's token prev_length)."""
    prev, cur = [], []
    for gi, (pc, cc) in enumerate(zip(prev_counts, cur_counts)):
        p = torch.randperm(prev_length, generator=g)[:pc].sort().values
        shared = p[torch.randperm(pc, generator=g)[: min(pc, cc // 2)]] if pc else p[:0]
        extra = torch.randperm(L, generator=g)[: cc]
        c = torch.unique(torch.cat((shared, extra)))[:cc]
        if gi % 2 == 0 and prev_length < L:
            c = torch.unique(torch.cat((c[:-1], torch.tensor([prev_length]))))
        prev.append(p.long())
        cur.append(c.sort().values.long())
    return prev, cur


def _pad(lists, width, dev):
    out = torch.zeros((len(lists), width), dtype=torch.int32)
    for i, x in enumerate(lists):
        out[i, : len(x)] = x.int()
    return out.to(dev), torch.tensor([len(x) for x in lists], dtype=torch.int32, device=dev)


def _plant_map(row_map, prev, prev_length, tag, row_of):
    """Row-map entries of the previous step (tag) for its union rows and its
    token, plus stale entries (older tag) that must not be used."""
    m = torch.zeros_like(row_map, device="cpu")
    for gi, p in enumerate(prev):
        for j, pos in enumerate(p.tolist()):
            m[gi, pos] = (tag << 32) | row_of(gi, j)
        m[gi, prev_length] = (tag << 32) | row_of(gi, len(p))
        m[gi, 1] = ((tag - 1) << 32) | row_of(gi, 0) if 1 not in p.tolist() else m[gi, 1]
    row_map.copy_(m)


def _expected_source(prev, gi, pos, prev_length):
    rank = {int(p): j for j, p in enumerate(prev[gi].tolist())}
    return rank.get(pos, len(prev[gi]) if pos == prev_length else -1)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("R", [4, 8])
def test_attend_union_reads_previous_rows(tw, cuda, dtype, R):
    G, L, max_len = 3, 3000, 3100
    slab, keys, vals, g = _slab(tw, G, max_len, dtype, 11 + R)
    prev_length = L - 1
    prev, cur = _unions(g, L, [0, 40, 1800], [5, 60, 2200], prev_length)
    S = max(max(len(c) for c in cur), max(len(p) for p in prev)) + 1
    union_pos, union_count = _pad(cur, L, cuda)
    # planted previous rows (strided): slab row + 0.5 for union rows, a random row for the token
    prev_k = torch.zeros((G, S, 128), dtype=dtype)
    prev_v = torch.zeros_like(prev_k)
    for gi, p in enumerate(prev):
        prev_k[gi, : len(p)] = (keys[gi, p].float() + 0.5).to(dtype)
        prev_v[gi, : len(p)] = (vals[gi, p].float() - 0.5).to(dtype)
        prev_k[gi, len(p)] = torch.randn(128, generator=g).to(dtype)
        prev_v[gi, len(p)] = torch.randn(128, generator=g).to(dtype)
    prev_k, prev_v = prev_k.to(cuda), prev_v.to(cuda)
    row_map = torch.zeros((G, max_len), dtype=torch.int64, device=cuda)
    _plant_map(row_map, prev, prev_length, 7, lambda gi, j: gi * S + j)
    cur_k = torch.randn(G, 128, generator=g).to(dtype).to(cuda)
    cur_v = torch.randn(G, 128, generator=g).to(dtype).to(cuda)
    q = (torch.randn(G, R, 128, generator=g) * 2).to(dtype).to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ws = torch.zeros(tw.ops.decode_attention_workspace_bytes(G, R, S), dtype=torch.uint8, device=cuda)
    next_k = torch.full((G, S, 128), 7.0, dtype=dtype, device=cuda)
    next_v = torch.full_like(next_k, 7.0)
    counts = torch.zeros((G, 2), dtype=torch.int32, device=cuda)
    r = tw.ops.row_reuse(row_map, 8, next_k=next_k, next_v=next_v, prev_tag=7, prev_k=prev_k,
                         prev_v=prev_v, row_counts=counts)
    out = tw.ops.attend_union(slab, 0, L, union_pos, union_count, cur_k, cur_v, q, S, workspace=ws,
                              error_flag=err, reuse=r)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # expected rows: previous rows for hits, slab rows for misses, then the token
    flat_k, flat_v, cu = [], [], [0]
    m = row_map.cpu()
    for gi, c in enumerate(cur):
        ks, vs = [], []
        for i, pos in enumerate(c.tolist()):
            j = _expected_source(prev, gi, pos, prev_length)
            ks.append(prev_k[gi, j].cpu() if j >= 0 else keys[gi, pos])
            vs.append(prev_v[gi, j].cpu() if j >= 0 else vals[gi, pos])
            assert int(m[gi, pos]) == (8 << 32) | (gi * S + i)
        ks.append(cur_k[gi].cpu())
        vs.append(cur_v[gi].cpu())
        assert int(m[gi, L]) == (8 << 32) | (gi * S + len(c))
        ek, ev = torch.stack(ks), torch.stack(vs)
        n = len(c) + 1
        assert torch.equal(next_k[gi, :n].cpu(), ek), gi
        assert torch.equal(next_v[gi, :n].cpu(), ev), gi
        flat_k.append(ek)
        flat_v.append(ev)
        cu.append(cu[-1] + n)
    staged = tw.ops.decode_attention(q, torch.cat(flat_k).to(cuda), torch.cat(flat_v).to(cuda),
                                     torch.tensor(cu, dtype=torch.int32, device=cuda), S, workspace=ws)
    assert torch.equal(out, staged)
    want = reuse_oracle.group_hit_miss(prev, cur, prev_length)
    np.testing.assert_array_equal(counts.cpu().numpy(), want)
    # no previous rows (prev_tag 0): every history row is a miss, rows are kept
    counts.zero_()
    first = tw.ops.row_reuse(row_map, 9, next_k=next_k, next_v=next_v, row_counts=counts)
    out0 = tw.ops.attend_union(slab, 0, L, union_pos, union_count, cur_k, cur_v, q, S,
                               workspace=ws, error_flag=err, reuse=first)
    plain = tw.ops.attend_union(slab, 0, L, union_pos, union_count, cur_k, cur_v, q, S,
                                workspace=ws, error_flag=err)
    torch.cuda.synchronize()
    assert torch.equal(out0, plain)
    np.testing.assert_array_equal(counts.cpu().numpy()[:, 1], [len(c) for c in cur])
    assert int(counts[:, 0].sum()) == 0
    for gi, c in enumerate(cur):
        assert torch.equal(next_k[gi, : len(c)].cpu(), keys[gi, c.long()])
    slab.close()


@pytest.mark.parametrize("dtype", DTYPES)
def test_gather_union_reads_previous_rows(tw, cuda, dtype):
    """The staged gather keeps its own packed output as the next step's rows."""
    import ctypes

    G, L, max_len = 4, 2500, 2600
    slab, keys, vals, g = _slab(tw, G, max_len, dtype, 5)
    prev_length = L - 1
    prev, cur = _unions(g, L, [0, 30, 700, 1200], [3, 50, 900, 1000], prev_length)
    union_pos, union_count = _pad(cur, L, cuda)
    rows_cap = max(sum(len(p) for p in prev), sum(len(c) for c in cur)) + G + 16
    prev_k = torch.zeros((rows_cap, 128), dtype=dtype)
    prev_v = torch.zeros_like(prev_k)
    poff = np.cumsum([0] + [len(p) + 1 for p in prev])
    for gi, p in enumerate(prev):
        o = poff[gi]
        prev_k[o: o + len(p)] = (keys[gi, p].float() * 2).to(dtype)
        prev_v[o: o + len(p)] = (vals[gi, p].float() * 2).to(dtype)
        prev_k[o + len(p)] = torch.randn(128, generator=g).to(dtype)
        prev_v[o + len(p)] = torch.randn(128, generator=g).to(dtype)
    prev_k, prev_v = prev_k.to(cuda), prev_v.to(cuda)
    row_map = torch.zeros((G, max_len), dtype=torch.int64, device=cuda)
    _plant_map(row_map, prev, prev_length, 3, lambda gi, j: int(poff[gi]) + j)
    cur_k = torch.randn(G, 128, generator=g).to(dtype).to(cuda)
    cur_v = torch.randn(G, 128, generator=g).to(dtype).to(cuda)
    out_k = torch.empty(rows_cap, 128, dtype=dtype, device=cuda)
    out_v = torch.empty_like(out_k)
    cu = torch.zeros(G + 1, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    counts = torch.zeros((G, 2), dtype=torch.int32, device=cuda)
    r = tw.ops.row_reuse(row_map, 4, prev_tag=3, prev_k=prev_k, prev_v=prev_v, row_counts=counts)
    lib = tw.load_library()

    def gather(reuse):
        return lib.tw_gather_union(
            slab.key_device_ptr, slab.value_device_ptr, None, 0, max_len, 0, G, L,
            union_pos.data_ptr(), L, union_count.data_ptr(), cur_k.data_ptr(), cur_v.data_ptr(), 128,
            DTYPE_CODE[dtype], out_k.data_ptr(), out_v.data_ptr(), rows_cap, cu.data_ptr(),
            err.data_ptr(), ctypes.byref(reuse) if reuse is not None else None,
            torch.cuda.current_stream().cuda_stream)

    tw._lib.check(gather(r), "gather_union")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    m = row_map.cpu()
    row = 0
    for gi, c in enumerate(cur):
        for pos in c.tolist():
            j = _expected_source(prev, gi, pos, prev_length)
            src_k = prev_k[poff[gi] + j].cpu() if j >= 0 else keys[gi, pos]
            assert torch.equal(out_k[row].cpu(), src_k), (gi, pos)
            assert int(m[gi, pos]) == (4 << 32) | row
            row += 1
        assert torch.equal(out_k[row].cpu(), cur_k[gi].cpu())
        assert int(m[gi, L]) == (4 << 32) | row
        row += 1
    assert int(cu[-1]) == row
    want = reuse_oracle.group_hit_miss(prev, cur, prev_length)
    np.testing.assert_array_equal(counts.cpu().numpy(), want)
    # the oracle mapping (attention layout + previous token) gives the same sources
    hs, hd, _, _, _ = reuse_oracle.resident_map(prev, cur, list(range(G)), max_len,
                                                attention_layout=True, previous_length=prev_length)
    for s_, d_ in zip(hs.tolist(), hd.tolist()):
        assert torch.equal(out_k[d_].cpu(), prev_k[s_].cpu())
    # host-side checks: no next rows here, previous rows may not alias the output, tags differ
    bad = tw.ops.row_reuse(row_map, 5, next_k=out_k.view(1, rows_cap, 128),
                           next_v=out_v.view(1, rows_cap, 128))
    assert gather(bad) == tw._lib.TW_ERR_BAD_ARG
    alias = tw.ops.row_reuse(row_map, 5, prev_tag=4, prev_k=out_k, prev_v=prev_v)
    assert gather(alias) == tw._lib.TW_ERR_BAD_ARG
    same = tw.ops.row_reuse(row_map, 4, prev_tag=4, prev_k=prev_k, prev_v=prev_v)
    assert gather(same) == tw._lib.TW_ERR_BAD_ARG
    slab.close()


def test_attend_union_reuse_argument_checks(tw, cuda):
    """Aliased rows, a zero or repeated tag, a short row map or narrow next
    rows are rejected before any launch."""
    G, L, max_len, S = 2, 256, 300, 64
    slab, _, _, g = _slab(tw, G, max_len, torch.float16, 3)
    union_pos = torch.zeros((G, L), dtype=torch.int32, device=cuda)
    union_count = torch.zeros(G, dtype=torch.int32, device=cuda)
    cur = torch.zeros((G, 128), dtype=torch.float16, device=cuda)
    q = torch.zeros((G, 4, 128), dtype=torch.float16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    ws = torch.zeros(tw.ops.decode_attention_workspace_bytes(G, 4, S), dtype=torch.uint8, device=cuda)
    rows = torch.zeros((2, G, S, 128), dtype=torch.float16, device=cuda)
    other = torch.zeros_like(rows)
    row_map = torch.zeros((G, max_len), dtype=torch.int64, device=cuda)
    cases = [
        dict(row_map=row_map, next_tag=2, next_k=rows[0], next_v=rows[1], prev_tag=1,
             prev_k=rows[0], prev_v=other[1]),                                    # prev overlaps next
        dict(row_map=row_map, next_tag=0, next_k=rows[0], next_v=rows[1]),        # zero tag
        dict(row_map=row_map, next_tag=3, next_k=rows[0], next_v=rows[1], prev_tag=3,
             prev_k=other[0], prev_v=other[1]),                                   # repeated tag
        dict(row_map=row_map[:, :L], next_tag=2, next_k=rows[0], next_v=rows[1]),  # map too short
        dict(row_map=row_map, next_tag=2, next_k=rows[0, :, :8], next_v=rows[1, :, :8]),  # narrow
    ]
    for kw in cases:
        with pytest.raises(ValueError):
            mk = kw.pop("row_map")
            tag = kw.pop("next_tag")
            r = tw.ops.row_reuse(mk.contiguous(), tag, **{k: (v.contiguous() if torch.is_tensor(v) else v)
                                                        for k, v in kw.items()})
            tw.ops.attend_union(slab, 0, L, union_pos, union_count, cur, cur, q, S, workspace=ws,
                                error_flag=err, reuse=r)
    slab.close()


def _make(tw, dev, *, layers, G, R, L, dtype, **kw):
    return tw.TwilightMatchedBudgetOffloadedCache(
        num_cache_entries=layers * G, max_cache_len=L + 16, head_dim=128,
        num_query_heads_per_kv=R, dtype=dtype, device=dev, sink_tokens=64, recent_tokens=256,
        block_size=16, candidate_token_budget=512, top_p=0.9, budget_mode="dynamic",
        layer_batched_selection=True, gqa_groupwise_execution=True, qk_backend="cuda",
        int4_group_size=32, **kw)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_resident_cache_matches_direct(tw, cuda, dtype):
    """Staged steps (update_layer_gqa_group_ragged), then fused one-call steps
    (decode_layer), then prepare + attend_layer: the resident cache's outputs
    equal the direct cache's bit for bit; its trace has one row per layer-step,
    no hits on a layer's first step, hits afterwards (also across the switches
    between the staged and fused paths), and hit rows equal the oracle's count
    over the direct cache's unions."""
    layers, G, R, L = 2, 2, 4, 2048
    tdt = synth.TORCH_DTYPES[dtype]
    data = [synth.make_layer(groups=G, heads_per_group=R, length=L, dtype=dtype, seed=60 + i,
                             workload="outliers") for i in range(layers)]
    direct = _make(tw, cuda, layers=layers, G=G, R=R, L=L, dtype=tdt)
    resident = _make(tw, cuda, layers=layers, G=G, R=R, L=L, dtype=tdt,
                     previous_token_resident_cache=True, resident_zero_copy=True,
                     resident_mapping_backend="gpu_bitmap", resident_hit_copy_backend="triton")
    for c in (direct, resident):
        for li, d in enumerate(data):
            for g in range(G):
                c.update(d.keys[g].view(1, 1, L, 128).to(cuda), d.values[g].view(1, 1, L, 128).to(cuda),
                         li * G + g)
    gen = torch.Generator().manual_seed(99)
    base_q = torch.randn(layers, G, R, 128, generator=gen)
    modes = ["staged", "staged", "fused", "fused", "fused", "two_call", "two_call"]
    prev_union = {}
    expected = []  # (hits, history) per layer-step
    for step, mode in enumerate(modes):
        for li in range(layers):
            entries = [li * G + g for g in range(G)]
            q = (base_q[li] + 0.05 * torch.randn(G, R, 128, generator=gen)).to(tdt).to(cuda)
            kn = torch.randn(G, 128, generator=gen).to(tdt).to(cuda)
            vn = torch.randn(G, 128, generator=gen).to(tdt).to(cuda)
            qs = [q[g].view(1, R, 1, 128) for g in range(G)]
            ks = [kn[g].view(1, 1, 1, 128) for g in range(G)]
            vs = [vn[g].view(1, 1, 1, 128) for g in range(G)]
            old = L + step
            outs = []
            for c in (direct, resident):
                if mode == "staged":
                    c.prepare_layer_selection(entries=entries, queries=qs)
                    outs.append(c.update_layer_gqa_group_ragged(key_states=ks, value_states=vs,
                                                                queries=qs, entries=entries))
                elif mode == "fused":
                    outs.append((c.decode_layer(queries=q, key_states=kn, value_states=vn,
                                                entries=entries),))
                else:
                    c.prepare_layer_selection(entries=entries, queries=qs)
                    outs.append((c.attend_layer(key_states=ks, value_states=vs, queries=qs,
                                                entries=entries),))
                torch.cuda.synchronize()
            for a, b in zip(outs[0][:3], outs[1][:3]):
                assert torch.equal(a, b), (step, li, mode)
            assert outs[0][3:] == outs[1][3:]
            bufs = direct._layer_bufs[G]
            union = [bufs["union_pos"][g, : int(bufs["union_count"][g])].long().cpu() for g in range(G)]
            prev = prev_union.get(li)
            hits = 0 if prev is None else int(
                reuse_oracle.group_hit_miss(prev, union, old - 1)[:, 0].sum())
            expected.append((hits, sum(len(u) for u in union)))
            prev_union[li] = union
    trace = resident.resident_reuse_trace()
    assert len(trace) == len(modes) * layers
    for row, (hits, history) in zip(trace, expected):
        assert row["hit_rows"] == hits, row
        assert row["history_rows"] == history
        assert row["hit_rows"] + row["miss_rows"] == row["history_rows"]
    assert trace[0]["hit_rows"] == 0 and trace[layers]["hit_rows"] > 0
    assert all(row["hit_rows"] > 0 for row in trace[layers:])
    snap = resident.state_snapshot()
    assert snap["previous_token_resident_cache"] and snap["resident_cache_allocated_bytes"] > 0
    for c in (direct, resident):
        c.synchronize()
        c.close()
