"""GPU parity of each sm_100a kernel (called through the C ABI via ops.py).

Integer / index / code outputs must equal oracle/exact.c bit for bit; the
arithmetic order of the fp32 stages (Quest score, INT4 QK) is also restated
there, so those are compared bit for bit too.  Where the reference's own
torch expression runs on CUDA (oracle/torch_ref.py) it pins the CUDA
semantics (INT4 reciprocal division, Quest score order).
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import exact, synth, torch_ref
from pipeline import DTYPE_CODE, bits, twilight_oracle
from tolerance import ATTN_TOL_16BIT, ATTN_TOL_FP32

pytestmark = pytest.mark.gpu

DTYPES = [torch.float16, torch.bfloat16]


def _rand_keys(E, S, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(E, S, 128, generator=g)
    k[..., 5] *= 4.0
    return k.to(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("scale_div", [0, 1])
def test_int4_pack_bitexact(tw, cuda, dtype, group, scale_div):
    E, S, cap = 2, 777, 800
    keys = _rand_keys(E, S, dtype, 1 + group)
    keys[0, 3] = 1.0                       # constant row
    keys[1, 7, :64] = -3.0                 # two-valued row
    keys[1, 7, 64:] = 5.0
    ng = 128 // group
    packed = torch.zeros((E, cap, 64), dtype=torch.uint8, device=cuda)
    scale = torch.zeros((E, cap, ng), dtype=dtype, device=cuda)
    minimum = torch.zeros_like(scale)
    tw.ops.int4_pack(keys.to(cuda), group_size=group, packed=packed, scale=scale, minimum=minimum,
                     out_row_offset=10, scale_div=scale_div)
    torch.cuda.synchronize()
    for e in range(E):
        p, s, m = exact.int4_pack(bits(keys[e]), group, DTYPE_CODE[dtype], scale_div)
        np.testing.assert_array_equal(packed[e, 10:10 + S].cpu().numpy(), p)
        np.testing.assert_array_equal(scale[e, 10:10 + S].cpu().float().numpy(),
                                      torch.from_numpy(s.view(np.int16)).view(dtype).float().numpy())
        np.testing.assert_array_equal(minimum[e, 10:10 + S].cpu().float().numpy(),
                                      torch.from_numpy(m.view(np.int16)).view(dtype).float().numpy())


@pytest.mark.parametrize("dtype", DTYPES)
def test_int4_pack_matches_reference_expression_on_cuda(tw, cuda, dtype):
    """tw_int4_pack (reciprocal mode) == the reference's affine_int4_pack run by torch on CUDA."""
    keys = _rand_keys(1, 4096, dtype, 7)[0].to(cuda)
    p_ref, s_ref, m_ref = torch_ref.affine_int4_pack(keys)
    packed = torch.zeros((1, 4096, 64), dtype=torch.uint8, device=cuda)
    scale = torch.zeros((1, 4096, 1), dtype=dtype, device=cuda)
    minimum = torch.zeros_like(scale)
    tw.ops.int4_pack(keys[None], group_size=128, packed=packed, scale=scale, minimum=minimum)
    torch.cuda.synchronize()
    assert torch.equal(packed[0], p_ref)
    assert torch.equal(scale[0, :, 0].float(), s_ref.float())
    assert torch.equal(minimum[0, :, 0].float(), m_ref.float())


@pytest.mark.parametrize("dtype", DTYPES)
def test_quest_metadata_bitexact(tw, cuda, dtype):
    E, S, sink, block = 3, 64 + 16 * 40 + 5, 64, 16
    keys = _rand_keys(E, S, dtype, 3)
    cap = 50
    pmin = torch.zeros((E, cap, 128), dtype=dtype, device=cuda)
    pmax = torch.zeros_like(pmin)
    n = tw.ops.quest_page_metadata(keys.to(cuda), sink=sink, block_size=block, page_min=pmin,
                                   page_max=pmax)
    torch.cuda.synchronize()
    assert n == 40
    for e in range(E):
        a, b = exact.quest_page_metadata(bits(keys[e]), sink, block, DTYPE_CODE[dtype])
        ta, tb = torch_ref.quest_page_metadata(keys[e], sink, block)
        assert torch.equal(pmin[e, :40].cpu(), ta) and torch.equal(pmax[e, :40].cpu(), tb)
        np.testing.assert_array_equal(bits(pmin[e, :40].cpu()), a)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("R", [1, 3, 4, 8])
def test_quest_score_bitexact(tw, cuda, dtype, R):
    G, P, cap = 4, 1000, 1024
    g = torch.Generator().manual_seed(R)
    a = torch.randn(G, cap, 128, generator=g).to(dtype)
    b = torch.randn(G, cap, 128, generator=g).to(dtype)
    lo, hi = torch.minimum(a, b), torch.maximum(a, b)
    q = torch.randn(G, R, 128, generator=g)
    q[0, 0] = q[0, 0].bfloat16().float()
    q[-1, -1] *= torch.exp2(torch.randint(-12, 12, (128,), generator=g).float())
    scores = tw.ops.quest_score(q.to(cuda), lo.to(cuda), hi.to(cuda), P)
    torch.cuda.synchronize()
    ref = exact.quest_score(q.numpy(), bits(lo[:, :P]), bits(hi[:, :P]), DTYPE_CODE[dtype])
    np.testing.assert_array_equal(scores.cpu().numpy(), ref)
    # the reference's torch expression on CUDA (pinned bit-equal to its fused
    # kernel by the reference's own test under torch 2.7): agreement to fp32 rounding
    tref = torch_ref.quest_scores(q.to(cuda), lo[:, :P].to(cuda), hi[:, :P].to(cuda)).cpu().numpy()
    assert np.max(np.abs(tref - ref)) <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("n,k", [(17, 1), (186, 64), (2028, 256), (2048, 2048), (8188, 256), (16384, 1000)])
def test_topk_pages_bitexact(tw, cuda, n, k):
    g = torch.Generator().manual_seed(n)
    scores = torch.randn(6, n, generator=g)
    scores[1] = torch.round(scores[1] * 4) / 4        # many ties
    scores[2] = 0.0                                   # all tied
    scores[3, : n // 2] = -0.0
    scores[4] = torch.arange(n, dtype=torch.float32)  # distinct ascending
    out = tw.ops.topk_pages(scores.to(cuda), k)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), exact.topk_pages(scores.numpy(), k))
    # set equality with torch.topk wherever the k-th value is not tied
    ref = torch.topk(scores, k, dim=-1).indices.sort(dim=-1).values
    assert torch.equal(out[0].cpu().long(), ref[0]) and torch.equal(out[4].cpu().long(), ref[4])


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("group", [32, 128])
@pytest.mark.parametrize("R,block", [(4, 16), (3, 1), (8, 16)])
def test_int4_qk_bitexact(tw, cuda, dtype, group, R, block):
    G, S, sink = 2, 1200, 64
    keys = _rand_keys(G, S, dtype, 11)
    ng = 128 // group
    packed = torch.zeros((G, S, 64), dtype=torch.uint8, device=cuda)
    scale = torch.zeros((G, S, ng), dtype=dtype, device=cuda)
    minimum = torch.zeros_like(scale)
    tw.ops.int4_pack(keys.to(cuda), group_size=group, packed=packed, scale=scale, minimum=minimum)
    P = (S - sink - 255) // block
    b0 = min(P, 512 // block)
    g = torch.Generator().manual_seed(5)
    pages = torch.stack([torch.stack([torch.randperm(P, generator=g)[:b0].sort().values
                                      for _ in range(R)]) for _ in range(G)]).int()
    q = torch.randn(G, R, 128, generator=g)
    logits = tw.ops.int4_qk(q.to(cuda), packed, scale, minimum, pages.to(cuda), block_size=block,
                            sink=sink)
    torch.cuda.synchronize()
    ref = exact.int4_qk(q.numpy(), packed.cpu().numpy(), bits(scale.cpu()), bits(minimum.cpu()),
                        pages.numpy(), block, sink, group, DTYPE_CODE[dtype])
    np.testing.assert_array_equal(logits.cpu().numpy(), ref)


CASES_TOP_P = ["random", "ties", "peaked", "p_one", "tiny", "large_radix", "large_ties"]


@pytest.mark.parametrize("case", CASES_TOP_P)
def test_top_p_union_bitexact(tw, cuda, case):
    """Both top-p paths: the bitonic-sort path (<= 8192 candidates per row) and
    the radix path (the two large_* cases, 10240 candidates)."""
    G, R, block, sink, top_p = 3, 4, 16, 64, 0.95
    b0 = 64
    L = 64 + 16 * 300 + 255
    g = torch.Generator().manual_seed(CASES_TOP_P.index(case))
    if case == "tiny":
        R, block, sink, b0, L, top_p = 3, 1, 1, 8, 16, 0.85
    elif case.startswith("large"):
        b0, L = 640, 64 + 16 * 700 + 255
    n = b0 * block
    P = (max(sink, L - 255 if case != "tiny" else L - 1) - sink) // block
    pages = torch.stack([torch.stack([torch.randperm(P, generator=g)[:b0].sort().values
                                      for _ in range(R)]) for _ in range(G)]).int()
    logits = torch.randn(G, R, n, generator=g)
    if case in ("ties", "large_ties"):
        logits = torch.round(logits * 2) / 2
    elif case == "peaked":
        logits = logits * 10
    elif case == "p_one":
        top_p = 1.0
    recent = 256 if case != "tiny" else 2
    sink_end = min(sink, L)
    recent_start = max(sink_end, L - (recent - 1))
    union_pos = torch.full((G, L), -7, dtype=torch.int32, device=cuda)
    union_count = torch.zeros(G, dtype=torch.int32, device=cuda)
    head_count = torch.zeros((G, R), dtype=torch.int32, device=cuda)
    head_pos = torch.full((G, R, n), -7, dtype=torch.int32, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    tw.ops.top_p_union(logits.to(cuda), pages.to(cuda), block_size=block, sink=sink, top_p=top_p,
                       old_length=L, sink_end=sink_end, recent_start=recent_start,
                       union_pos=union_pos, union_count=union_count, head_count=head_count,
                       head_pos=head_pos, error_flag=err)
    torch.cuda.synchronize()
    unions, hc, hp, bad = exact.top_p_union(logits.numpy(), pages.numpy(), block, sink, top_p, L,
                                            sink_end, recent_start)
    assert int(err.item()) == 0 and bad == 0
    np.testing.assert_array_equal(head_count.cpu().numpy(), hc)
    for gi in range(G):
        np.testing.assert_array_equal(union_pos[gi, : int(union_count[gi])].cpu().numpy(), unions[gi])
        for r in range(R):
            np.testing.assert_array_equal(head_pos[gi, r, : hc[gi, r]].cpu().numpy(), hp[gi][r])


@pytest.mark.parametrize("name,cfg", [
    ("twilight_outliers", dict(groups=2, heads=4, length=2048, dtype="float16", seed=11,
                               workload="outliers", sink=64, recent=256, block=16, b0_tokens=512,
                               top_p=0.95, n_needles=0)),
    ("twilight_needles", dict(groups=2, heads=4, length=1536, dtype="bfloat16", seed=12,
                              workload="needles", sink=64, recent=256, block=16, b0_tokens=256,
                              top_p=0.9, n_needles=8)),
])
def test_select_layer_matches_reference_golden(tw, cuda, name, cfg):
    """Whole-layer selection on the GPU (INT4 packed in the CPU rounding mode the
    golden run used) reproduces the reference's unions and per-head counts."""
    from pathlib import Path
    golden = np.load(Path(__file__).resolve().parent / "golden" / f"{name}.npz")
    layer = synth.make_layer(groups=cfg["groups"], heads_per_group=cfg["heads"], length=cfg["length"],
                             dtype=cfg["dtype"], seed=cfg["seed"], workload=cfg["workload"],
                             sink=cfg["sink"], recent=cfg["recent"], block=cfg["block"],
                             n_needles=cfg["n_needles"])
    G, R, L = cfg["groups"], cfg["heads"], cfg["length"]
    dt = layer.keys.dtype
    keys = layer.keys.to(cuda)
    cap = (L - cfg["sink"]) // cfg["block"] + 1
    pmin = torch.zeros((G, cap, 128), dtype=dt, device=cuda)
    pmax = torch.zeros_like(pmin)
    P_built = tw.ops.quest_page_metadata(keys, sink=cfg["sink"], block_size=cfg["block"],
                                         page_min=pmin, page_max=pmax)
    packed = torch.zeros((G, L, 64), dtype=torch.uint8, device=cuda)
    scale = torch.zeros((G, L, 1), dtype=dt, device=cuda)
    minimum = torch.zeros_like(scale)
    tw.ops.int4_pack(keys, group_size=128, packed=packed, scale=scale, minimum=minimum,
                     scale_div=tw.ops.SCALE_DIVIDE)
    w = torch_ref.window(L, sink=cfg["sink"], recent=cfg["recent"], block=cfg["block"],
                         candidate_token_budget=cfg["b0_tokens"], metadata_pages=P_built)
    q = layer.queries.float().to(cuda)
    scores = tw.ops.quest_score(q, pmin, pmax, w.candidate_pages)
    pages = tw.ops.topk_pages(scores, w.b0_pages)
    logits = tw.ops.int4_qk(q, packed, scale, minimum, pages, block_size=cfg["block"], sink=cfg["sink"])
    union_pos = torch.zeros((G, L), dtype=torch.int32, device=cuda)
    union_count = torch.zeros(G, dtype=torch.int32, device=cuda)
    head_count = torch.zeros((G, R), dtype=torch.int32, device=cuda)
    tw.ops.top_p_union(logits, pages, block_size=cfg["block"], sink=cfg["sink"], top_p=cfg["top_p"],
                       old_length=L, sink_end=w.sink_end, recent_start=w.recent_start,
                       union_pos=union_pos, union_count=union_count, head_count=head_count)
    # the same layer through tw_select_layer (the fused one-launch selection)
    f_pos = torch.zeros_like(union_pos)
    f_cnt = torch.zeros_like(union_count)
    f_hc = torch.zeros_like(head_count)
    f_pages = tw.ops.select_layer(q, pmin, pmax, w.candidate_pages, packed, scale, minimum,
                                  b0_pages=w.b0_pages, block_size=cfg["block"], sink=cfg["sink"],
                                  top_p=cfg["top_p"], old_length=L, sink_end=w.sink_end,
                                  recent_start=w.recent_start, union_pos=f_pos, union_count=f_cnt,
                                  head_count=f_hc)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(head_count.cpu().numpy(), golden["desired"])
    np.testing.assert_array_equal(f_hc.cpu().numpy(), golden["desired"])
    assert torch.equal(f_pages, pages)
    for gi in range(G):
        n = int(union_count[gi])
        np.testing.assert_array_equal(union_pos[gi, :n].cpu().numpy(),
                                      golden["unions"][gi][: golden["union_counts"][gi]])
        assert int(f_cnt[gi]) == n
        assert torch.equal(f_pos[gi, :n], union_pos[gi, :n])


def test_gather_kv_contract(tw, cuda):
    """hi/cpu_kv_gather.cpp contract on the GPU, from device and from mapped host memory."""
    g = torch.Generator().manual_seed(123)
    k = torch.randn(10000, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(10000, 128, generator=g).to(torch.bfloat16)
    geom = tw.SlabGeometry(num_entries=1, batch_size=1, max_cache_len=10000, head_dim=128)
    slab = tw.MappedHostSlab(geom, torch.bfloat16)
    slab.entry("key", 0)[0, 0].copy_(k)
    slab.entry("value", 0)[0, 0].copy_(v)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for source in ("device", "mapped"):
        for n in (0, 1, 8192):
            rows = torch.randint(10000, (n,), generator=g)
            a = torch.zeros(n, 128, dtype=k.dtype, device=cuda)
            b = torch.zeros_like(a)
            src_k = k.to(cuda) if source == "device" else (slab.entry("key", 0)[0, 0], slab.key_device_ptr)
            src_v = v.to(cuda) if source == "device" else (slab.entry("value", 0)[0, 0], slab.value_device_ptr)
            tw.ops.gather_kv(src_k, src_v, rows.to(cuda), a, b, err)
            torch.cuda.synchronize()
            assert torch.equal(a.cpu(), k[rows]) and torch.equal(b.cpu(), v[rows])
            assert int(err.item()) == 0
    for bad in (-1, 10000):
        out = torch.full((2, 128), 7.0, dtype=k.dtype, device=cuda)
        rows = torch.tensor([bad, 3], device=cuda)
        tw.ops.gather_kv(k.to(cuda), v.to(cuda), rows, out, out.clone(), err)
        torch.cuda.synchronize()
        assert int(err.item()) == tw._lib.TW_ERR_INVALID_INDEX
        assert torch.equal(out[0].cpu(), torch.full((128,), 7.0, dtype=k.dtype))  # skipped
        assert torch.equal(out[1].cpu(), k[3])
        err.zero_()
    slab.close()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("S,R,lengths", [
    (8, 4, [1, 2, 129, 300, 4400, 1, 4096, 257]),
    (4, 8, [1000, 1, 128, 8193]),
    (32, 1, [1300] * 32),
    (3, 3, [17, 0, 5]),
])
def test_decode_attention(tw, cuda, dtype, S, R, lengths):
    g = torch.Generator().manual_seed(S * 100 + R)
    total = sum(lengths)
    q = (torch.randn(S, R, 128, generator=g) * 2).to(dtype)
    k = torch.randn(total, 128, generator=g).to(dtype)
    v = torch.randn(total, 128, generator=g).to(dtype)
    cu = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32)
    max_len = max(lengths)
    ws = torch.zeros(tw.ops.decode_attention_workspace_bytes(S, R, max_len), dtype=torch.uint8, device=cuda)
    lse = torch.zeros(S, R, device=cuda)
    out32 = tw.ops.decode_attention(q.to(cuda), k.to(cuda), v.to(cuda), cu.to(cuda), max_len,
                                    workspace=ws, out_dtype=torch.float32, lse=lse)
    out16 = tw.ops.decode_attention(q.to(cuda), k.to(cuda), v.to(cuda), cu.to(cuda), max_len,
                                    workspace=ws)
    torch.cuda.synchronize()
    for s in range(S):
        a, b = int(cu[s]), int(cu[s + 1])
        if b == a:
            assert torch.all(out32[s].cpu() == 0)
            continue
        ref = torch_ref.decode_attention(q[s], k[a:b], v[a:b])
        np.testing.assert_allclose(out32[s].cpu().double().numpy(), ref.numpy(), atol=ATTN_TOL_FP32, rtol=0)
        np.testing.assert_allclose(out16[s].cpu().double().numpy(), ref.numpy(), atol=ATTN_TOL_16BIT, rtol=0)
        sc = (q[s].double() @ k[a:b].double().T) / math.sqrt(128)
        np.testing.assert_allclose(lse[s].cpu().double().numpy(), torch.logsumexp(sc, -1).numpy(),
                                   atol=1e-3, rtol=0)
    # the workspace counters are left at zero for the next call
    assert int(ws[:4 * S].view(torch.int32).abs().sum().item()) == 0


@pytest.mark.parametrize("dtype", DTYPES)
def test_append_token_running_metadata(tw, cuda, dtype):
    """Appending rows one by one gives the slab rows, the bulk page min/max and
    the INT4 codes of those rows."""
    E, max_len, sink, block, G = 2, 160, 4, 16, 2
    keys = _rand_keys(E, max_len, dtype, 9)
    vals = _rand_keys(E, max_len, dtype, 10)
    geom = tw.SlabGeometry(num_entries=E, batch_size=1, max_cache_len=max_len, head_dim=128)
    slab = tw.MappedHostSlab(geom, dtype)
    cap = math.ceil((max_len - sink) / block)
    pmin = torch.zeros((E, cap, 128), dtype=dtype, device=cuda)
    pmax = torch.zeros_like(pmin)
    packed = torch.zeros((E, max_len, 64), dtype=torch.uint8, device=cuda)
    scale = torch.zeros((E, max_len, 4), dtype=dtype, device=cuda)
    minimum = torch.zeros_like(scale)
    lib = tw.load_library()
    kd, vd = keys.to(cuda), vals.to(cuda)
    for pos in range(max_len):
        kn = kd[:, pos].contiguous()
        vn = vd[:, pos].contiguous()
        tw._lib.check(lib.tw_append_token(
            slab.key_device_ptr, slab.value_device_ptr, None, 0, max_len, 0, G, pos, kn.data_ptr(),
            vn.data_ptr(), 128, DTYPE_CODE[dtype], sink, block, pmin.data_ptr(), pmax.data_ptr(),
            cap * 128, packed.data_ptr(), scale.data_ptr(), minimum.data_ptr(), 32,
            torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert torch.equal(slab.rows[0, :, :], keys) and torch.equal(slab.rows[1, :, :], vals)
    full = (max_len - sink) // block
    for e in range(E):
        a, b = exact.quest_page_metadata(bits(keys[e]), sink, block, DTYPE_CODE[dtype])
        np.testing.assert_array_equal(bits(pmin[e, :full].cpu()), a)
        np.testing.assert_array_equal(bits(pmax[e, :full].cpu()), b)
        p, s, m = exact.int4_pack(bits(keys[e]), 32, DTYPE_CODE[dtype], 0)
        np.testing.assert_array_equal(packed[e].cpu().numpy(), p)
        np.testing.assert_array_equal(bits(scale[e].cpu()), s)
    slab.close()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("R", [1, 4, 8])
def test_attend_union_matches_gather_then_attention(tw, cuda, dtype, R):
    """The fused kernel (rows read in place from the mapped slab) equals the staged
    path (tw_gather_union, then tw_decode_attention) bit for bit, and the float64
    attention of the oracle within the stated tolerance."""
    G, L, max_len = 3, 3000, 3100
    g = torch.Generator().manual_seed(R)
    keys = torch.randn(G, max_len, 128, generator=g).to(dtype)
    vals = torch.randn(G, max_len, 128, generator=g).to(dtype)
    geom = tw.SlabGeometry(num_entries=G, batch_size=1, max_cache_len=max_len, head_dim=128)
    slab = tw.MappedHostSlab(geom, dtype)
    slab.rows[0].copy_(keys)
    slab.rows[1].copy_(vals)
    counts = [0, 1, 2500]
    union_pos = torch.zeros((G, L), dtype=torch.int32)
    for gi, c in enumerate(counts):
        union_pos[gi, :c] = torch.randperm(L, generator=g)[:c].sort().values.int()
    union_pos, union_count = union_pos.to(cuda), torch.tensor(counts, dtype=torch.int32, device=cuda)
    cur_k = torch.randn(G, 128, generator=g).to(dtype).to(cuda)
    cur_v = torch.randn(G, 128, generator=g).to(dtype).to(cuda)
    q = (torch.randn(G, R, 128, generator=g) * 2).to(dtype).to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    rows_cap = sum(counts) + G
    flat_k = torch.empty(rows_cap, 128, dtype=dtype, device=cuda)
    flat_v = torch.empty_like(flat_k)
    cu = torch.zeros(G + 1, dtype=torch.int32, device=cuda)
    lib = tw.load_library()
    tw._lib.check(lib.tw_gather_union(
        slab.key_device_ptr, slab.value_device_ptr, None, 0, max_len, 0, G, L, union_pos.data_ptr(), L,
        union_count.data_ptr(), cur_k.data_ptr(), cur_v.data_ptr(), 128, DTYPE_CODE[dtype],
        flat_k.data_ptr(), flat_v.data_ptr(), rows_cap, cu.data_ptr(), err.data_ptr(), None,
        torch.cuda.current_stream().cuda_stream))
    max_rows = max(counts) + 1
    ws = torch.zeros(tw.ops.decode_attention_workspace_bytes(G, R, max_rows), dtype=torch.uint8, device=cuda)
    for out_dtype in (torch.float32, dtype):
        staged = tw.ops.decode_attention(q, flat_k, flat_v, cu, max_rows, workspace=ws, out_dtype=out_dtype)
        fused = tw.ops.attend_union(slab, 0, L, union_pos, union_count, cur_k, cur_v, q, max_rows,
                                    workspace=ws, error_flag=err, out_dtype=out_dtype)
        torch.cuda.synchronize()
        assert torch.equal(staged, fused)
        tol = ATTN_TOL_FP32 if out_dtype == torch.float32 else ATTN_TOL_16BIT
        for gi, c in enumerate(counts):
            pos = union_pos[gi, :c].long().cpu()
            kk = torch.cat((keys[gi].index_select(0, pos), cur_k[gi:gi + 1].cpu()))
            vv = torch.cat((vals[gi].index_select(0, pos), cur_v[gi:gi + 1].cpu()))
            ref = torch_ref.decode_attention(q[gi].cpu(), kk, vv)
            assert (fused[gi].cpu().double() - ref).abs().max().item() <= tol
    assert int(err.item()) == 0
    # a position outside [0, old_length) is skipped and flagged
    union_pos[2, 5] = L + 7
    tw.ops.attend_union(slab, 0, L, union_pos, union_count, cur_k, cur_v, q, max_rows, workspace=ws,
                        error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == tw._lib.TW_ERR_INVALID_INDEX
    slab.close()


@pytest.mark.parametrize("R,L,budget", [(1, 3007, 768), (2, 3014, 768), (3, 3021, 768),
                                         (4, 3028, 768), (5, 3035, 768), (6, 3042, 768),
                                         (7, 3049, 768), (8, 3056, 768), (8, 131072, 4096)])
@pytest.mark.parametrize("dtype,group", [("float16", 32), ("bfloat16", 128), ("bfloat16", 64)])
def test_select_layer_fused_equals_stages(tw, cuda, R, L, budget, dtype, group):
    """tw_select_layer (one launch: a thread-block cluster per query-head row,
    the GQA union merged by the group's last row cluster) gives the per-stage
    kernels' pages, per-head counts and positions and the union, bit for bit,
    for every R <= 8; 131072 tokens with B0 4096 is the long-context
    head-sharded shape."""
    G, sink, recent, block = 3 if L < 100000 else 2, 64, 256, 16
    layer = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype=dtype, seed=70 + R,
                             workload="needles" if R % 2 else "outliers", sink=sink,
                             recent=recent, block=block, n_needles=6)
    dt = layer.keys.dtype
    keys = layer.keys.to(cuda)
    cap = (L + 64 - sink) // block + 1
    pmin = torch.zeros((G, cap, 128), dtype=dt, device=cuda)
    pmax = torch.zeros_like(pmin)
    P_built = tw.ops.quest_page_metadata(keys, sink=sink, block_size=block, page_min=pmin,
                                         page_max=pmax)
    packed = torch.zeros((G, L + 64, 64), dtype=torch.uint8, device=cuda)
    scale = torch.zeros((G, L + 64, 128 // group), dtype=dt, device=cuda)
    minimum = torch.zeros_like(scale)
    tw.ops.int4_pack(keys, group_size=group, packed=packed, scale=scale, minimum=minimum)
    w = torch_ref.window(L, sink=sink, recent=recent, block=block, candidate_token_budget=budget,
                         metadata_pages=P_built)
    q = layer.queries.float().to(cuda)
    n = w.b0_pages * block
    outs = []
    for fused in (False, True):
        upos = torch.full((G, L + 64), -1, dtype=torch.int32, device=cuda)
        ucnt = torch.zeros(G, dtype=torch.int32, device=cuda)
        hc = torch.zeros((G, R), dtype=torch.int32, device=cuda)
        hp = torch.full((G, R, n), -1, dtype=torch.int32, device=cuda)
        if fused:
            pg = tw.ops.select_layer(q, pmin, pmax, w.candidate_pages, packed, scale, minimum,
                                     b0_pages=w.b0_pages, block_size=block, sink=sink, top_p=0.9,
                                     old_length=L, sink_end=w.sink_end, recent_start=w.recent_start,
                                     union_pos=upos, union_count=ucnt, head_count=hc, head_pos=hp)
        else:
            scores = tw.ops.quest_score(q, pmin, pmax, w.candidate_pages)
            pg = tw.ops.topk_pages(scores, w.b0_pages)
            logits = tw.ops.int4_qk(q, packed, scale, minimum, pg, block_size=block, sink=sink)
            tw.ops.top_p_union(logits, pg, block_size=block, sink=sink, top_p=0.9, old_length=L,
                               sink_end=w.sink_end, recent_start=w.recent_start, union_pos=upos,
                               union_count=ucnt, head_count=hc, head_pos=hp)
        torch.cuda.synchronize()
        outs.append((pg, upos, ucnt, hc, hp))
    (pg0, up0, uc0, hc0, hp0), (pg1, up1, uc1, hc1, hp1) = outs
    assert torch.equal(pg0, pg1)
    assert torch.equal(uc0, uc1)
    assert torch.equal(hc0, hc1)
    assert torch.equal(up0, up1)
    assert torch.equal(hp0, hp1)


def test_select_layer_reuses_its_workspace(tw, cuda):
    """Consecutive tw_select_layer calls on one zero-filled workspace give the
    same result (the fused selection's union merge state at the workspace's
    end is left zero by every call), also after a call of another layer shape
    (fewer candidate pages) on the same buffer."""
    import ctypes

    G, R, L, sink, recent, block = 4, 4, 8192, 64, 256, 16
    layer = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype="float16", seed=91,
                             workload="outliers")
    keys = layer.keys.to(cuda)
    cap = (L - sink) // block + 1
    pmin = torch.zeros((G, cap, 128), dtype=keys.dtype, device=cuda)
    pmax = torch.zeros_like(pmin)
    P_built = tw.ops.quest_page_metadata(keys, sink=sink, block_size=block, page_min=pmin,
                                         page_max=pmax)
    packed = torch.zeros((G, L, 64), dtype=torch.uint8, device=cuda)
    scale = torch.zeros((G, L, 4), dtype=keys.dtype, device=cuda)
    minimum = torch.zeros_like(scale)
    tw.ops.int4_pack(keys, group_size=32, packed=packed, scale=scale, minimum=minimum)
    q = layer.queries.float().to(cuda)
    lib = tw.load_library()
    w_full = torch_ref.window(L, sink=sink, recent=recent, block=block, candidate_token_budget=1024,
                              metadata_pages=P_built)
    ws_bytes = tw.ops.select_layer_workspace_bytes(G, R, w_full.candidate_pages, w_full.b0_pages, block)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda)

    def run(old_length, budget):
        w = torch_ref.window(old_length, sink=sink, recent=recent, block=block,
                             candidate_token_budget=budget, metadata_pages=P_built)
        pages = torch.zeros((G, R, w.b0_pages), dtype=torch.int32, device=cuda)
        upos = torch.full((G, L), -1, dtype=torch.int32, device=cuda)
        ucnt = torch.zeros(G, dtype=torch.int32, device=cuda)
        hc = torch.zeros((G, R), dtype=torch.int32, device=cuda)
        err = torch.zeros(1, dtype=torch.int32, device=cuda)
        rc = lib.tw_select_layer(
            q.data_ptr(), pmin.data_ptr(), pmax.data_ptr(), cap * 128, w.candidate_pages,
            packed.data_ptr(), scale.data_ptr(), minimum.data_ptr(), L, G, R, w.b0_pages, block,
            sink, 128, 32, 0, ctypes.c_double(0.95), old_length, w.sink_end, w.recent_start,
            pages.data_ptr(), upos.data_ptr(), L, ucnt.data_ptr(), hc.data_ptr(), None,
            err.data_ptr(), ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        return pages.cpu(), upos.cpu(), ucnt.cpu(), hc.cpu()

    first = run(L, 1024)
    for _ in range(2):
        again = run(L, 1024)
        assert all(torch.equal(a, b) for a, b in zip(first, again))
    run(L - 3000, 512)  # another shape on the same buffer
    again = run(L, 1024)
    assert all(torch.equal(a, b) for a, b in zip(first, again))
    tail = ws[-4096:].cpu()
    assert int(tail.count_nonzero()) == 0
