"""GPU contract of tw_gather_quest_heads, the per-query-head Quest packing
(hi/quest_offload_cache.py:403-511, :724-987): segment s = g*R + r holds the
sink rows, the rows of head r's pages in the order given, the recent window
and the current token.  The kernel reads each distinct row of a group once
and writes it to every segment holding it, so the cases repeat pages across
heads and within a head, give them unsorted, run past the sharing limit
(R * k > 1024 page slots per group), and read from device memory and from the
mapped host slab.  Expected rows come from plain torch indexing."""

from __future__ import annotations

import ctypes

import pytest
import torch

from pipeline import DTYPE_CODE

pytestmark = pytest.mark.gpu


def _expected(rows, first, G, R, sink_end, recent_start, old_length, sink, block, pages, cur):
    """rows [E, max_len, D] host copy; pages [G*R, k] int64 -> [G*R*seg, D]."""
    out = []
    for g in range(G):
        src = rows[first + g]
        for r in range(R):
            s = g * R + r
            pos = [torch.arange(sink_end)]
            for p in pages[s].tolist():
                pos.append(sink + p * block + torch.arange(block))
            pos.append(torch.arange(recent_start, old_length))
            out.append(src.index_select(0, torch.cat(pos)))
            out.append(cur[g:g + 1])
    return torch.cat(out)


def _gather(tw, slab_k, slab_v, n_entries, max_len, first, G, R, old_length, sink_end,
            recent_start, sink, block, pages, k_pages, cur_k, cur_v, dtype, err, cuda):
    seg = sink_end + k_pages * block + (old_length - recent_start) + 1
    out_k = torch.full((G * R * seg, 128), 7.0, dtype=dtype, device=cuda)
    out_v = torch.full_like(out_k, 7.0)
    st = tw._lib.load().tw_gather_quest_heads(
        slab_k, slab_v, None, n_entries, max_len, first, G, R, old_length, sink_end,
        recent_start, sink, block, None if pages is None else pages.data_ptr(), k_pages,
        cur_k.data_ptr(), cur_v.data_ptr(), 128, DTYPE_CODE[dtype], out_k.data_ptr(),
        out_v.data_ptr(), err.data_ptr(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    tw._lib.check(st, "gather_quest_heads")
    torch.cuda.synchronize()
    return out_k.cpu(), out_v.cpu()


@pytest.mark.parametrize("source", ["device", "mapped"])
@pytest.mark.parametrize("G,R,k_pages,block,sink,recent", [
    (3, 4, 64, 16, 64, 256),    # cfg1-like: shared protected rows, overlapping pages
    (2, 8, 200, 16, 64, 256),   # 1600 page slots: past the sharing limit
    (2, 1, 5, 32, 0, 1),        # no sink, only the current token after the pages
    (1, 3, 0, 16, 16, 40),      # no pages
    (2, 2, 7, 16, 13, 300),     # sink not a multiple of anything
])
def test_gather_quest_heads_matches_indexing(tw, cuda, source, G, R, k_pages, block, sink, recent):
    dtype = torch.bfloat16
    E, max_len, first = G + 2, 4096 + 64, 1
    old_length = 4096
    sink_end = min(sink, old_length)
    recent_start = max(sink_end, old_length - max(0, recent - 1))
    P = (recent_start - sink_end) // block
    g = torch.Generator().manual_seed(7 + G * 31 + R * 7 + k_pages)
    geom = tw.SlabGeometry(num_entries=E, batch_size=1, max_cache_len=max_len, head_dim=128)
    slab = tw.MappedHostSlab(geom, dtype)
    slab.rows.copy_(torch.randn(2, E, max_len, 128, generator=g).to(dtype))
    host_rows = slab.rows.clone()
    if source == "device":
        dev = host_rows.to(cuda)
        slab_k, slab_v = dev[0].data_ptr(), dev[1].data_ptr()
    else:
        slab_k, slab_v = slab.key_device_ptr, slab.value_device_ptr
    # pages: heads of a group draw from a small pool (many shared pages), each
    # list unsorted, with a repeat inside one head's list
    pages = None
    if k_pages:
        pool = torch.randperm(P, generator=g)[:max(k_pages + 8, P // 2)]
        pages = torch.stack([pool[torch.randperm(len(pool), generator=g)[:k_pages]]
                             for _ in range(G * R)])
        if k_pages > 2:
            pages[0, 1] = pages[0, 0]
        pages_dev = pages.to(torch.int32).to(cuda)
    else:
        pages_dev = None
    cur = torch.randn(2, G, 128, generator=g).to(dtype)
    cur_k, cur_v = cur[0].to(cuda), cur[1].to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for _ in range(2):  # the second call overwrites the same outputs identically
        ok, ov = _gather(tw, slab_k, slab_v, E, max_len, first, G, R, old_length, sink_end,
                         recent_start, sink, block, pages_dev, k_pages, cur_k, cur_v, dtype, err,
                         cuda)
        pg = pages if pages is not None else torch.zeros(G * R, 0, dtype=torch.int64)
        ek = _expected(host_rows[0], first, G, R, sink_end, recent_start, old_length, sink, block,
                       pg, cur[0])
        ev = _expected(host_rows[1], first, G, R, sink_end, recent_start, old_length, sink, block,
                       pg, cur[1])
        assert torch.equal(ok, ek) and torch.equal(ov, ev)
        assert int(err.item()) == 0
    slab.close()


def test_gather_quest_heads_bad_page(tw, cuda):
    """A page id < 0 or past the context: error flag, zeros for its rows, the
    other rows as usual (the same page id in another head included)."""
    dtype = torch.float16
    G, R, k_pages, block, sink = 1, 4, 3, 16, 16
    old_length, max_len = 512, 600
    sink_end, recent_start = sink, old_length - 31
    g = torch.Generator().manual_seed(3)
    rows = torch.randn(2, G, max_len, 128, generator=g).to(dtype)
    dev = rows.to(cuda)
    cur = torch.randn(2, G, 128, generator=g).to(dtype)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    pages = torch.tensor([[1, 2, 3], [-1, 2, 4], [5, 40, 1], [3, 3, 0]], dtype=torch.int32)
    ok, ov = _gather(tw, dev[0].data_ptr(), dev[1].data_ptr(), G, max_len, 0, G, R, old_length,
                     sink_end, recent_start, sink, block, pages.to(cuda), k_pages,
                     cur[0].to(cuda), cur[1].to(cuda), dtype, err, cuda)
    assert int(err.item()) == tw._lib.TW_ERR_INVALID_INDEX
    seg = sink_end + k_pages * block + (old_length - recent_start) + 1
    zero = torch.zeros(block, 128, dtype=dtype)
    for s in range(R):
        for j in range(k_pages):
            p = int(pages[s, j])
            got = ok[s * seg + sink_end + j * block: s * seg + sink_end + (j + 1) * block]
            pos = sink + p * block
            if p < 0 or pos + block > old_length:
                assert torch.equal(got, zero)
            else:
                assert torch.equal(got, rows[0, 0, pos:pos + block])
