"""Protected-row staging of the one-call layer-step (tw_twilight_decode_layer).

Each group's sink rows and recent window belong to its union whatever the
selection picks, so the selection launch copies them into device memory while
it selects and the attention reads them from there.  Only the place a row is
read from changes: the outputs must equal the unstaged path's bit for bit,
over consecutive steps (each step's append moves the recent window), with the
slab addressed directly or through the entry directory (resident heads).
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from oracle import synth

pytestmark = pytest.mark.gpu

SINK, RECENT, BLOCK = 64, 256, 16


def _cache(tw, dev, *, G, R, L, dtype, staging, **kw):
    return tw.TwilightMatchedBudgetOffloadedCache(
        num_cache_entries=G, max_cache_len=L + 8, head_dim=128, num_query_heads_per_kv=R,
        dtype=dtype, device=dev, sink_tokens=SINK, recent_tokens=RECENT, block_size=BLOCK,
        candidate_token_budget=512, top_p=0.95, budget_mode="dynamic",
        layer_batched_selection=True, gqa_groupwise_execution=True, qk_backend="cuda",
        int4_group_size=32, protected_row_staging=staging, **kw)


def _inputs(G, R, tdt, seed, dev):
    g = torch.Generator().manual_seed(seed)
    return tuple(t.to(tdt).to(dev) for t in (torch.randn(G, R, 128, generator=g),
                                             torch.randn(G, 128, generator=g),
                                             torch.randn(G, 128, generator=g)))


@pytest.mark.parametrize("R,dtype,L,resident", [
    (4, "float16", 4096, ()),
    (8, "bfloat16", 400, ()),       # 5 candidate pages; sink and recent nearly meet
    (2, "float16", 2000, (1, 2)),   # resident heads: rows staged through the entry directory
])
def test_staged_decode_layer_equals_unstaged(tw, cuda, R, dtype, L, resident):
    G = 4
    tdt = synth.TORCH_DTYPES[dtype]
    d = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype=dtype, seed=17,
                         workload="outliers")
    kw = {"resident_entries": list(resident)} if resident else {}
    caches = [_cache(tw, cuda, G=G, R=R, L=L, dtype=tdt, staging=s, **kw) for s in (True, False)]
    for c in caches:
        c.prefill_layer(key_states=d.keys.to(cuda), value_states=d.values.to(cuda),
                        entries=list(range(G)))
    assert caches[0]._layer_bufs.get(G) is None or caches[0]._layer_bufs[G]["stage"] is not None
    for step in range(4):
        q, kn, vn = _inputs(G, R, tdt, 300 + step, cuda)
        outs = [c.decode_layer(queries=q, key_states=kn, value_states=vn, entries=list(range(G)))
                for c in caches]
        torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1]), step
        b0, b1 = caches[0]._layer_bufs[G], caches[1]._layer_bufs[G]
        assert torch.equal(b0["union_count"], b1["union_count"])
        assert b0["stage"] is not None and b1["stage"] is None
    for c in caches:
        c.synchronize()
        c.close()


class _SlabStep:
    """One layer on a directly addressed mapped slab (no entry directory),
    driven through tw_decode_layer_args as a C caller would."""

    def __init__(self, tw, dev, G, R, L, seed):
        self.tw, self.G, self.R, self.L = tw, G, R, L
        self.max_len = L + 8
        d = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype="float16", seed=seed,
                             workload="outliers")
        self.data = d
        geom = tw.SlabGeometry(num_entries=G, batch_size=1, max_cache_len=self.max_len, head_dim=128)
        self.slab = tw.MappedHostSlab(geom, torch.float16)
        self.slab.rows[0, :, :L].copy_(d.keys)
        self.slab.rows[1, :, :L].copy_(d.values)
        self.page_cap = math.ceil((self.max_len - SINK) / BLOCK)
        keys = d.keys.to(dev)
        self.pmin = torch.empty((G, self.page_cap, 128), dtype=torch.float16, device=dev)
        self.pmax = torch.empty_like(self.pmin)
        meta = tw.ops.quest_page_metadata(keys, sink=SINK, block_size=BLOCK, page_min=self.pmin,
                                          page_max=self.pmax)
        self.packed = torch.empty((G, self.max_len, 64), dtype=torch.uint8, device=dev)
        self.scale = torch.empty((G, self.max_len, 4), dtype=torch.float16, device=dev)
        self.minimum = torch.empty_like(self.scale)
        tw.ops.int4_pack(keys, group_size=32, packed=self.packed, scale=self.scale,
                         minimum=self.minimum)
        self.sink_end = min(SINK, L)
        self.recent_start = max(self.sink_end, L - (RECENT - 1))
        self.n_pages = min((self.recent_start - self.sink_end) // BLOCK, meta)
        self.b0 = min(self.n_pages, 512 // BLOCK)
        self.per_group = min(L, SINK + RECENT + R * self.b0 * BLOCK) + 1
        self.pages = torch.empty((G, R, self.b0), dtype=torch.int32, device=dev)
        self.union_pos = torch.empty((G, self.max_len), dtype=torch.int32, device=dev)
        self.union_count = torch.zeros(G, dtype=torch.int32, device=dev)
        self.head_count = torch.zeros((G, R), dtype=torch.int32, device=dev)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)
        ws = tw.ops.select_layer_workspace_bytes(G, R, self.n_pages, self.b0, BLOCK)
        self.ws = torch.zeros(ws, dtype=torch.uint8, device=dev)
        aws = tw.ops.decode_attention_workspace_bytes(G, R, self.per_group)
        self.attn_ws = torch.zeros(aws, dtype=torch.uint8, device=dev)
        self.out = torch.empty((G, R, 128), dtype=torch.float16, device=dev)

    def args(self, q, kn, vn, stage, stage_rows=None, append=0):
        a = self.tw._lib.DecodeLayerArgs()
        a.slab_k, a.slab_v = self.slab.key_device_ptr, self.slab.value_device_ptr
        a.entry_dirs, a.n_entries, a.max_len, a.first_entry = None, self.G, self.max_len, 0
        a.groups, a.heads_per_group, a.dtype = self.G, self.R, 0
        a.page_min, a.page_max, a.page_capacity = self.pmin.data_ptr(), self.pmax.data_ptr(), self.page_cap
        a.n_pages, a.b0_pages = self.n_pages, self.b0
        a.packed, a.scale, a.minimum = self.packed.data_ptr(), self.scale.data_ptr(), self.minimum.data_ptr()
        a.int4_group_size, a.sink, a.block_size, a.top_p = 32, SINK, BLOCK, 0.95
        a.old_length, a.sink_end, a.recent_start = self.L, self.sink_end, self.recent_start
        a.q, a.k_new, a.v_new = q.data_ptr(), kn.data_ptr(), vn.data_ptr()
        a.out, a.out_dtype, a.append = self.out.data_ptr(), 0, append
        a.pages, a.union_pos, a.pos_stride = self.pages.data_ptr(), self.union_pos.data_ptr(), self.max_len
        a.union_count, a.head_count = self.union_count.data_ptr(), self.head_count.data_ptr()
        a.head_pos, a.error_flag = None, self.err.data_ptr()
        a.select_workspace, a.select_workspace_bytes = self.ws.data_ptr(), self.ws.numel()
        a.attn_workspace, a.attn_workspace_bytes = self.attn_ws.data_ptr(), self.attn_ws.numel()
        a.max_rows_per_group, a.reuse = self.per_group, None
        if stage is not None:
            a.stage_k, a.stage_v = stage[0].data_ptr(), stage[1].data_ptr()
            a.stage_rows = stage.shape[2] if stage_rows is None else stage_rows
        return a

    def call(self, a) -> int:
        st = torch.cuda.current_stream().cuda_stream
        return self.tw.load_library().tw_twilight_decode_layer(ctypes.byref(a), st)


def test_staging_through_the_c_abi_on_a_direct_slab(tw, cuda):
    """With no entry directory the staging cluster reads the slab by entry
    stride.  The stage then holds exactly the slab's sink and recent rows, and
    the output equals the unstaged call's bit for bit."""
    G, R, L = 8, 4, 6000
    s = _SlabStep(tw, cuda, G, R, L, seed=5)
    q, kn, vn = _inputs(G, R, torch.float16, 77, cuda)
    stage = torch.full((2, G, SINK + RECENT, 128), float("nan"), dtype=torch.float16, device=cuda)
    assert s.call(s.args(q, kn, vn, None)) == 0
    torch.cuda.synchronize()
    plain = s.out.clone()
    counts = s.union_count.clone()
    assert s.call(s.args(q, kn, vn, stage)) == 0
    torch.cuda.synchronize()
    assert int(s.err.item()) == 0
    assert torch.equal(s.out, plain)
    assert torch.equal(s.union_count, counts)
    n_sink, n_recent = s.sink_end, L - s.recent_start
    for plane, src in ((0, s.data.keys), (1, s.data.values)):
        want = torch.cat((src[:, :n_sink], src[:, s.recent_start:L]), dim=1)
        assert torch.equal(stage[plane, :, :n_sink + n_recent].cpu(), want)
    # with the append (run by the same extra cluster) the token lands at
    # position L of every entry's slab rows, and the output is unchanged
    assert s.call(s.args(q, kn, vn, stage, append=1)) == 0
    torch.cuda.synchronize()
    assert torch.equal(s.out, plain)
    assert torch.equal(s.slab.rows[0, :, L], kn.cpu())
    assert torch.equal(s.slab.rows[1, :, L], vn.cpu())
    s.slab.close()


def test_staging_capacity_is_checked(tw, cuda):
    """A stage smaller than the protected rows is refused before any launch."""
    G, R, L = 2, 4, 2000
    s = _SlabStep(tw, cuda, G, R, L, seed=6)
    q, kn, vn = _inputs(G, R, torch.float16, 78, cuda)
    stage = torch.empty((2, G, SINK + RECENT, 128), dtype=torch.float16, device=cuda)
    need = s.sink_end + (L - s.recent_start)
    assert s.call(s.args(q, kn, vn, stage, stage_rows=need - 1)) == tw._lib.TW_ERR_CAPACITY
    assert s.call(s.args(q, kn, vn, stage, stage_rows=need)) == 0
    torch.cuda.synchronize()
    s.slab.close()


@pytest.mark.parametrize("dtype,group,resident", [("float16", 32, ()), ("bfloat16", 128, (0, 3))])
def test_fused_append_equals_append_kernel(tw, cuda, dtype, group, resident):
    """decode_layer appends the new token in the selection launch's extra
    cluster; prepare_layer_selection + attend_layer appends it with the
    separate append kernel.  Over 20 steps (a new Quest page starts at the first
    one) the slab rows, the running page min / max and the INT4 codes, scales
    and minima are identical, and so are the outputs."""
    G, R, L, steps = 4, 4, 2000, 20
    tdt = synth.TORCH_DTYPES[dtype]
    d = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype=dtype, seed=23,
                         workload="outliers")
    kw = {"resident_entries": list(resident)} if resident else {}
    caches = []
    for _ in range(2):
        c = tw.TwilightMatchedBudgetOffloadedCache(
            num_cache_entries=G, max_cache_len=L + steps + 8, head_dim=128,
            num_query_heads_per_kv=R, dtype=tdt, device=cuda, sink_tokens=SINK,
            recent_tokens=RECENT, block_size=BLOCK, candidate_token_budget=512, top_p=0.95,
            budget_mode="dynamic", layer_batched_selection=True, gqa_groupwise_execution=True,
            qk_backend="cuda", int4_group_size=group, incremental_page_metadata=True, **kw)
        c.prefill_layer(key_states=d.keys.to(cuda), value_states=d.values.to(cuda),
                        entries=list(range(G)))
        caches.append(c)
    assert (L - SINK) % BLOCK == 0  # the first appended token opens a page
    for step in range(steps):
        q, kn, vn = _inputs(G, R, tdt, 700 + step, cuda)
        one = caches[0].decode_layer(queries=q, key_states=kn, value_states=vn,
                                     entries=list(range(G)))
        qs = [q[g].view(1, R, 1, 128) for g in range(G)]
        caches[1].prepare_layer_selection(entries=list(range(G)), queries=qs)
        two = caches[1].attend_layer(key_states=[kn[g].view(1, 1, 1, 128) for g in range(G)],
                                     value_states=[vn[g].view(1, 1, 1, 128) for g in range(G)],
                                     queries=qs, entries=list(range(G)))
        torch.cuda.synchronize()
        assert torch.equal(one, two), step
    a, b = caches
    pages = (L + steps - SINK + BLOCK - 1) // BLOCK  # pages holding written tokens
    for name in ("_page_min", "_page_max"):
        assert torch.equal(getattr(a, name)[:, :pages], getattr(b, name)[:, :pages]), name
    for name in ("_packed", "_scale", "_minimum"):  # positions written so far
        assert torch.equal(getattr(a, name)[:, :L + steps], getattr(b, name)[:, :L + steps]), name
    for g in range(G):
        for kind in ("key", "value"):
            ra = a.entry_kv(kind, g)[L:L + steps].cpu()
            rb = b.entry_kv(kind, g)[L:L + steps].cpu()
            assert torch.equal(ra, rb), (kind, g)
    for c in caches:
        c.synchronize()
        c.close()
