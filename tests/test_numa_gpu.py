"""NUMA-placed slabs (tw_host_alloc_mapped_numa): the slab lands on the host
NUMA node closest to the GPU (or the one asked for), kernels read it like the
default pinned slab, and a cache built on it decodes bit-identically."""

from __future__ import annotations

import pytest
import torch

from oracle import synth

pytestmark = pytest.mark.gpu


def test_numa_slab_placement_and_reads(tw, cuda):
    geom = tw.SlabGeometry(num_entries=2, batch_size=1, max_cache_len=4096, head_dim=128)
    slab = tw.MappedHostSlab(geom, torch.bfloat16, numa_node="auto")
    plain = tw.MappedHostSlab(geom, torch.bfloat16)
    g = torch.Generator().manual_seed(0)
    data = torch.randn(2, 2, 4096, 128, generator=g).to(torch.bfloat16)
    slab.rows.copy_(data)
    plain.rows.copy_(data)
    if slab.numa_node is not None:
        # every touched page sits on the bound node
        for off in (0, slab.nbytes // 2, slab.nbytes - 4096):
            assert slab.page_node(off) == slab.numa_node
    rows = torch.randperm(2 * 4096, generator=g)[:1000].to(torch.int64).to(cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    outs = []
    for s in (slab, plain):
        ok = torch.empty(1000, 128, dtype=torch.bfloat16, device=cuda)
        ov = torch.empty_like(ok)
        tw.ops.gather_kv((s.rows[0].view(-1, 128), s.key_device_ptr),
                         (s.rows[1].view(-1, 128), s.value_device_ptr), rows, ok, ov, err)
        outs.append((ok, ov))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert torch.equal(outs[0][0].cpu(), data[0].view(-1, 128)[rows.cpu()])
    slab.close()
    plain.close()


def test_numa_cache_decodes_like_default(tw, cuda):
    G, R, L = 2, 4, 2048
    d = synth.make_layer(groups=G, heads_per_group=R, length=L, dtype="bfloat16", seed=9)
    caches = []
    for numa in (None, "auto"):
        c = tw.TwilightMatchedBudgetOffloadedCache(
            num_cache_entries=G, max_cache_len=L + 8, head_dim=128, num_query_heads_per_kv=R,
            dtype=torch.bfloat16, device=cuda, candidate_token_budget=512, top_p=0.95,
            budget_mode="dynamic", layer_batched_selection=True, gqa_groupwise_execution=True,
            qk_backend="cuda", int4_group_size=32, host_numa_node=numa)
        for e in range(G):
            c.update(d.keys[e].view(1, 1, L, 128).to(cuda), d.values[e].view(1, 1, L, 128).to(cuda), e)
        caches.append(c)
    assert "host_slab_numa_node" in caches[1].state_snapshot()
    for step in range(2):
        g = torch.Generator().manual_seed(step)
        q = torch.randn(G, R, 128, generator=g).to(torch.bfloat16).to(cuda)
        kn = torch.randn(G, 128, generator=g).to(torch.bfloat16).to(cuda)
        vn = torch.randn(G, 128, generator=g).to(torch.bfloat16).to(cuda)
        a, b = (c.decode_layer(queries=q, key_states=kn, value_states=vn, entries=[0, 1]) for c in caches)
        torch.cuda.synchronize()
        assert torch.equal(a, b)
    for c in caches:
        c.close()
