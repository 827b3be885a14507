"""KV-head-sharded decode of one request over 2 GPUs (NCCL all-gather of the
per-head outputs) equals the same request decoded on one GPU, bit for bit.
Skipped with fewer than 2 GPUs."""

from __future__ import annotations

import importlib
import os
import socket
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make(tw, entries, R, L, dev, resident):
    return tw.TwilightMatchedBudgetOffloadedCache(
        num_cache_entries=entries, max_cache_len=L + 8, head_dim=128, num_query_heads_per_kv=R,
        dtype=torch.bfloat16, device=dev, candidate_token_budget=512, top_p=0.95,
        budget_mode="dynamic", layer_batched_selection=True, gqa_groupwise_execution=True,
        qk_backend="cuda", int4_group_size=32, resident_entries=resident)


def _worker(rank, world, port, results):
    sys.path.insert(0, str(REPO))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        tw = importlib.import_module("twilight-cpu-gpu-offloading_b200")
        sh = importlib.import_module("twilight-cpu-gpu-offloading_b200.sharding")
        from oracle import synth
        layers, G, R, L = 2, 4, 8, 2048
        data = [synth.make_layer(groups=G, heads_per_group=R, length=L, dtype="bfloat16",
                                 seed=60 + li, workload="outliers") for li in range(layers)]
        heads = sh.shard_kv_heads(G, world, rank)
        hl = len(heads)
        cache = _make(tw, layers * hl, R, L, dev, resident=[0] if rank == 0 else [])
        for li, d in enumerate(data):
            for i, h in enumerate(heads):
                cache.update(d.keys[h].view(1, 1, L, 128).to(dev), d.values[h].view(1, 1, L, 128).to(dev),
                             li * hl + i)
        stepper = sh.HeadShardedLayerStep(cache, G)
        full = _make(tw, layers * G, R, L, dev, resident=[0]) if rank == 0 else None
        if full is not None:
            for li, d in enumerate(data):
                for h in range(G):
                    full.update(d.keys[h].view(1, 1, L, 128).to(dev), d.values[h].view(1, 1, L, 128).to(dev),
                                li * G + h)
        ok = True
        for step in range(2):
            for li in range(layers):
                g = torch.Generator().manual_seed(100 * step + li)
                q = torch.randn(G, R, 128, generator=g).to(torch.bfloat16).to(dev)
                kn = torch.randn(G, 128, generator=g).to(torch.bfloat16).to(dev)
                vn = torch.randn(G, 128, generator=g).to(torch.bfloat16).to(dev)
                out = stepper.step(li, q, kn, vn)
                if full is not None:
                    ref = full.decode_layer(queries=q, key_states=kn, value_states=vn,
                                            entries=list(range(li * G, li * G + G)))
                    torch.cuda.synchronize()
                    ok = ok and torch.equal(out, ref)
        torch.cuda.synchronize()
        results[rank] = ok
        cache.close()
        if full is not None:
            full.close()
    finally:
        dist.destroy_process_group()


def test_head_sharded_decode_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    mp.start_processes(_worker, args=(2, _free_port(), results), nprocs=2, join=True,
                       start_method="spawn")
    assert results[0] and results[1]
