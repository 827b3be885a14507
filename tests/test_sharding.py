"""Multi-rank host logic on CPU with gloo, world size 2 (request and KV-head
sharding, the head-output all-gather, the max-over-ranks timer)."""

from __future__ import annotations

import importlib
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    sys.path.insert(0, str(REPO))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = importlib.import_module("twilight-cpu-gpu-offloading_b200.sharding")
        heads = sh.shard_kv_heads(8, world, rank)
        R, D = 4, 128
        local = torch.stack([torch.full((R, D), float(h), dtype=torch.float32) for h in heads])
        full = sh.gather_head_outputs(local)
        ok_gather = full.shape == (8, R, D) and all(
            bool((full[h] == float(h)).all()) for h in range(8))
        slowest = sh.max_over_ranks(10.0 + rank)
        reqs = sh.shard_requests(16, world, rank)
        results[rank] = (ok_gather, slowest, reqs, list(heads))
    finally:
        dist.destroy_process_group()


def test_sharding_with_gloo_world_size_2():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, port, results), nprocs=world, join=True,
                       start_method="spawn")
    assert results[0][0] and results[1][0]
    assert results[0][1] == results[1][1] == 11.0
    assert results[0][2] + results[1][2] == list(range(16))
    assert results[0][3] == [0, 1, 2, 3] and results[1][3] == [4, 5, 6, 7]


def test_shard_ranges(tw):
    sh = importlib.import_module("twilight-cpu-gpu-offloading_b200.sharding")
    for n in (0, 1, 7, 16, 17):
        for world in (1, 2, 3, 8):
            parts = [list(sh.shard_range(n, world, r)) for r in range(world)]
            assert sum(parts, []) == list(range(n))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
    with pytest.raises(ValueError):
        sh.shard_kv_heads(8, 3, 0)


def test_gather_head_outputs_without_process_group():
    """A single process with no process group owns every KV head: the
    all-gather is the identity (HeadShardedLayerStep then runs unsharded)."""
    import torch.distributed as dist

    if dist.is_initialized():
        pytest.skip("a process group is already initialised")
    sys.path.insert(0, str(REPO))
    sh = importlib.import_module("twilight-cpu-gpu-offloading_b200.sharding")
    local = torch.arange(24, dtype=torch.float32).view(2, 3, 4)
    assert sh.gather_head_outputs(local) is local
