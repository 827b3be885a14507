"""Multi-GPU partitioning of the sparse decode path (one process per GPU).

The path needs no collective on its data plane: requests are independent, and
so are the (layer, KV head) entries of one request.  Two layouts:

* request sharding: each rank owns whole requests (its own slab on its own
  GPU); nothing is exchanged;
* KV-head sharding of one request: each rank owns a contiguous block of KV
  heads of every layer and computes their attention outputs; one all-gather
  of the [G_local, R, D] outputs per layer rebuilds the [G, R, D] input of
  o_proj (hi/mp.py:276-278 feeds the reshaped attention output to o_proj).
  With NCCL over NVLink that is G*R*D*2 bytes per layer (e.g. 8*8*128*2 =
  16 KiB for a 70B layer).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> range:
    """Contiguous block of n items owned by `rank` (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("invalid world/rank")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def shard_requests(n_requests: int, world: int, rank: int) -> list[int]:
    """Request ids this rank serves (request sharding)."""
    return list(shard_range(n_requests, world, rank))


def shard_kv_heads(kv_heads: int, world: int, rank: int) -> range:
    """KV heads of every layer this rank owns (KV-head sharding); requires an
    even split so that every rank's all-gather contribution has one shape."""
    if kv_heads % world:
        raise ValueError(f"{kv_heads} KV heads do not split evenly over {world} ranks")
    return shard_range(kv_heads, world, rank)


def gather_head_outputs(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather [G_local, R, D] attention outputs into [G, R, D] (rank order =
    KV-head order).  Runs on the tensors' device: NCCL on CUDA, gloo on CPU."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return local
    out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out


def max_over_ranks(value: float, device: torch.device | None = None, group=None) -> float:
    """Max of a per-rank float (the slowest rank's time)."""
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=device if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class HeadShardedLayerStep:
    """Decode layer-steps of one request whose KV heads are sharded over the
    ranks of a process group (e.g. a 70B layer at 131072 tokens with one KV-head
    group per GPU).

    Each rank owns `cache`, a TwilightMatchedBudgetOffloadedCache holding only
    its KV heads (entries = layer * heads_local + i).  `step` runs the local
    sparse layer-step (selection, zero-copy gather + attention, append) and
    all-gathers the [heads_local, R, D] outputs into the [G, R, D] tensor that
    o_proj consumes.  q / k_new / v_new are the full [G, R, D] / [G, D] inputs;
    each rank reads its own slice (in a tensor-parallel model each rank would
    compute only that slice)."""

    def __init__(self, cache, kv_heads: int, group=None) -> None:
        self.cache = cache
        self.group = group
        # without a process group the one process owns every KV head
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.heads = shard_kv_heads(kv_heads, self.world, self.rank)
        self.heads_local = len(self.heads)
        if cache.geometry.num_entries % self.heads_local:
            raise ValueError("cache entries must be layers x local KV heads")

    def step(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             out_local: torch.Tensor | None = None) -> torch.Tensor:
        h0, h1 = self.heads.start, self.heads.stop
        entries = [layer * self.heads_local + i for i in range(self.heads_local)]
        local = self.cache.decode_layer(queries=q[h0:h1].contiguous(),
                                        key_states=k_new[h0:h1].contiguous(),
                                        value_states=v_new[h0:h1].contiguous(), entries=entries,
                                        out=out_local)
        return gather_head_outputs(local, self.group)
