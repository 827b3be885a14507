"""Seeded synthetic decode inputs.  TEST INFRASTRUCTURE ONLY.

Used by tests/, tests/golden/make_golden.py, __graft_entry__.smoke() and
bench.py to build the same K/V/query data on any machine.  The generator is
splitmix64 + Box-Muller in float64 (no dependence on numpy's distribution
algorithms), rounded to the K/V dtype by torch (round to nearest even).

Workloads (the reference publishes no inputs for this path; these follow the
configurations the benchmark is defined on):

* ``needles``: K, V ~ N(0, 1); per KV head ``n_needles`` random eligible pages
  whose keys are 0.5 * q_hat + N(0, 0.5), q_hat = sqrt(D) * m / |m| with m the
  group's mean query (a needle key then has an ordinary key's magnitude).
* ``outliers``: K ~ N(0, 1) with ``n_outlier_channels`` channels per KV head
  scaled by exp(N(0, 1)); V ~ N(0, 1).  Optional needles at random pages.
Queries are N(0, 1) per head, rounded to the K/V dtype.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def _splitmix(seed: int, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        i = np.arange(1, n + 1, dtype=np.uint64)
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) * _GOLDEN + i * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, n: int) -> np.ndarray:
    """n doubles in (0, 1)."""
    z = _splitmix(seed, n)
    return ((z >> np.uint64(11)).astype(np.float64) + 0.5) * (1.0 / 9007199254740992.0)


def normal(seed: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    u1 = uniform(seed * 2 + 1, n)
    u2 = uniform(seed * 2 + 2, n)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return z.reshape(shape)


def integers(seed: int, n: int, high: int) -> np.ndarray:
    return (_splitmix(seed, n) % np.uint64(high)).astype(np.int64)


def distinct(seed: int, k: int, high: int) -> np.ndarray:
    """k distinct integers in [0, high) (k <= high), ascending."""
    if k > high:
        raise ValueError("cannot draw more distinct values than the range holds")
    keys = _splitmix(seed, high)
    return np.sort(np.argsort(keys, kind="stable")[:k]).astype(np.int64)


TORCH_DTYPES = {"float16": torch.float16, "bfloat16": torch.bfloat16}


@dataclass
class DecodeLayer:
    """One decoder layer's cache content and decode inputs.

    keys/values: [G, L, D]; queries: [G, R, D]; key_new/value_new: [G, D].
    """

    keys: torch.Tensor
    values: torch.Tensor
    queries: torch.Tensor
    key_new: torch.Tensor
    value_new: torch.Tensor
    needle_pages: np.ndarray  # [G, n_needles] (page ids after the sink)


def make_layer(*, groups: int, heads_per_group: int, length: int, head_dim: int = 128,
               dtype: str = "float16", seed: int = 0, workload: str = "outliers",
               sink: int = 64, recent: int = 256, block: int = 16, n_needles: int = 0,
               n_outlier_channels: int = 4) -> DecodeLayer:
    G, R, L, D = groups, heads_per_group, length, head_dim
    tdt = TORCH_DTYPES[dtype]
    base = seed * 1000003
    keys = normal(base + 1, (G, L, D))
    values = normal(base + 2, (G, L, D))
    queries = normal(base + 3, (G, R, D))
    key_new = normal(base + 4, (G, D))
    value_new = normal(base + 5, (G, D))
    if workload == "outliers":
        for g in range(G):
            ch = distinct(base + 100 + g, n_outlier_channels, D)
            scale = np.exp(normal(base + 200 + g, (n_outlier_channels,)))
            keys[g][:, ch] *= scale
    elif workload != "needles":
        raise ValueError(f"unknown workload {workload!r}")
    q_round = torch.from_numpy(queries).to(tdt).to(torch.float64).numpy()
    sink_end = min(sink, L)
    recent_start = max(sink_end, L - max(0, recent - 1))
    eligible_pages = max(0, recent_start - sink_end) // block
    needle_pages = np.zeros((G, 0), dtype=np.int64)
    if n_needles and eligible_pages:
        k = min(n_needles, eligible_pages)
        needle_pages = np.stack([distinct(base + 300 + g, k, eligible_pages) for g in range(G)])
        for g in range(G):
            m = q_round[g].mean(axis=0)
            q_hat = np.sqrt(D) * m / max(np.linalg.norm(m), 1e-12)
            for p in needle_pages[g]:
                start = sink + int(p) * block
                noise = 0.5 * normal(base + 400 + g * 100003 + int(p), (block, D))
                keys[g, start:start + block] = 0.5 * q_hat + noise
    to = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(tdt)  # noqa: E731
    return DecodeLayer(to(keys), to(values), to(queries), to(key_new), to(value_new), needle_pages)
