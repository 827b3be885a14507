"""The reference's own OpenMP gather (hi/cpu_kv_gather.cpp, hi/cpu_kv_run_gather.cpp),
compiled from its sources into oracle/_ref/ — the CPU baseline's gather — holds
the reference's test contract (scripts/test_cpu_kv_gather_v1.py,
scripts/test_cpu_kv_run_gather_v1.py)."""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


def _load(name):
    path = REF / name
    if not path.exists():
        pytest.skip(f"{path.name} not built (needs the reference sources: make -C oracle)")
    lib = ctypes.CDLL(str(path))
    lib.gather_kv.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 3 + [ctypes.c_int]
    lib.gather_kv.restype = ctypes.c_int
    return lib


@pytest.mark.parametrize("name", ["libref_cpu_kv_gather.so", "libref_cpu_kv_run_gather.so"])
def test_reference_gather_contract(name):
    lib = _load(name)
    g = torch.Generator().manual_seed(123)
    k = torch.randn(10000, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(10000, 128, generator=g).to(torch.bfloat16)
    patterns = [torch.empty(0, dtype=torch.long), torch.tensor([9999]), torch.arange(9999),
                torch.randint(10000, (8192,), generator=g), torch.arange(8192).flip(0),
                torch.cat([torch.arange(100, 500), torch.tensor([0, 0, 9999]), torch.arange(1000, 7000)])]
    for threads in (1, 4):
        for rows in patterns:
            a = torch.full((rows.numel() + 2, 128), -42.0, dtype=k.dtype)
            b = torch.full_like(a, -42.0)
            n = rows.numel()
            if n:
                rc = lib.gather_kv(k.data_ptr(), v.data_ptr(), a[1:].data_ptr(), b[1:].data_ptr(),
                                   rows.data_ptr(), n, 10000, 256, threads)
                assert rc == 0
            assert torch.equal(a[1:-1], k.index_select(0, rows))
            assert torch.equal(b[1:-1], v.index_select(0, rows))
            assert (a[[0, -1]] == -42).all()
    for bad in (-1, 10000):
        rows = torch.tensor([bad])
        out = torch.empty(1, 128, dtype=k.dtype)
        assert lib.gather_kv(k.data_ptr(), v.data_ptr(), out.data_ptr(), out.data_ptr(),
                             rows.data_ptr(), 1, 10000, 256, 1) == 1
