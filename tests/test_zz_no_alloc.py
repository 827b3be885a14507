"""tw_decode_attention_noalloc: the allocation-free entry point.

It exists for callers that cannot allocate device memory (a serving runtime
whose device memory is all reserved for its own arena, a host in another
language that receives device buffers but has no CUDA allocator), so it keeps
its split-K scratch in a fixed array inside the library instead of a caller
workspace.  These checks call it through the C ABI and compare it with the
workspace entry point, tw_decode_attention, on two calls in a row (the second
call finds the first call's leftovers in the shared array).  This file is
collected last so a failure here comes after every other test has run.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

from tolerance import ATTN_TOL_16BIT, ATTN_TOL_FP32

pytestmark = pytest.mark.gpu


def _call_noalloc(lib, q, k, v, cu, max_len, out, out_dtype_code, lse):
    return lib.tw_decode_attention_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), cu.data_ptr(), q.shape[0], q.shape[1], max_len,
        128, 0 if q.dtype == torch.float16 else 1, ctypes.c_float(1.0 / math.sqrt(128)),
        out.data_ptr(), out_dtype_code, lse.data_ptr(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_noalloc_matches_workspace_entry_point(tw, cuda, dtype):
    lib = tw.load_library()
    for call, (S, R, lengths) in enumerate([(8, 4, [4400, 1, 129, 300, 2000, 8, 4096, 257]),
                                            (4, 8, [1000, 3000, 1, 128])]):
        g = torch.Generator().manual_seed(100 + call)
        total = sum(lengths)
        q = torch.randn(S, R, 128, generator=g).to(dtype).to(cuda)
        k = torch.randn(total, 128, generator=g).to(dtype).to(cuda)
        v = torch.randn(total, 128, generator=g).to(dtype).to(cuda)
        cu = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32, device=cuda)
        max_len = max(lengths)
        ws = torch.zeros(tw.ops.decode_attention_workspace_bytes(S, R, max_len), dtype=torch.uint8,
                         device=cuda)
        for out_dtype in (torch.float32, dtype):
            code = tw._lib.TW_F32 if out_dtype == torch.float32 else (0 if dtype == torch.float16 else 1)
            ref_lse = torch.zeros(S, R, device=cuda)
            ref = tw.ops.decode_attention(q, k, v, cu, max_len, workspace=ws, out_dtype=out_dtype,
                                          lse=ref_lse)
            out = torch.full((S, R, 128), float("nan"), dtype=out_dtype, device=cuda)
            lse = torch.zeros(S, R, device=cuda)
            tw._lib.check(_call_noalloc(lib, q, k, v, cu, max_len, out, code, lse), "noalloc")
            torch.cuda.synchronize()
            tol = ATTN_TOL_FP32 if out_dtype == torch.float32 else ATTN_TOL_16BIT
            diff = (out.float() - ref.float()).abs().max().item()
            assert diff <= tol, (call, out_dtype, diff)
            assert (lse - ref_lse).abs().max().item() <= ATTN_TOL_FP32


def test_noalloc_rejects_oversized_scratch(tw, cuda):
    lib = tw.load_library()
    q = torch.zeros(64, 8, 128, dtype=torch.float16, device=cuda)
    k = torch.zeros(1, 128, dtype=torch.float16, device=cuda)
    cu = torch.zeros(65, dtype=torch.int32, device=cuda)
    out = torch.zeros_like(q)
    lse = torch.zeros(64, 8, device=cuda)
    # 64 segments x 8 heads x 1024 splits of partials: far beyond the fixed array
    rc = _call_noalloc(lib, q, k, k, cu, 131072, out, 0, lse)
    assert rc == tw._lib.TW_ERR_CAPACITY
