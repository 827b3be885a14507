"""Decode-layer front end (tw_qkv_rope): q / k / v projection + rotary embedding.

Floating-point kernel, so the check is against torch:
* the projection (cos = 1, sin = 0 leaves it unrotated) against a float64
  matmul of the same operands: within one unit in the last place of the model
  dtype plus the fp32 summation error bound of the dot product;
* the rotation against the Llama formula out = x*cos + rotate_half(x)*sin
  (hi/mp.py:139, :169, :205 call it) evaluated by torch in the model dtype on
  the kernel's own projections: bit for bit (each product and the sum rounded
  to the dtype, as torch's elementwise ops do).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def rope_tables(position: int, dtype, dev, base: float = 500000.0):
    inv = 1.0 / (base ** (torch.arange(0, 128, 2, dtype=torch.float32) / 128))
    freqs = position * inv
    emb = torch.cat((freqs, freqs))
    return emb.cos().to(dtype).to(dev), emb.sin().to(dtype).to(dev)


def ulp(x: torch.Tensor, dtype) -> torch.Tensor:
    mant = 7 if dtype == torch.bfloat16 else 10
    e = torch.floor(torch.log2(x.abs().clamp_min(1e-30)))
    return torch.exp2(e - mant)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(4096, 32, 8), (2048, 16, 4), (8192, 64, 8)])
def test_qkv_rope_matches_torch(tw, cuda, dtype, shape):
    H, n_q, n_kv = shape
    g = torch.Generator().manual_seed(H + n_q)
    scale = H ** -0.5
    hidden = torch.randn(H, generator=g).to(dtype).to(cuda)
    w_q = (torch.randn(n_q * 128, H, generator=g) * scale).to(dtype).to(cuda)
    w_k = (torch.randn(n_kv * 128, H, generator=g) * scale).to(dtype).to(cuda)
    w_v = (torch.randn(n_kv * 128, H, generator=g) * scale).to(dtype).to(cuda)
    one = torch.ones(128, dtype=dtype, device=cuda)
    zero = torch.zeros(128, dtype=dtype, device=cuda)
    q_raw, k_raw, v_raw = tw.ops.qkv_rope(hidden, w_q, w_k, w_v, one, zero)
    torch.cuda.synchronize()
    for w, got in ((w_q, q_raw), (w_k, k_raw), (w_v, v_raw)):
        ref32 = (w.double() @ hidden.double()).view_as(got)
        # one rounding to the dtype plus the fp32 summation error of an
        # H-term dot product (probabilistic bound 4 * 2^-24 * sqrt(H) * sum|w h|)
        mag = (w.double().abs() @ hidden.double().abs()).view_as(got)
        tol = ulp(ref32.float(), dtype).double() + 4 * 2.0 ** -24 * H ** 0.5 * mag
        err = (got.double() - ref32).abs()
        assert bool((err <= tol).all()), float((err / tol).max())
    for position in (0, 7, 32767, 131071):
        cos, sin = rope_tables(position, dtype, cuda)
        q, k, v = tw.ops.qkv_rope(hidden, w_q, w_k, w_v, cos, sin)
        torch.cuda.synchronize()
        q_ref = (q_raw * cos) + (rotate_half(q_raw) * sin)
        k_ref = (k_raw * cos) + (rotate_half(k_raw) * sin)
        assert torch.equal(q, q_ref), position
        assert torch.equal(k, k_ref), position
        assert torch.equal(v, v_raw), position


def test_qkv_rope_argument_checks(tw, cuda):
    dt = torch.bfloat16
    h = torch.zeros(300, dtype=dt, device=cuda)  # not a multiple of 256
    w = torch.zeros(128, 300, dtype=dt, device=cuda)
    c = torch.zeros(128, dtype=dt, device=cuda)
    with pytest.raises(ValueError):
        tw.ops.qkv_rope(h, w, w, w, c, c)
    h = torch.zeros(256, dtype=dt, device=cuda)
    w = torch.zeros(128, 256, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError):
        tw.ops.qkv_rope(h, w, w, w, c, c)
