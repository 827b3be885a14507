"""Drop-in for the reference's varlen decode attention call.

hi/mp.py:21-52 wraps flash_attn_varlen_func and hi/mp.py:258-279 calls it with
q [G, R, D] (one query token per group), K/V [sum_T, 1, D], cu_seqlens_q =
arange(G + 1), cu_seqlens_k [G + 1], max_seqlen_q = 1, causal (q_len 1: all
keys visible), default softmax scale 1/sqrt(D).  This module runs the same
contract on the sm_100a split-K kernel.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops

_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index or 0, nbytes)
    ws = _workspaces.get(key)
    if ws is None:
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def flash_attention_varlen_forward(query_states: torch.Tensor, key_states: torch.Tensor,
                                   value_states: torch.Tensor, cu_seqlens_q: torch.Tensor,
                                   cu_seqlens_k: torch.Tensor, max_seqlen_q: int,
                                   max_seqlen_k: int, *, dropout: float = 0.0,
                                   is_causal: bool = True,
                                   sliding_window: Optional[int] = None,
                                   softmax_scale: Optional[float] = None) -> torch.Tensor:
    """Same arguments as hi/mp.py:21-52 for the decode shapes the GQA group path uses."""
    if max_seqlen_q != 1:
        raise ValueError("the sparse decode attention handles one query token per segment")
    if dropout != 0.0:
        raise ValueError("dropout is not supported at decode")
    if sliding_window is not None and max_seqlen_k > sliding_window:
        raise ValueError("sliding-window attention is not supported")
    S = cu_seqlens_k.numel() - 1
    if query_states.shape[0] != S:
        raise ValueError("one query token per segment expected (cu_seqlens_q = arange(S + 1))")
    k = key_states.reshape(key_states.shape[0], -1)
    v = value_states.reshape(value_states.shape[0], -1)
    R = query_states.shape[1]
    ws = _workspace(query_states.device, ops.decode_attention_workspace_bytes(S, R, max_seqlen_k))
    return ops.decode_attention(query_states.contiguous(), k, v, cu_seqlens_k.to(torch.int32),
                                max_seqlen_k, workspace=ws, softmax_scale=softmax_scale)


def sparse_gqa_decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                cu_seqlens_k: torch.Tensor, max_seqlen_k: int,
                                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """q [S, R, D], k/v [rows, D] -> [S, R, D] (out_dtype: q's dtype or float32)."""
    S, R, _ = q.shape
    ws = _workspace(q.device, ops.decode_attention_workspace_bytes(S, R, max_seqlen_k))
    return ops.decode_attention(q, k, v, cu_seqlens_k, max_seqlen_k, workspace=ws,
                                out_dtype=out_dtype)
