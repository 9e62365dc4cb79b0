"""Public API -- drop-in for flash_attention/interface.py:5-23 of the reference."""
from __future__ import annotations

import torch

from flash_attention._C import forward, forward_with_lse


def flash_attn_func(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    *,
    return_lse: bool = False,
):
    """
    Flash Attention forward pass on B200 (sm_100a).

    Args:
        q: (batch, seqlen_q, heads, head_dim), fp16/bf16, CUDA
        k: (batch, seqlen_k, heads_k, head_dim), fp16/bf16
        v: (batch, seqlen_k, heads_k, head_dim), fp16/bf16
        causal: whether to apply the causal mask (key j > query i is masked,
            top-left aligned like the reference kernel)
        return_lse: keyword-only addition; also return the log-sum-exp
            (batch, heads, seqlen_q), fp32, natural log

    Returns:
        o: (batch, seqlen_q, heads, head_dim), or (o, lse) if return_lse
    """
    if return_lse:
        return forward_with_lse(q, k, v, causal)
    return forward(q, k, v, causal)
