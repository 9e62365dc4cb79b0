"""Attention backward on B200 and an autograd-enabled attention call.

The reference ships a forward only; its README lists the backward as not done.
`flash_attn_backward` computes dQ, dK, dV from dO and the forward's O and LSE
through the C ABI (`fa_sm100_bwd`, include/fa_sm100.h), and
`flash_attn_func_train` wraps forward + backward in a torch.autograd.Function.
"""
from __future__ import annotations

import ctypes
import math

import torch

from flash_attention._C import _check, _validate, forward_with_lse, lib


class FaBwdParams(ctypes.Structure):
    """Mirror of ``struct FaBwdParams`` in include/fa_sm100.h."""

    _fields_ = (
        [(n, ctypes.c_void_p) for n in ("q", "k", "v", "o", "dout", "lse", "dq", "dk", "dv", "dvec")]
        + [(n, ctypes.c_int32) for n in ("batch", "seqlen_q", "seqlen_k", "heads", "heads_k", "head_dim")]
        + [
            (f"{t}_{s}_stride", ctypes.c_int64)
            for t in ("q", "k", "v", "o", "do", "dq", "dk", "dv")
            for s in ("batch", "row", "head")
        ]
        + [("lse_batch_stride", ctypes.c_int64), ("lse_head_stride", ctypes.c_int64)]
        + [("softmax_scale", ctypes.c_float), ("is_causal", ctypes.c_int32), ("is_bf16", ctypes.c_int32)]
        + [("q_pos_offset", ctypes.c_int64), ("k_pos_offset", ctypes.c_int64), ("error_flag", ctypes.c_void_p)]
    )


lib.fa_sm100_bwd.argtypes = [ctypes.POINTER(FaBwdParams), ctypes.c_void_p]
lib.fa_sm100_bwd.restype = ctypes.c_int
lib.fa_sm100_bwd_params_size.argtypes = []
lib.fa_sm100_bwd_params_size.restype = ctypes.c_int
if lib.fa_sm100_bwd_params_size() != ctypes.sizeof(FaBwdParams):
    raise ImportError(
        f"FaBwdParams layout mismatch: library {lib.fa_sm100_bwd_params_size()} bytes, "
        f"binding {ctypes.sizeof(FaBwdParams)} bytes"
    )


def flash_attn_backward(
    dout: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    out: torch.Tensor,
    lse: torch.Tensor,
    causal: bool = False,
    *,
    softmax_scale: float | None = None,
    q_pos_offset: int = 0,
    k_pos_offset: int = 0,
):
    """Gradients (dq, dk, dv) of attention given dO, the inputs, and the
    forward's O and LSE ((batch, heads, seqlen_q) fp32).  Shapes, dtypes and
    masking conventions are those of the forward."""
    _validate(q, k, v)
    if dout.stride(-1) != 1:
        dout = dout.contiguous()
    for name, t in (("dout", dout), ("out", out)):
        if t.shape != q.shape or t.dtype != q.dtype or t.device != q.device or t.stride(-1) != 1:
            raise RuntimeError(f"{name} must match q's shape, dtype and device, contiguous in last dim")
    b, sq, h, d = q.shape
    if lse.shape != (b, h, sq) or lse.dtype != torch.float32 or lse.device != q.device or lse.stride(-1) != 1:
        raise RuntimeError("lse must be (batch, heads, seqlen_q) fp32 on q's device, contiguous in its last dim")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dvec = torch.empty((b * h * sq,), dtype=torch.float32, device=q.device)
    p = FaBwdParams()
    p.q, p.k, p.v, p.o, p.dout = q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr()
    p.lse, p.dq, p.dk, p.dv, p.dvec = lse.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dvec.data_ptr()
    p.batch, p.seqlen_q, p.heads, p.head_dim = b, sq, h, d
    p.seqlen_k, p.heads_k = k.size(1), k.size(2)
    for name, t in (("q", q), ("k", k), ("v", v), ("o", out), ("do", dout), ("dq", dq), ("dk", dk), ("dv", dv)):
        setattr(p, f"{name}_batch_stride", t.stride(0))
        setattr(p, f"{name}_row_stride", t.stride(1))
        setattr(p, f"{name}_head_stride", t.stride(2))
    p.lse_batch_stride, p.lse_head_stride = lse.stride(0), lse.stride(1)
    p.softmax_scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
    p.is_causal = 1 if causal else 0
    p.is_bf16 = 1 if q.dtype == torch.bfloat16 else 0
    p.q_pos_offset, p.k_pos_offset = int(q_pos_offset), int(k_pos_offset)
    p.error_flag = None
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        _check(lib.fa_sm100_bwd(ctypes.byref(p), ctypes.c_void_p(stream)), "fa_sm100_bwd")
    return dq, dk, dv


class _FlashAttnFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal):
        o, lse = forward_with_lse(q, k, v, causal)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal = causal
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = flash_attn_backward(do, q, k, v, o, lse, ctx.causal)
        return dq, dk, dv, None


def flash_attn_func_train(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """flash_attn_func with autograd: the backward runs the sm_100a kernels."""
    return _FlashAttnFunction.apply(q, k, v, causal)
