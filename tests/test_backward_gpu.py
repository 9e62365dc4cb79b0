"""Backward kernels (fa_sm100_bwd) against fp32 autograd on the CPU.

Tolerance, as in the flash-attention project's own backward tests: the error
of each gradient against the fp32 oracle must stay within twice the error of
a straightforward implementation that computes in the input dtype (torch
attention with autograd on the GPU), plus 1e-3 of the gradient's magnitude.
"""
import math

import pytest
import torch

from oracle.attention_oracle import make_inputs, math_attention_backward

pytestmark = pytest.mark.gpu


def _lowp_grads(q, k, v, do, causal, q_off):
    """Gradients from plain torch attention computed in the input dtype."""
    h, hk = q.shape[2], k.shape[2]
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    kr, vr = kd.repeat_interleave(h // hk, dim=2), vd.repeat_interleave(h // hk, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", qd, kr).float() / math.sqrt(q.shape[3])
    dead = None
    if causal:
        i = torch.arange(q.shape[1], device="cuda")[:, None] + q_off
        j = torch.arange(k.shape[1], device="cuda")[None, :]
        s = s.masked_fill(j > i, float("-inf"))
        # rows that see no key at all contribute nothing (P = 0), as in the kernels
        dead = torch.isinf(s).all(dim=-1, keepdim=True)
        s = s.masked_fill(dead, 0.0)
    p = torch.softmax(s, dim=-1)
    if dead is not None:
        p = p.masked_fill(dead, 0.0)
    p = p.to(q.dtype)
    o = torch.einsum("bhqk,bkhd->bqhd", p, vr)
    o.backward(do.cuda())
    return qd.grad.float().cpu(), kd.grad.float().cpu(), vd.grad.float().cpu()


def _check(grads, lowp, ref):
    for name, g, l, r in zip(("dq", "dk", "dv"), grads, lowp, ref):
        err = (g.float().cpu() - r).abs().max().item()
        err_lowp = (l - r).abs().max().item()
        bound = 2 * err_lowp + 1e-3 * r.abs().max().item()
        assert err <= bound, f"{name}: max err {err:.3e} > bound {bound:.3e} (low-precision reference {err_lowp:.3e})"


@pytest.mark.parametrize(
    "b,sq,sk,h,hk,d,dtype,causal",
    [
        (2, 256, 256, 4, 4, 128, torch.bfloat16, False),
        (2, 300, 300, 4, 4, 64, torch.float16, True),
        (1, 384, 640, 8, 2, 128, torch.bfloat16, True),  # GQA, s_q < s_k, bottom-right causal
        (2, 129, 200, 2, 2, 128, torch.float16, False),  # tails
        (1, 1024, 1024, 2, 1, 64, torch.bfloat16, True),  # MQA
        (1, 640, 384, 4, 2, 128, torch.bfloat16, True),  # s_q > s_k: the first 256 rows see no key
    ],
)
def test_backward_matches_fp32_autograd(b, sq, sk, h, hk, d, dtype, causal):
    from flash_attention._C import forward_with_lse
    from flash_attention.backward import flash_attn_backward

    q, k, v = make_inputs(b, sq, h, d, dtype, seed=71, seqlen_k=sk, heads_k=hk)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(72)).to(dtype)
    q_off = sk - sq if causal else 0
    qd, kd, vd, dod = q.cuda(), k.cuda(), v.cuda(), do.cuda()
    o, lse = forward_with_lse(qd, kd, vd, causal, q_pos_offset=q_off)
    grads = flash_attn_backward(dod, qd, kd, vd, o, lse, causal, q_pos_offset=q_off)
    torch.cuda.synchronize()
    ref = math_attention_backward(q, k, v, do, causal, q_pos_offset=q_off)
    _check(grads, _lowp_grads(q, k, v, do, causal, q_off), ref)


def test_backward_is_deterministic():
    from flash_attention._C import forward_with_lse
    from flash_attention.backward import flash_attn_backward

    q, k, v = (t.cuda() for t in make_inputs(2, 512, 4, 128, torch.bfloat16, seed=73))
    do = torch.randn_like(q)
    o, lse = forward_with_lse(q, k, v, True)
    a = flash_attn_backward(do, q, k, v, o, lse, True)
    b = flash_attn_backward(do, q, k, v, o, lse, True)
    assert all(torch.equal(x, y) for x, y in zip(a, b))


def test_autograd_function():
    from flash_attention.backward import flash_attn_func_train

    q, k, v = make_inputs(1, 256, 2, 64, torch.float16, seed=74)
    do = torch.randn(q.shape, generator=torch.Generator().manual_seed(75)).to(torch.float16)
    qd, kd, vd = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = flash_attn_func_train(qd, kd, vd, True)
    o.backward(do.cuda())
    ref = math_attention_backward(q, k, v, do, True)
    _check((qd.grad, kd.grad, vd.grad), _lowp_grads(q, k, v, do, True, 0), ref)


def test_backward_empty_keys_and_strided_dout():
    from flash_attention._C import forward_with_lse
    from flash_attention.backward import flash_attn_backward

    q = torch.randn(1, 64, 2, 64, device="cuda", dtype=torch.float16)
    k = torch.empty(1, 0, 2, 64, device="cuda", dtype=torch.float16)
    o = torch.zeros_like(q)
    lse = torch.full((1, 2, 64), float("-inf"), device="cuda")
    dq, dk, dv = flash_attn_backward(torch.randn_like(q), q, k, k, o, lse, False)
    assert dk.numel() == 0 and dv.numel() == 0 and bool((dq == 0).all())
    # dO given as a non-contiguous view gives the same gradients as its copy
    q, k, v = (t.cuda() for t in make_inputs(1, 256, 2, 128, torch.bfloat16, seed=76))
    o, lse = forward_with_lse(q, k, v, True)
    do_big = torch.randn(1, 256, 2, 256, device="cuda", dtype=torch.bfloat16)
    do = do_big[..., ::2]
    a = flash_attn_backward(do, q, k, v, o, lse, True)
    b = flash_attn_backward(do.contiguous(), q, k, v, o, lse, True)
    assert all(torch.equal(x, y) for x, y in zip(a, b))
