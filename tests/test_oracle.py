"""CPU checks of the oracle itself (no GPU)."""
import math

import numpy as np
import pytest
import torch

from oracle.attention_oracle import make_inputs, math_attention, tiled_reference_algorithm


def naive(q, k, v, causal, scale=None, q_off=0, k_off=0):
    qf, kf, vf = (t.float() for t in (q, k, v))
    d = q.shape[-1]
    scale = 1 / math.sqrt(d) if scale is None else scale
    s = torch.einsum("bihd,bjhd->bhij", qf, kf) * scale
    if causal:
        i = torch.arange(q.shape[1])[:, None] + q_off
        j = torch.arange(k.shape[1])[None, :] + k_off
        s = s.masked_fill(j > i, float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.softmax(s, -1)
    return torch.einsum("bhij,bjhd->bihd", p, vf), lse


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("sq,sk", [(17, 17), (64, 64), (33, 70), (70, 33)])
def test_math_attention_matches_naive(causal, sq, sk):
    q, k, v = make_inputs(2, sq, 3, 64, torch.float32, seed=1, seqlen_k=sk)
    o, lse = math_attention(q, k, v, causal, q_chunk=16)
    o_ref, lse_ref = naive(q, k, v, causal)
    if causal and sq > sk:
        # rows i >= sk see all keys; no row is empty for top-left alignment
        pass
    assert torch.allclose(o, o_ref, atol=1e-5, rtol=1e-5)
    assert torch.allclose(lse, lse_ref, atol=1e-5, rtol=1e-5)


def test_math_attention_offsets_and_empty_rows():
    q, k, v = make_inputs(1, 8, 2, 64, torch.float32, seed=3, seqlen_k=8)
    # keys start after the queries: rows 0..2 see nothing
    o, lse = math_attention(q, k, v, True, q_pos_offset=0, k_pos_offset=3)
    assert torch.all(o[:, :3] == 0)
    assert torch.all(torch.isneginf(lse[:, :, :3]))
    o_ref, lse_ref = naive(q[:, 3:], k, v, True, q_off=3, k_off=3)
    assert torch.allclose(o[:, 3:], o_ref, atol=1e-5)
    assert torch.allclose(lse[:, :, 3:], lse_ref, atol=1e-5)


def test_math_attention_linear_in_v():
    q, k, v = make_inputs(1, 40, 2, 64, torch.float32, seed=4)
    v2 = torch.randn_like(v)
    o1, _ = math_attention(q, k, v, True)
    o2, _ = math_attention(q, k, v2, True)
    o12, _ = math_attention(q, k, 2 * v + 3 * v2, True)
    assert torch.allclose(o12, 2 * o1 + 3 * o2, atol=1e-4)


@pytest.mark.parametrize("dtype,tol", [(torch.float16, 2e-3), (torch.bfloat16, 1e-2)])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [64, 128])
def test_tiled_algorithm_close_to_math(dtype, tol, causal, d):
    q, k, v = make_inputs(1, 192, 2, d, dtype, seed=5)
    o_tiled = tiled_reference_algorithm(q, k, v, causal)
    o_math, _ = math_attention(q, k, v, causal)
    assert np.abs(o_tiled - o_math.numpy()).max() <= tol


def test_make_inputs_deterministic():
    a = make_inputs(1, 16, 2, 64, torch.bfloat16, seed=9)
    b = make_inputs(1, 16, 2, 64, torch.bfloat16, seed=9)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("h,hk", [(8, 2), (6, 1)])
def test_math_attention_grouped_heads_equal_repeated_kv(h, hk):
    """GQA in the oracle = plain attention with each K/V head repeated for its
    group of h // hk query heads."""
    q, k, v = make_inputs(2, 96, h, 64, torch.float32, seed=3, heads_k=hk)
    o, lse = math_attention(q, k, v, True)
    rep = h // hk
    o2, lse2 = math_attention(q, k.repeat_interleave(rep, dim=2), v.repeat_interleave(rep, dim=2), True)
    assert torch.equal(o, o2) and torch.equal(lse, lse2)
