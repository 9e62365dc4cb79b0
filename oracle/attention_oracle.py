"""CPU oracle for the attention forward.  TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` may import this module, and only as the checker / the timed CPU
baseline.  The product path (``flash_attention``) never calls it: it has no
CPU fallback and fails loudly without its CUDA library.

Two restatements of the reference's attention forward
(YangFan0918/flash-attention-cute, paths below are inside that tree):

``math_attention``
    fp32 math definition  O = softmax(scale * Q K^T [+ causal mask]) V  and
    LSE = logsumexp(scale * Q K^T)  (natural log).  This is the oracle the
    north star names; it is also the CPU baseline that bench.py times.
    Mask semantics follow the reference kernel: key j is hidden from query i
    when j > i (top-left aligned, csrc/flash_fwd_kernel.cuh:174-188), here
    generalised with global position offsets (j + k_off > i + q_off).
    A row with no visible key gives O = 0 (kernel.cuh:277) and LSE = -inf.

``tiled_reference_algorithm``
    Step-by-step restatement of the reference kernel's own algorithm:
    64x64 tiles (csrc/flash_fwd_traits.h:21), fp32 scores, causal mask only
    on diagonal tiles (kernel.cuh:174-188), running max with the scale folded
    into exp2 (kernel.cuh:190-218), an unconditional O rescale every tile
    (kernel.cuh:220-226), P = exp2(s*c - m*c) summed in fp32 (kernel.cuh:228-235),
    P rounded to the input dtype before P.V (kernel.cuh:246-252), final
    O / rowsum with the rowsum==0 -> 1 guard (kernel.cuh:267-282), O rounded
    to the input dtype (kernel.cuh:284-288).  It reproduces the reference's
    outputs to within one rounding of the output dtype, which is what the
    golden vectors under tests/golden/ (outputs of the reference kernel
    itself, built from its sources and run on a B200) pin.

Parity is pinned: tests/test_oracle_golden.py checks both functions against
the reference kernel's own outputs in tests/golden/ref_kernel_cases.npz.
"""
from __future__ import annotations

import math

import numpy as np
import torch

LOG2E = 1.4426950408889634


def _visible_mask(sq: int, sk: int, q_off: int, k_off: int) -> torch.Tensor:
    """True where key j is visible to query i under the causal rule."""
    i = torch.arange(sq, dtype=torch.int64).unsqueeze(1) + q_off
    j = torch.arange(sk, dtype=torch.int64).unsqueeze(0) + k_off
    return j <= i


def math_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    softmax_scale: float | None = None,
    q_pos_offset: int = 0,
    k_pos_offset: int = 0,
    q_chunk: int = 1024,
    heads: list[int] | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 attention on the CPU.

    q: (b, sq, h, d), k/v: (b, sk, hk, d) in any float dtype (upcast to fp32),
    hk dividing h: query head hi attends K/V head hi // (h // hk) (GQA/MQA).
    Returns O (b, sq, h, d) fp32 and LSE (b, h, sq) fp32.  Work is chunked
    by (batch, head, query block) so memory stays at q_chunk x sk floats.
    `heads` restricts the computation to a subset of heads (others left 0).
    """
    b, sq, h, d = q.shape
    sk, hk = k.shape[1], k.shape[2]
    assert h % hk == 0, "heads must be divisible by heads_k"
    group = h // hk
    scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
    out = torch.zeros((b, sq, h, d), dtype=torch.float32)
    lse = torch.full((b, h, sq), float("-inf"), dtype=torch.float32)
    if sq == 0 or b == 0:
        return out, lse
    qf = q.detach().to("cpu", torch.float32)
    kf = k.detach().to("cpu", torch.float32)
    vf = v.detach().to("cpu", torch.float32)
    head_list = range(h) if heads is None else heads
    for bi in range(b):
        for hi in head_list:
            kk = kf[bi, :, hi // group, :]
            vv = vf[bi, :, hi // group, :]
            for r0 in range(0, sq, q_chunk):
                r1 = min(sq, r0 + q_chunk)
                s = (qf[bi, r0:r1, hi, :] @ kk.T) * scale
                if causal:
                    vis = _visible_mask(r1 - r0, sk, q_pos_offset + r0, k_pos_offset)
                    s = s.masked_fill(~vis, float("-inf"))
                row_lse = torch.logsumexp(s, dim=1) if sk > 0 else torch.full((r1 - r0,), float("-inf"))
                finite = torch.isfinite(row_lse)
                p = torch.exp(s - torch.where(finite, row_lse, torch.zeros_like(row_lse)).unsqueeze(1))
                p = torch.where(finite.unsqueeze(1), p, torch.zeros_like(p))
                out[bi, r0:r1, hi, :] = p @ vv
                lse[bi, hi, r0:r1] = row_lse
    return out, lse


def math_attention_backward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    dout: torch.Tensor,
    causal: bool = False,
    softmax_scale: float | None = None,
    q_pos_offset: int = 0,
    k_pos_offset: int = 0,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """fp32 gradients (dq, dk, dv) of softmax(scale Q K^T [+ mask]) V on the
    CPU by torch autograd, for the backward's parity tests.  K/V heads are
    shared by groups of query heads (GQA) exactly as in math_attention; rows
    with no visible key contribute nothing."""
    b, sq, h, d = q.shape
    hk = k.shape[2]
    group = h // hk
    scale = (1.0 / math.sqrt(d)) if softmax_scale is None else float(softmax_scale)
    qf = q.detach().to("cpu", torch.float32).requires_grad_(True)
    kf = k.detach().to("cpu", torch.float32).requires_grad_(True)
    vf = v.detach().to("cpu", torch.float32).requires_grad_(True)
    kr = kf.repeat_interleave(group, dim=2).permute(0, 2, 1, 3)
    vr = vf.repeat_interleave(group, dim=2).permute(0, 2, 1, 3)
    s = (qf.permute(0, 2, 1, 3) @ kr.transpose(-1, -2)) * scale
    if causal:
        vis = _visible_mask(sq, k.shape[1], q_pos_offset, k_pos_offset)
        s = s.masked_fill(~vis, float("-inf"))
    lse = torch.logsumexp(s, dim=-1, keepdim=True)
    p = torch.where(torch.isfinite(lse), torch.exp(s - torch.where(torch.isfinite(lse), lse, torch.zeros_like(lse))),
                    torch.zeros_like(s))
    o = (p @ vr).permute(0, 2, 1, 3)
    o.backward(dout.detach().to("cpu", torch.float32))
    return qf.grad, kf.grad, vf.grad


def tiled_reference_algorithm(
    q: np.ndarray | torch.Tensor,
    k: np.ndarray | torch.Tensor,
    v: np.ndarray | torch.Tensor,
    causal: bool = False,
    block: int = 64,
) -> np.ndarray:
    """The reference kernel's algorithm (kernel.cuh:130-297) in numpy.

    Inputs are fp16/bf16 torch tensors (or fp16 numpy arrays); the return
    value is O in fp32 holding values rounded to the input dtype, shape
    (b, s, h, d).  The reference requires sq % 64 == 0 and sk % 64 == 0
    (unpredicated tile copies, kernel.cuh:130,145,154,297).
    """
    dtype = q.dtype if isinstance(q, torch.Tensor) else torch.float16

    def f32(x):
        return x.detach().to("cpu", torch.float32).numpy() if isinstance(x, torch.Tensor) else x.astype(np.float32)

    def round_to_dtype(x: np.ndarray) -> np.ndarray:
        return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).to(torch.float32).numpy()

    qf, kf, vf = f32(q), f32(k), f32(v)
    b, sq, h, d = qf.shape
    sk = kf.shape[1]
    c = np.float32((1.0 / math.sqrt(d)) * LOG2E)  # softmax_scale_log2, flash_api.cpp:59-60
    out = np.zeros((b, sq, h, d), dtype=np.float32)
    n_blocks = (sk + block - 1) // block
    for bi in range(b):
        for hi in range(h):
            for m in range((sq + block - 1) // block):
                qt = qf[bi, m * block:(m + 1) * block, hi, :]
                rows = qt.shape[0]
                row_max = np.full((rows,), -np.inf, dtype=np.float32)
                row_sum = np.zeros((rows,), dtype=np.float32)
                acc = np.zeros((rows, d), dtype=np.float32)
                n_max = -(-((m + 1) * block) // block) if causal else n_blocks  # kernel.cuh:138-141
                for n in range(n_max):
                    kt = kf[bi, n * block:(n + 1) * block, hi, :]
                    vt = vf[bi, n * block:(n + 1) * block, hi, :]
                    s = (qt @ kt.T).astype(np.float32)
                    if causal and n * block >= m * block:  # diagonal tiles only
                        ri = m * block + np.arange(rows)[:, None]
                        ci = n * block + np.arange(s.shape[1])[None, :]
                        s = np.where(ci > ri, np.float32(-np.inf), s)
                    new_max = np.maximum(row_max, s.max(axis=1))
                    max_scaled = new_max * c
                    with np.errstate(invalid="ignore"):
                        rescale = np.exp2(row_max * c - max_scaled).astype(np.float32)
                    rescale = np.where(np.isnan(rescale), np.float32(0), rescale)
                    row_max = new_max
                    row_sum = row_sum * rescale
                    acc = acc * rescale[:, None]
                    p = np.exp2(s * c - max_scaled[:, None]).astype(np.float32)
                    row_sum = row_sum + p.sum(axis=1, dtype=np.float32)
                    acc = acc + round_to_dtype(p) @ vt
                inv = np.where(row_sum == 0, np.float32(1), np.float32(1) / row_sum)
                out[bi, m * block:m * block + rows, hi, :] = round_to_dtype(acc * inv[:, None])
    return out


def make_inputs(
    batch: int,
    seqlen: int,
    heads: int,
    head_dim: int,
    dtype: torch.dtype,
    seed: int = 0,
    seqlen_k: int | None = None,
    device: str | torch.device = "cpu",
    heads_k: int | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Seeded i.i.d. N(0,1) q, k, v drawn in fp32 in that order, then cast.

    Generation happens on the CPU so every device and every rank sees the
    same values for the same seed.
    """
    g = torch.Generator(device="cpu").manual_seed(seed)
    sk = seqlen if seqlen_k is None else seqlen_k
    hk = heads if heads_k is None else heads_k
    q = torch.randn((batch, seqlen, heads, head_dim), generator=g, dtype=torch.float32)
    k = torch.randn((batch, sk, hk, head_dim), generator=g, dtype=torch.float32)
    v = torch.randn((batch, sk, hk, head_dim), generator=g, dtype=torch.float32)
    return tuple(t.to(dtype).to(device) for t in (q, k, v))


def attention_flops(batch: int, seqlen_q: int, seqlen_k: int, heads: int, head_dim: int, causal: bool) -> float:
    """4*b*h*sq*sk*d, halved for causal (benchmark/bench.py:76 counts 4*b*h*s^2*d)."""
    f = 4.0 * batch * heads * seqlen_q * seqlen_k * head_dim
    return f / 2 if causal else f
