"""Attention over host-resident tensors, streamed through the GPU.

`flash_attn_func_host(q, k, v, causal)` takes q/k/v in pinned CPU memory and
returns O (and LSE) in CPU memory.  The batch is cut into chunks that move
through a small ring of device buffers on three streams: chunk i+1 is copied
host->device while chunk i runs on the GPU and chunk i-1 is copied back.  PCIe
carries both directions at once, so the call costs about the host->device
transfer of q/k/v plus one chunk's compute and return copy, instead of the sum
of all copies and all compute.  (The reference API accepts CUDA tensors only;
this is an addition for callers whose tensors live on the host.)
"""
from __future__ import annotations

import torch

from flash_attention._C import forward_with_lse

_streams: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream]] = {}


def _side_streams(device: int) -> tuple[torch.cuda.Stream, torch.cuda.Stream]:
    if device not in _streams:
        _streams[device] = (torch.cuda.Stream(device), torch.cuda.Stream(device))
    return _streams[device]


def _check_host(name: str, t: torch.Tensor) -> None:
    if t.is_cuda:
        raise RuntimeError(f"{name} must be a CPU tensor (use flash_attn_func for CUDA tensors)")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if not t.is_pinned():
        raise RuntimeError(f"{name} must be in pinned host memory (tensor.pin_memory())")


def flash_attn_func_host(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    *,
    return_lse: bool = False,
    out: torch.Tensor | None = None,
    lse_out: torch.Tensor | None = None,
    chunks: int = 16,
    device: int | None = None,
):
    """Attention forward of pinned host tensors on the GPU, results on the host.

    q: (batch, seqlen_q, heads, head_dim), k/v: (batch, seqlen_k, heads_k,
    head_dim), fp16/bf16, contiguous, pinned.  `out` (like q) and `lse_out`
    ((batch, heads, seqlen_q) fp32) may be given as pinned host buffers;
    otherwise they are allocated (pinned).  The batch is split into at most
    `chunks` pieces.  Blocks until the host outputs are complete.
    Returns o, or (o, lse) if return_lse.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_host(name, t)
    if out is not None:
        _check_host("out", out)
        if out.shape != q.shape or out.dtype != q.dtype:
            raise RuntimeError("out must have q's shape and dtype")
    b, sq, h, d = q.shape
    if lse_out is not None:
        _check_host("lse_out", lse_out)
        if lse_out.shape != (b, h, sq) or lse_out.dtype != torch.float32:
            raise RuntimeError("lse_out must be (batch, heads, seqlen_q) fp32")
    if out is None:
        out = torch.empty_like(q, pin_memory=True)
    if lse_out is None and return_lse:
        lse_out = torch.empty((b, h, sq), dtype=torch.float32, pin_memory=True)
    if b == 0 or q.numel() == 0:
        return (out, lse_out) if return_lse else out

    dev = torch.cuda.current_device() if device is None else int(device)
    with torch.cuda.device(dev):
        comp = torch.cuda.current_stream(dev)
        h2d, d2h = _side_streams(dev)
        n_chunks = max(1, min(chunks, b))
        step = (b + n_chunks - 1) // n_chunks
        ranges = [(i, min(b, i + step)) for i in range(0, b, step)]
        ring = min(3, len(ranges))
        cu = torch.device("cuda", dev)
        bufs = []
        for _ in range(ring):
            qd = torch.empty((step,) + tuple(q.shape[1:]), dtype=q.dtype, device=cu)
            kd = torch.empty((step,) + tuple(k.shape[1:]), dtype=k.dtype, device=cu)
            vd = torch.empty((step,) + tuple(v.shape[1:]), dtype=v.dtype, device=cu)
            od = torch.empty_like(qd)
            ld = torch.empty((step, h, sq), dtype=torch.float32, device=cu)
            for t in (qd, kd, vd, od, ld):
                t.record_stream(h2d)
                t.record_stream(d2h)
            bufs.append((qd, kd, vd, od, ld))
        in_ready = [torch.cuda.Event() for _ in range(ring)]
        computed = [torch.cuda.Event() for _ in range(ring)]
        copied_back = [torch.cuda.Event() for _ in range(ring)]
        for i, (b0, b1) in enumerate(ranges):
            slot, n = i % ring, b1 - b0
            qd, kd, vd, od, ld = (t[:n] for t in bufs[slot])
            with torch.cuda.stream(h2d):
                if i >= ring:
                    h2d.wait_event(computed[slot])  # the kernel of chunk i-ring has read this slot
                qd.copy_(q[b0:b1], non_blocking=True)
                kd.copy_(k[b0:b1], non_blocking=True)
                vd.copy_(v[b0:b1], non_blocking=True)
                in_ready[slot].record(h2d)
            comp.wait_event(in_ready[slot])
            if i >= ring:
                comp.wait_event(copied_back[slot])  # chunk i-ring's output has left this slot
            forward_with_lse(qd, kd, vd, causal, out=od, lse_out=ld if lse_out is not None else None,
                             want_lse=lse_out is not None)
            computed[slot].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(computed[slot])
                out[b0:b1].copy_(od, non_blocking=True)
                if lse_out is not None:
                    lse_out[b0:b1].copy_(ld, non_blocking=True)
                copied_back[slot].record(d2h)
        d2h.synchronize()
        comp.synchronize()
    return (out, lse_out) if return_lse else out
