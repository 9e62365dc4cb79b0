"""Attention over host-resident tensors, streamed through the GPU.

`flash_attn_func_host(q, k, v, causal)` takes q/k/v in pinned CPU memory and
returns O (and LSE) in CPU memory.  The batch is cut into chunks that move
through a ring of device buffers on three streams: chunk i+1 is copied
host->device while chunk i runs on the GPU and chunk i-1 is copied back.  PCIe
carries both directions at once, so the call costs about the host->device
transfer of q/k/v plus one chunk's compute and return copy, instead of the sum
of all copies and all compute.  (The reference API accepts CUDA tensors only;
this is an addition for callers whose tensors live on the host.)
"""
from __future__ import annotations

import threading

import torch

from flash_attention._C import forward_with_lse

# Chunks smaller than this cost more in per-chunk host work (three copies, a
# launch, events) than their overlap saves.
MIN_CHUNK_BYTES = 8 << 20


class _Workspace:
    """Per-device state kept across calls: the two side streams, the ring of
    device buffers (sized for the largest chunk seen with the current shapes)
    and its events.  A lock serialises calls on one device, since they share
    the buffers (the call blocks until done, so nothing is in flight between
    calls)."""

    def __init__(self, device: int):
        self.device = device
        self.lock = threading.Lock()
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        self.key = None
        self.rows = 0
        self.bufs: list[tuple[torch.Tensor, ...]] = []
        self.events = [[torch.cuda.Event() for _ in range(3)] for _ in range(3)]

    def ring(self, q: torch.Tensor, k: torch.Tensor, rows: int, slots: int):
        key = (q.dtype, tuple(q.shape[1:]), tuple(k.shape[1:]))
        if key != self.key or rows > self.rows or slots > len(self.bufs):
            self.bufs = []  # release the old ring before allocating the new one
            cu = torch.device("cuda", self.device)
            _, sq, h, _ = q.shape
            for _ in range(slots):
                qd = torch.empty((rows,) + tuple(q.shape[1:]), dtype=q.dtype, device=cu)
                kd = torch.empty((rows,) + tuple(k.shape[1:]), dtype=k.dtype, device=cu)
                vd = torch.empty_like(kd)
                od = torch.empty_like(qd)
                ld = torch.empty((rows, h, sq), dtype=torch.float32, device=cu)
                self.bufs.append((qd, kd, vd, od, ld))
            self.key, self.rows = key, rows
        return self.bufs


_workspaces: dict[int, _Workspace] = {}
_workspaces_lock = threading.Lock()


def _workspace(device: int) -> _Workspace:
    with _workspaces_lock:
        ws = _workspaces.get(device)
        if ws is None:
            ws = _workspaces[device] = _Workspace(device)
        return ws


def release_workspaces() -> None:
    """Free the device buffers kept between calls (they are re-made on demand)."""
    with _workspaces_lock:
        for ws in _workspaces.values():
            with ws.lock:
                ws.bufs, ws.key, ws.rows = [], None, 0


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
    min_chunk_bytes: int = MIN_CHUNK_BYTES,
    device: int | None = None,
):
    """Attention forward of pinned host tensors on the GPU, results on the host.

    q: (batch, seqlen_q, heads, head_dim), k/v: (batch, seqlen_k, heads_k,
    head_dim), fp16/bf16, contiguous, pinned.  `out` (like q) and `lse_out`
    ((batch, heads, seqlen_q) fp32) may be given as pinned host buffers;
    otherwise they are allocated (pinned).  The batch is split into at most
    `chunks` pieces of at least `min_chunk_bytes` of q/k/v each; a problem that
    makes one piece is copied in, computed and copied out on the current
    stream.  Device buffers are kept per device between calls
    (`release_workspaces` frees them).  Blocks until the host outputs are
    complete.
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
    per_batch = (q[0].numel() + 2 * k[0].numel()) * q.element_size()
    n_chunks = max(1, min(chunks, b, (b * per_batch) // max(1, min_chunk_bytes)))
    step = (b + n_chunks - 1) // n_chunks
    ranges = [(i, min(b, i + step)) for i in range(0, b, step)]
    want_lse = lse_out is not None
    ws = _workspace(dev)
    with torch.cuda.device(dev), ws.lock:
        comp = torch.cuda.current_stream(dev)
        if len(ranges) == 1:
            # one chunk: copies and kernel in order on the current stream
            qd, kd, vd, od, ld = (t[:b] for t in ws.ring(q, k, step, 1)[0])
            qd.copy_(q, non_blocking=True)
            kd.copy_(k, non_blocking=True)
            vd.copy_(v, non_blocking=True)
            forward_with_lse(qd, kd, vd, causal, out=od, lse_out=ld if want_lse else None, want_lse=want_lse)
            out.copy_(od, non_blocking=True)
            if want_lse:
                lse_out.copy_(ld, non_blocking=True)
            comp.synchronize()
            return (out, lse_out) if return_lse else out
        ring = min(3, len(ranges))
        bufs = ws.ring(q, k, step, ring)
        h2d, d2h = ws.h2d, ws.d2h
        # the ring's memory comes from the allocator on the current stream:
        # earlier work there may still use it, so the side stream waits for it
        h2d.wait_stream(comp)
        in_ready, computed, copied_back = (list(e) for e in zip(*ws.events[:ring]))
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
            forward_with_lse(qd, kd, vd, causal, out=od, lse_out=ld if want_lse else None, want_lse=want_lse)
            computed[slot].record(comp)
            with torch.cuda.stream(d2h):
                d2h.wait_event(computed[slot])
                out[b0:b1].copy_(od, non_blocking=True)
                if want_lse:
                    lse_out[b0:b1].copy_(ld, non_blocking=True)
                copied_back[slot].record(d2h)
        d2h.synchronize()
        comp.synchronize()
    return (out, lse_out) if return_lse else out
