"""Multi-GPU execution of the attention forward: one process per GPU.

Two modes (the reference is single-GPU; these are additions):

* **batch x head sharding** (`shard_units`): the (batch, head) units of an
  attention call are independent, so each rank computes a contiguous slice of
  them with no data-path collective.

* **zigzag context parallelism** (`context_parallel_attention`) for long
  causal sequences: the sequence is cut into 2W chunks; rank r owns chunks r
  and 2W-1-r of Q, K and V, which gives every rank the same amount of causal
  work.  K and V are all-gathered (NCCL over NVLink on GPUs, gloo on CPU in the
  tests) into sequence order, and each local query chunk is attended against
  the gathered keys with its global position passed to the kernel
  (q_pos_offset), so the causal mask is applied on global positions and the
  kernel only visits the key blocks a chunk can see.  With the whole K/V
  present every output row is exact: no LSE merge is needed.  The
  overlapped variant hides the gather behind compute by attending each chunk
  to the keys already present first and merging fp32 partial (O, LSE) pairs
  with the library's LSE-merge kernel (`flash_attention._C.lse_merge`).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist


def shard_units(batch: int, heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, end) range of the batch*heads units owned by `rank`.

    Units are numbered batch-major (u = b*heads + h); the first `n % world`
    ranks get one extra unit.
    """
    n = batch * heads
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def zigzag_chunks(seqlen: int, world: int, rank: int) -> tuple[tuple[int, int], tuple[int, int]]:
    """Global [start, end) of the two sequence chunks rank `rank` owns."""
    if seqlen % (2 * world) != 0:
        raise ValueError(f"seqlen {seqlen} must be divisible by 2*world = {2 * world}")
    c = seqlen // (2 * world)
    a, b = rank, 2 * world - 1 - rank
    return (a * c, (a + 1) * c), (b * c, (b + 1) * c)


def zigzag_shard(x: torch.Tensor, world: int, rank: int, dim: int = 1) -> torch.Tensor:
    """The rank's two chunks of `x` along `dim`, concatenated (a contiguous copy)."""
    (a0, a1), (b0, b1) = zigzag_chunks(x.size(dim), world, rank)
    return torch.cat([x.narrow(dim, a0, a1 - a0), x.narrow(dim, b0, b1 - b0)], dim=dim).contiguous()


def zigzag_unshard(parts: list[torch.Tensor], dim: int = 1) -> torch.Tensor:
    """Inverse of zigzag_shard over all ranks' local tensors (test helper)."""
    world = len(parts)
    c = parts[0].size(dim) // 2
    chunks: list[torch.Tensor | None] = [None] * (2 * world)
    for r, t in enumerate(parts):
        chunks[r] = t.narrow(dim, 0, c)
        chunks[2 * world - 1 - r] = t.narrow(dim, c, c)
    return torch.cat(chunks, dim=dim)


def gather_zigzag(local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather zigzag-sharded (b, 2c, h, d) tensors into (b, 2*world*c, h, d)
    in sequence order.

    The first-half chunks (r = 0..W-1) arrive in rank order, which is already
    sequence order; the second-half chunks (2W-1-r) arrive reversed and are
    put back in order with one copy.
    """
    world = dist.get_world_size(group)
    b, two_c, h, d = local.shape
    c = two_c // 2
    first = local[:, :c].contiguous()
    second = local[:, c:].contiguous()
    # gathered as a concatenation along dim 0 (the form every backend accepts)
    g1 = torch.empty((world * b, c, h, d), dtype=local.dtype, device=local.device)
    g2 = torch.empty_like(g1)
    dist.all_gather_into_tensor(g1, first, group=group)
    dist.all_gather_into_tensor(g2, second, group=group)
    g1 = g1.view(world, b, c, h, d)
    g2 = g2.view(world, b, c, h, d)
    out = torch.empty((b, 2 * world * c, h, d), dtype=local.dtype, device=local.device)
    # chunk r -> position r; chunk 2W-1-r -> position 2W-1-r
    out[:, : world * c].view(b, world, c, h, d).copy_(g1.permute(1, 0, 2, 3, 4))
    out[:, world * c :].view(b, world, c, h, d).copy_(g2.flip(0).permute(1, 0, 2, 3, 4))
    return out


AttnFn = Callable[..., tuple[torch.Tensor, torch.Tensor]]
MergeFn = Callable[..., None]


def _kernel_attn(q, k, v, causal, q_pos_offset, out, lse_out, k_pos_offset=0):
    from flash_attention._C import forward_with_lse

    return forward_with_lse(q, k, v, causal, q_pos_offset=q_pos_offset, k_pos_offset=k_pos_offset, out=out,
                            lse_out=lse_out)


def _kernel_merge(o_parts, lse_parts, o_out, lse_out):
    """Merge fp32 partials o (b, c, h, d) / lse (b, h, c) into o_out (b, c, h, d)
    and lse_out (b, h, c) with the library's merge kernel, one batch at a time."""
    from flash_attention._C import lse_merge

    for bi in range(o_out.size(0)):
        lse_tmp = torch.empty((o_out.size(2), o_out.size(1)), dtype=torch.float32, device=o_out.device)
        lse_merge([p[bi] for p in o_parts], [p[bi] for p in lse_parts], o_out[bi], lse_tmp)
        lse_out[bi].copy_(lse_tmp)


def context_parallel_attention(
    q_local: torch.Tensor,
    k_local: torch.Tensor,
    v_local: torch.Tensor,
    causal: bool = True,
    group=None,
    attn_fn: AttnFn | None = None,
    overlap: bool = False,
    merge_fn: MergeFn | None = None,
    workspace: dict | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention of this rank's zigzag query chunks against the whole sequence.

    q_local/k_local/v_local: (b, 2c, h, d) = zigzag_shard of the full tensors.
    Returns (o_local (b, 2c, h, d), lse_local (b, h, 2c) fp32) in the same
    zigzag order.  `attn_fn(q, k, v, causal, q_pos_offset, out, lse_out,
    k_pos_offset=0)` is the per-chunk attention; the default is the sm_100a
    kernel.

    overlap=False gathers all of K and V, then runs each query chunk once
    against it.  overlap=True (causal only) hides the gather behind compute:
    the gather is issued in two asynchronous halves, each query chunk is
    first attended against the keys this rank already holds, then against
    each half as it arrives, producing fp32 partial (O, LSE) pairs that
    `merge_fn` (default: the library's LSE-merge kernel) combines.

    `workspace`: an optional dict the overlapped schedule keeps its gather
    and partial buffers in between calls, so back-to-back calls allocate
    nothing (the buffers are reused in stream order).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    fn = attn_fn or _kernel_attn
    if overlap and causal:
        return _cp_overlapped(q_local, k_local, v_local, world, rank, group, fn, merge_fn or _kernel_merge,
                              workspace)
    k_full = gather_zigzag(k_local, group)
    v_full = gather_zigzag(v_local, group)
    b, two_c, h, _ = q_local.shape
    c = two_c // 2
    o_local = torch.empty_like(q_local)
    lse_local = torch.empty((b, h, two_c), dtype=torch.float32, device=q_local.device)
    for i, chunk in enumerate((rank, 2 * world - 1 - rank)):
        fn(
            q_local[:, i * c : (i + 1) * c],
            k_full,
            v_full,
            causal,
            chunk * c,
            o_local[:, i * c : (i + 1) * c],
            lse_local[:, :, i * c : (i + 1) * c],
        )
    return o_local, lse_local


def _in_sequence_order(g: torch.Tensor, world: int, b: int, idx: list[int]) -> torch.Tensor:
    """Chunks `idx` (in that order) of an all-gathered (world*b, c, h, d)
    buffer as one (b, len(idx)*c, h, d) key tensor; a view when it can be."""
    _, c, h, d = g.shape
    gv = g.view(world, b, c, h, d)
    if b == 1 and idx == list(range(idx[0], idx[0] + len(idx))):
        return gv[idx[0] : idx[0] + len(idx)].view(1, len(idx) * c, h, d)
    sel = gv[torch.tensor(idx, device=g.device)]
    return sel.permute(1, 0, 2, 3, 4).reshape(b, len(idx) * c, h, d)


def _buffer(workspace, name, shape, dtype, device):
    if workspace is None:
        return torch.empty(shape, dtype=dtype, device=device)
    t = workspace.get(name)
    if t is None or t.shape != torch.Size(shape) or t.dtype != dtype or t.device != device:
        t = workspace[name] = torch.empty(shape, dtype=dtype, device=device)
    return t


def _cp_overlapped(q_local, k_local, v_local, world, rank, group, fn, merge_fn, workspace=None):
    b, two_c, h, d = q_local.shape
    c = two_c // 2
    dev = q_local.device
    pa, pb = rank, 2 * world - 1 - rank  # sequence chunk positions of the two local query chunks
    first_k, first_v = k_local[:, :c].contiguous(), v_local[:, :c].contiguous()
    second_k, second_v = k_local[:, c:].contiguous(), v_local[:, c:].contiguous()
    # Chunk positions 0..W-1 arrive in rank order (first halves), positions
    # 2W-1..W in rank order (second halves).  Both gathers are in flight while
    # the local keys are processed.
    gk1, gv1, gk2, gv2 = (_buffer(workspace, n, (world * b, c, h, d), k_local.dtype, dev)
                          for n in ("gk1", "gv1", "gk2", "gv2"))
    works = [dist.all_gather_into_tensor(out, inp, group=group, async_op=True)
             for out, inp in ((gk1, first_k), (gv1, first_v), (gk2, second_k), (gv2, second_v))]

    qa, qb = q_local[:, :c], q_local[:, c:]
    parts_a, parts_b = [], []

    def part(q, k, v, q_pos, k_pos, parts):
        tag = f"{len(parts_a)}.{len(parts_b)}.{q_pos}"
        o = _buffer(workspace, "o" + tag, tuple(q.shape), torch.float32, dev)
        lse = _buffer(workspace, "l" + tag, (b, h, q.size(1)), torch.float32, dev)
        fn(q, k, v, True, q_pos * c, o, lse, k_pos_offset=k_pos * c)
        parts.append((o, lse))

    # 1. keys already here: each chunk's own diagonal block
    part(qa, first_k, first_v, pa, pa, parts_a)
    part(qb, second_k, second_v, pb, pb, parts_b)
    # 2. first halves (positions 0..W-1): chunk a needs [0, a), chunk b all of them
    works[0].wait()
    works[1].wait()
    if pa > 0:
        idx = list(range(pa))
        part(qa, _in_sequence_order(gk1, world, b, idx), _in_sequence_order(gv1, world, b, idx), pa, 0, parts_a)
    idx = list(range(world))
    part(qb, _in_sequence_order(gk1, world, b, idx), _in_sequence_order(gv1, world, b, idx), pb, 0, parts_b)
    # 3. second halves: chunk b needs positions W..pb-1 = gathered slots 2W-1-p
    works[2].wait()
    works[3].wait()
    if pb > world:
        idx = [2 * world - 1 - p for p in range(world, pb)]
        part(qb, _in_sequence_order(gk2, world, b, idx), _in_sequence_order(gv2, world, b, idx), pb, world, parts_b)

    o_local = torch.empty_like(q_local)
    lse_local = torch.empty((b, h, two_c), dtype=torch.float32, device=dev)
    for i, parts in enumerate((parts_a, parts_b)):
        merge_fn([p[0] for p in parts], [p[1] for p in parts], o_local[:, i * c : (i + 1) * c],
                 lse_local[:, :, i * c : (i + 1) * c])
    return o_local, lse_local
