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
  present every output row is exact: no LSE merge is needed.  Callers that
  process key chunks one at a time instead can merge their partial
  (O, LSE) pairs with `flash_attention._C.lse_merge`.
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


def _kernel_attn(q, k, v, causal, q_pos_offset, out, lse_out):
    from flash_attention._C import forward_with_lse

    return forward_with_lse(q, k, v, causal, q_pos_offset=q_pos_offset, out=out, lse_out=lse_out)


def context_parallel_attention(
    q_local: torch.Tensor,
    k_local: torch.Tensor,
    v_local: torch.Tensor,
    causal: bool = True,
    group=None,
    attn_fn: AttnFn | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Attention of this rank's zigzag query chunks against the whole sequence.

    q_local/k_local/v_local: (b, 2c, h, d) = zigzag_shard of the full tensors.
    Returns (o_local (b, 2c, h, d), lse_local (b, h, 2c) fp32) in the same
    zigzag order.  `attn_fn(q, k, v, causal, q_pos_offset, out, lse_out)` is
    the per-chunk attention; the default is the sm_100a kernel.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    fn = attn_fn or _kernel_attn
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
