"""Image sharding across ranks and the ordered gather of pooled embeddings.

The batched towers are data-parallel: every GPU holds a full weight replica
and encodes its own images, and the only exchange is collecting the 1152-d
pooled embeddings (one all-gather, the reference's scoring input) on every
rank in the caller's image order.  Works with any torch.distributed backend
(NCCL on the GPU box, gloo for the CPU tests).
"""
from __future__ import annotations

from typing import Sequence


def shard_images(grids: Sequence[tuple[int, int]], rank: int, world: int) -> list[int]:
    """Length-balanced deal: images sorted by patch count (largest first, ties
    by index) are dealt round-robin; returns this rank's image indices in
    ascending order.  Every image lands on exactly one rank and per-rank token
    counts differ by at most one image's worth."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world {rank}/{world}")
    order = sorted(range(len(grids)), key=lambda i: (-grids[i][0] * grids[i][1], i))
    return sorted(order[rank::world])


def shard_rows(n: int, rank: int, world: int) -> range:
    """Contiguous split of n items (prompts) over ranks, sizes differing by at most one."""
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def per_rank_capacity(n: int, world: int) -> int:
    return (n + world - 1) // world


def gather_in_order(local, mine: Sequence[int], n_total: int, group=None):
    """All-gather each rank's embeddings (local: [len(mine), H] tensor on this
    rank's device) and return the [n_total, H] tensor in the original order on
    every rank.  `mine` are this rank's original indices (shard_images or
    shard_rows), as a sequence or as an int64 tensor already on the device
    (which keeps the call free of host synchronisation)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    cap = per_rank_capacity(n_total, world)
    H = local.shape[1]
    dev = local.device
    buf = torch.zeros((cap, H), dtype=local.dtype, device=dev)
    n_mine = int(mine.numel()) if isinstance(mine, torch.Tensor) else len(mine)
    buf[:n_mine] = local[:n_mine]
    idx = torch.full((cap,), -1, dtype=torch.int64, device=dev)
    idx[:n_mine] = mine if isinstance(mine, torch.Tensor) else torch.as_tensor(list(mine), dtype=torch.int64,
                                                                                   device=dev)
    all_buf = torch.empty((world * cap, H), dtype=local.dtype, device=dev)
    all_idx = torch.empty((world * cap,), dtype=torch.int64, device=dev)
    dist.all_gather_into_tensor(all_buf, buf, group=group)
    dist.all_gather_into_tensor(all_idx, idx, group=group)
    # padding rows carry index -1: send them to a scratch row past the end
    dst = torch.where(all_idx >= 0, all_idx, torch.full_like(all_idx, n_total))
    out = torch.empty((n_total + 1, H), dtype=local.dtype, device=dev)
    out.index_copy_(0, dst, all_buf)
    return out[:n_total]
