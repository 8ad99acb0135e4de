"""Batch sharding of the recurrence across ranks (one process per GPU).

Lanes (b, h) are independent, so the path shards over batch rows with all H
heads of a row on one rank.  There is no collective on the data path; the
helpers below only compute shard ranges and gather results for verification.
"""
from __future__ import annotations

from typing import List, Tuple

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of n items for `rank` of `world` (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad world/rank {world}/{rank}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def checksum(t: torch.Tensor) -> torch.Tensor:
    """Order-sensitive fp64 checksum (sum and weighted sum) of a tensor, as a [2] tensor."""
    x = t.detach().double().flatten()
    w = torch.arange(1, x.numel() + 1, dtype=torch.float64, device=x.device) / max(x.numel(), 1)
    return torch.stack([x.sum(), (x * w).sum()])


def gather_to_rank0(t: torch.Tensor, group=None) -> List[torch.Tensor]:
    """Gathers one tensor per rank onto rank 0 (all ranks must call; shapes may differ
    only in dim 0).  Returns the list on rank 0 and [] elsewhere."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = torch.tensor([t.shape[0]], dtype=torch.int64, device=t.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    mx = int(max(s.item() for s in sizes))
    pad = torch.zeros((mx,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    if rank != 0:
        return []
    return [b[: int(s.item())] for b, s in zip(bufs, sizes)]
