"""Batch sharding of soft Smith-Waterman problems across processes.

The problems of a batch are independent (no exchange inside a DP), so the
multi-GPU path is: one process per GPU, each rank runs the operators on a
contiguous slice of the batch, and only the per-problem values are gathered.
Marginals and gradients stay on the rank that computed them.

These helpers hold that host-side logic; they work with any
``torch.distributed`` backend (NCCL on GPUs, gloo for CPU tests).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_bounds(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous slice [start, stop) of a batch of `batch` problems for `rank`.

    The first ``batch % world`` ranks take one extra problem, so shard sizes
    differ by at most one and every problem is owned by exactly one rank.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if batch < 0:
        raise ValueError(f"batch must be non-negative, got {batch}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_values(local: torch.Tensor, batch: int, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather per-problem values [shard] from every rank into [batch], in rank order.

    Shards may differ in size by one (see `shard_bounds`): each rank pads its
    shard to the largest size for one fixed-size all-gather, and the padding
    is dropped afterwards.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_bounds(batch, world, rank)
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds {local.shape[0]} values, its shard has {hi - lo}")
    width = -(-batch // world) if batch else 0
    padded = local.new_zeros(width)
    padded[: local.shape[0]] = local
    out = local.new_empty(world * width)
    dist.all_gather_into_tensor(out, padded, group=group)
    parts = []
    for r in range(world):
        a, b = shard_bounds(batch, world, r)
        parts.append(out[r * width: r * width + (b - a)])
    return torch.cat(parts) if parts else out[:0]


def soft_sw_sharded(scores: torch.Tensor, gap=-1.0, temperature=1.0, lengths=None,
                    group: Optional[dist.ProcessGroup] = None):
    """`soft_sw` on this rank's slice of a global batch.

    `scores` / `lengths` are the full global batch (as every rank would see
    it after a seeded generation or a broadcast); the rank computes its
    slice and returns (values of the whole batch [B], its own SWResult,
    (start, stop)).
    """
    from .sw import soft_sw

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    lo, hi = shard_bounds(scores.shape[0], world, rank)
    res = soft_sw(scores[lo:hi], gap=gap, temperature=temperature,
                  lengths=None if lengths is None else lengths[lo:hi])
    values = gather_values(res.value.detach(), scores.shape[0], group)
    return values, res, (lo, hi)
