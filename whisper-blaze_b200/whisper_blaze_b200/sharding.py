"""Batch (data) partitioning of encoder inference across the GPUs of one node.

Chunks (30 s windows, 1500 frames each) are independent through the encoder,
so ranks split the batch into contiguous slices, run the whole stack on their
slice with no communication, and exchange data exactly once: an
all_gather_into_tensor of the outputs over NCCL (NVLink/NVSwitch) at the end.
No collective touches a GEMM. One process per GPU (torchrun); the same code
runs on CPU `gloo` ranks for tests.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous slice; the first total % world ranks get one extra."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if total < 0:
        raise ValueError("total must be >= 0")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def max_shard(total: int, world: int) -> int:
    return (total + world - 1) // world


def gather_batch(local: torch.Tensor, total: int, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """All-gather per-rank batch slices [b_r, ...] into the full [total, ...] on every rank.

    Slices may differ by one element along dim 0 (shard_bounds); they are
    padded to the largest slice for the collective and the padding is
    dropped afterwards, preserving rank order.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    start, stop = shard_bounds(total, world, rank)
    if local.shape[0] != stop - start:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, expected {stop - start}")
    per = max_shard(total, world)
    if local.shape[0] != per:
        padded = torch.zeros((per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
        padded[: local.shape[0]] = local
        local = padded
    full = torch.empty((per * world,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(full, local.contiguous(), group=group)
    if per * world == total:
        return full
    parts = []
    for r in range(world):
        s, e = shard_bounds(total, world, r)
        parts.append(full[r * per: r * per + (e - s)])
    return torch.cat(parts, 0)


def run_sharded(fn: Callable[[torch.Tensor], torch.Tensor], full_batch: torch.Tensor,
                group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """Run `fn` on this rank's slice of `full_batch` (dim 0) and gather all results."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    total = full_batch.shape[0]
    start, stop = shard_bounds(total, world, rank)
    local_out = fn(full_batch[start:stop])
    return gather_batch(local_out, total, group)
