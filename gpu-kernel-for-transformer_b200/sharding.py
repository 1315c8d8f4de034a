"""Batch sharding across GPUs (one process per GPU).

Sequences are independent in this model (attention never crosses the batch
dimension; every other op is per token), so the forward shards over the batch
with no collective: each rank runs its contiguous slice and the outputs are
gathered once at the end if one rank needs them all. This replaces the
reference's single-GPU batch chunking (batch_chunk_runner.py:49-154), whose
exactness rests on the same independence.
"""

from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of `total` sequences for `rank` of `world`;
    shard sizes differ by at most one, and ranks past `total` get empty shards
    (a batch of 4 on 8 GPUs leaves four ranks idle)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("need total >= 0, world > 0 and 0 <= rank < world")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_shards(local: torch.Tensor, total: int, dst: int = 0,
                  group: Optional[dist.ProcessGroup] = None) -> Optional[torch.Tensor]:
    """Gather every rank's shard (first dim) to rank `dst` in rank order.

    Shards may differ in size (see shard_range); they are padded to the
    largest for the collective and trimmed afterwards. Returns the
    concatenated [total, ...] tensor on `dst`, None elsewhere. Every rank must
    call it (it is one collective)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    sizes = [shard_range(total, world, r) for r in range(world)]
    longest = max(stop - start for start, stop in sizes)
    start, stop = sizes[rank]
    if local.shape[0] != stop - start:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard is {stop - start}")
    padded = local.new_zeros((longest,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    bufs: Optional[List[torch.Tensor]] = (
        [torch.empty_like(padded) for _ in range(world)] if rank == dst else None
    )
    dist.gather(padded, bufs, dst=dst, group=group)
    if rank != dst:
        return None
    return torch.cat([b[: e - s] for b, (s, e) in zip(bufs, sizes)], dim=0)
