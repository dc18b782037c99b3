"""Data-parallel layout of the chains over several GPUs (one process per GPU).

Independent sequences are split across ranks with the weights replicated on
every rank, so the data path needs no collective: each rank runs its own
device-resident chain on its slice of the global batch. The split is the
contiguous ownership split the reference's isolate pool uses for columns
(`GemmPool`, lib/src/parallel_pool.dart:236-260: `n ~/ workers` each, the
first `n % workers` workers one more), applied to sequences. Collectives
appear only around the timed region: a barrier, and the slowest rank's time
(`max_over_ranks`) for whole-job throughput.
"""
from __future__ import annotations

import numpy as np


def shard(total: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank `rank`'s contiguous slice of `total` items."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request: total={total} world={world} rank={rank}")
    base, rem = divmod(total, world)
    count = base + (1 if rank < rem else 0)
    start = rank * base + min(rank, rem)
    return start, count


def local_slice(global_rows, world: int, rank: int):
    """This rank's rows of a global batch (first axis)."""
    start, count = shard(len(global_rows), world, rank)
    return global_rows[start:start + count]


def max_over_ranks(value: float, dist=None, device=None) -> float:
    """The largest `value` over all ranks (every rank gets it); the value
    itself when torch.distributed is not initialised."""
    if dist is None or not dist.is_available() or not dist.is_initialized():
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_slices(local_rows, dist=None) -> np.ndarray:
    """Concatenates every rank's rows in rank order (for checks and reports;
    not on the data path)."""
    if dist is None or not dist.is_available() or not dist.is_initialized():
        return np.asarray(local_rows)
    parts = [None] * dist.get_world_size()
    dist.all_gather_object(parts, np.asarray(local_rows))
    return np.concatenate(parts, axis=0)


def job_throughput(units_per_rank: list[int] | int, world: int, slowest_ms: float) -> float:
    """Whole-job units per second: every rank's units over the slowest rank's
    device time."""
    total = sum(units_per_rank) if isinstance(units_per_rank, (list, tuple)) else units_per_rank * world
    return total / (slowest_ms / 1e3)
