"""Batch sharding across GPUs (one process per GPU, no data-path collective).

The CNN configs shard by batch: rank r of W owns images [r*n, (r+1)*n) of the
global batch and runs an independent replica of the graph (weights uploaded
once per GPU).  Ranks meet only outside the timed work: a barrier around the
timed region and one MAX reduction of each rank's device time, so the
reported time is the slowest rank's.
"""
from __future__ import annotations

import os


def dist_env() -> tuple[int, int, int]:
    """(world_size, rank, local_rank) from the torchrun environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [start, stop) of the global batch owned by `rank` (contiguous,
    sizes differ by at most one when the batch does not divide evenly)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_seed(base_seed: int, rank: int) -> int:
    """Seed of rank's synthetic input shard (independent per rank)."""
    return base_seed + rank


def max_over_ranks(value: float, device: str = "cpu") -> float:
    """MAX of a per-rank scalar over the process group (identity when the
    group is not initialised)."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def throughput(images_per_rank: int, world: int, max_ms_per_step: float) -> float:
    """Whole-job images/s: all ranks' images over the slowest rank's time."""
    return world * images_per_rank / (max_ms_per_step / 1e3)
