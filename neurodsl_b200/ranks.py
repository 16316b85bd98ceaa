"""Rank bookkeeping for running the hot path on several GPUs of one node.

Attention prefill and decode are independent per (batch, head): a job either
gives each rank its own batch (weak scaling: every rank runs the full
per-GPU workload) or splits one batch's (batch, head) units into contiguous
shards (strong scaling).  Neither needs a collective on the data path; the
only collectives are the barrier around the timed region and the max of the
ranks' times, taken here with torch.distributed (NCCL on GPUs, gloo on CPU).
"""
from __future__ import annotations

import os
from typing import Tuple


def dist_env() -> Tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_range(n_units: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, end) of n_units for `rank`; sizes differ by at most one."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(n_units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(x: float, device=None) -> float:
    """Max of a per-rank scalar (e.g. elapsed milliseconds) over the group;
    the identity when torch.distributed is not initialised."""
    import torch
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(work_per_rank: float, world: int, seconds_max: float) -> float:
    """Whole-job throughput: every rank's work divided by the slowest rank's time."""
    if seconds_max <= 0:
        raise ValueError("elapsed time must be positive")
    return work_per_rank * world / seconds_max
