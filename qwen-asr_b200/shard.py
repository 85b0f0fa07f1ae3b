"""Data-parallel placement of independent utterances over ranks.

Utterances (and streams) are independent, so a multi-GPU run is one process
per GPU, each owning a contiguous block of utterances, with no collective on
the data path. The only collectives are for timing: a barrier before the timed
region and the max over ranks of the measured durations (the slowest rank
defines the job's time).
"""
from __future__ import annotations


def shard_range(n_items: int, world: int, rank: int) -> tuple[int, int]:
    """[first, first+count) of rank's contiguous block; sizes differ by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    base, extra = divmod(n_items, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def max_over_ranks(values, device=None):
    """Element-wise max of a list of floats over all ranks (identity without a
    process group). Works with the gloo (CPU tensors) and nccl backends."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def sum_over_ranks(values, device=None):
    """Element-wise sum of a list of floats over all ranks (identity without a
    process group): counts of work done, for whole-job rates."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()
