"""Sequence sharding over ranks and the end-of-run reduction (no collective on
the hot path: sequences share nothing).

shard_range      contiguous share of n sequences for one rank
reduce_over_ranks  max of times, sum of counters over the process group (the
                 only collectives of a run, after the timed region)
Works with any torch.distributed backend (nccl on GPUs, gloo on CPU); with one
rank (or no process group) it is the identity.
"""
from __future__ import annotations

import torch


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's sequences: n split into world contiguous shares,
    the first n % world ranks one larger."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def reduce_over_ranks(times, counters, device: torch.device | str = "cpu"):
    """(max over ranks of each time, sum over ranks of each counter).  Every rank
    calls it once, with the same list lengths."""
    import torch.distributed as dist
    times = [float(t) for t in times]
    counters = [float(c) for c in counters]
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return times, counters
    t = torch.tensor(times, dtype=torch.float64, device=device)
    c = torch.tensor(counters, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(c, op=dist.ReduceOp.SUM)
    return t.tolist(), c.tolist()
