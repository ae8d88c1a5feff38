"""Replica data parallelism for the decode path: one process per GPU.

The decode step has no exchange between sequences (the reference serves every request
on one device, speech_serving/phase_aware_scheduler.py:1109-1149), so N GPUs run N
independent replicas.  Requests are dealt round-robin to ranks, nothing crosses NVLink
on the data path, and the only collectives are the timing barrier and the max over ranks
of the timed interval.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple, TypeVar

import torch
import torch.distributed as dist

T = TypeVar("T")


def shard(items: Sequence[T], world: int, rank: int) -> List[T]:
    """Round-robin share of ``items`` for ``rank`` (every item goes to exactly one rank)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    return list(items[rank::world])


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous share [lo, hi) of n units; shares differ in size by at most one."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    return n * rank // world, n * (rank + 1) // world


def _reduce_device() -> torch.device:
    if dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def max_over_ranks(value: float) -> float:
    """Max of a per-rank float over the default group (the value itself without one)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_reduce_device())
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_reduce_device())
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def whole_job_rate(units_all_ranks: float, ms_max: float) -> float:
    """Units per second of the whole job: units processed by all ranks over the slowest
    rank's timed interval."""
    if ms_max <= 0:
        raise ValueError("timed interval must be positive")
    return units_all_ranks / (ms_max / 1e3)


def gather_over_ranks(value: float) -> List[float]:
    """Every rank's float, in rank order (a one-element list without a group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(value)]
    n = dist.get_world_size()
    t = torch.zeros(n, dtype=torch.float64, device=_reduce_device())
    t[dist.get_rank()] = float(value)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return [float(x) for x in t.tolist()]
