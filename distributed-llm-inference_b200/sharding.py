"""Sequence sharding across GPUs (one process per GPU).

The decode path partitions naturally: sequences are independent, so rank r
owns sequences [r*B//P, (r+1)*B//P) together with its own KV pools, block
tables and allocator, and the hot path needs no collective. torch.distributed
is used only around the measured region: a barrier, the max over ranks of
the device-timed duration, and a sum of output checksums.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Even, contiguous split: sequence i goes to rank i*world//batch."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    return rank * batch // world, (rank + 1) * batch // world


def _reduce(value: float, op, device) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(value: float, device="cpu") -> float:
    """Slowest rank's value (device-timed durations are reported this way)."""
    return _reduce(value, dist.ReduceOp.MAX if dist.is_available() else None, device)


def sum_over_ranks(value: float, device="cpu") -> float:
    return _reduce(value, dist.ReduceOp.SUM if dist.is_available() else None, device)


def barrier(device=None) -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        if device is not None and torch.device(device).type == "cuda":
            dist.barrier(device_ids=[torch.device(device).index])
        else:
            dist.barrier()
