"""Sequence sharding across GPUs (one process per GPU).

The decode path partitions naturally: sequences are independent, so each
rank owns a set of whole sequences together with its own KV pools, block
tables and allocator, and the hot path needs no collective. Two even splits
(every rank gets B//P or B//P+1 sequences):
  contiguous  rank r owns sequences [r*B//P, (r+1)*B//P);
  balanced    the same counts, but sequences are dealt longest first to the
              rank with the fewest KV tokens so far that still has room, so
              every rank streams about the same KV bytes (decode time is
              proportional to them).
torch.distributed is used only around the measured region: a barrier, the
max over ranks of the device-timed duration, and a sum of output checksums.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(batch: int, world: int, rank: int) -> tuple[int, int]:
    """Even, contiguous split: sequence i goes to rank i*world//batch."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    return rank * batch // world, (rank + 1) * batch // world


def shard_counts(batch: int, world: int) -> list[int]:
    return [shard_bounds(batch, world, r)[1] - shard_bounds(batch, world, r)[0]
            for r in range(world)]


def balanced_assignment(lengths, world: int) -> list[list[int]]:
    """Equal-count, token-balanced split of sequence indices (each list sorted)."""
    lens = [int(x) for x in lengths]
    cap = shard_counts(len(lens), world)
    load, owned = [0] * world, [[] for _ in range(world)]
    for i in sorted(range(len(lens)), key=lambda i: (-lens[i], i)):
        r = min((r for r in range(world) if len(owned[r]) < cap[r]), key=lambda r: (load[r], r))
        owned[r].append(i)
        load[r] += lens[i]
    return [sorted(o) for o in owned]


def shard_indices(lengths, world: int, rank: int, mode: str = "balanced") -> list[int]:
    """Indices of the sequences rank `rank` owns under `mode`."""
    if mode == "contiguous":
        lo, hi = shard_bounds(len(lengths), world, rank)
        return list(range(lo, hi))
    if mode == "balanced":
        return balanced_assignment(lengths, world)[rank]
    raise ValueError(f"unknown sharding mode {mode!r}")


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
