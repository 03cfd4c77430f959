"""Size-1-safe collective helpers.

Parity: ``training/distributed/collectives.py:21-80`` (reference): sum / mean / max
all-reduce, ``all_ranks_true`` (MIN), and ``all_gather_variable`` (lengths first,
pad to the max, gather, trim).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _active(group) -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1


def all_reduce_sum(t: torch.Tensor, group=None) -> torch.Tensor:
    if _active(group):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def all_reduce_mean(t: torch.Tensor, group=None) -> torch.Tensor:
    if _active(group):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
        t.div_(dist.get_world_size(group))
    return t


def all_reduce_max(t: torch.Tensor, group=None) -> torch.Tensor:
    if _active(group):
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t


def all_ranks_true(value: bool, *, device=None, group=None) -> bool:
    if not _active(group):
        return bool(value)
    t = torch.tensor([1 if value else 0], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


def all_gather_variable(t: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenate tensors whose first dimension differs across ranks."""
    if not _active(group):
        return t
    world = dist.get_world_size(group)
    n = torch.tensor([t.shape[0]], device=t.device, dtype=torch.long)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    mx = max(sizes)
    padded = t.new_zeros((mx,) + tuple(t.shape[1:]))
    padded[: t.shape[0]] = t
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], 0)


__all__ = ["all_reduce_sum", "all_reduce_mean", "all_reduce_max", "all_ranks_true", "all_gather_variable"]
