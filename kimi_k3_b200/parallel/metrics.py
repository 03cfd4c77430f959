"""World reduction of scalar step metrics.

Parity: ``training/distributed/metrics.py:84-115`` (reference): a name containing ``max`` or
``peak`` reduces with MAX, ``min`` with MIN, everything else is a mean over the world.
The reference issues one collective per scalar (~100 per step); here the metrics are packed
into three float64 vectors (sum, max, min) and reduced with three collectives in total.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def reduction_for(name: str) -> str:
    low = name.lower()
    if "max" in low or "peak" in low:
        return "max"
    if "min" in low:
        return "min"
    return "mean"


def reduce_scalar_metrics(metrics: dict, *, context=None, group=None) -> dict:
    if context is None or not getattr(context, "initialized", False) or context.world_size <= 1:
        return dict(metrics)
    numeric = {k: float(v) for k, v in metrics.items()
               if isinstance(v, (int, float, bool)) and not isinstance(v, str)}
    out = dict(metrics)
    by_kind = {"mean": [], "max": [], "min": []}
    for k in sorted(numeric):
        by_kind[reduction_for(k)].append(k)
    dev = context.device
    world = dist.get_world_size(group)
    for kind, op in (("mean", dist.ReduceOp.SUM), ("max", dist.ReduceOp.MAX), ("min", dist.ReduceOp.MIN)):
        names = by_kind[kind]
        if not names:
            continue
        # non-finite values stay non-finite under every reduction (NaN propagates through SUM/MAX/MIN)
        t = torch.tensor([numeric[k] for k in names], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op, group=group)
        vals = t.tolist()
        for k, v in zip(names, vals):
            out[k] = v / world if kind == "mean" else v
    return out


__all__ = ["reduce_scalar_metrics", "reduction_for"]
