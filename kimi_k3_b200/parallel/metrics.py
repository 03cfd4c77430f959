"""World reduction of scalar step metrics.

Parity: ``training/distributed/metrics.py:84-115`` (reference): a name containing ``max`` or
``peak`` reduces with MAX, ``min`` with MIN, everything else is a mean over the world.
The reference issues one collective per scalar (~100 per step); here the metrics are packed
into three float64 vectors (sum, max, min) and reduced with three collectives in total.
"""
from __future__ import annotations

import math
import zlib

import torch
import torch.distributed as dist


def reduction_for(name: str) -> str:
    low = name.lower()
    if "max" in low or "peak" in low:
        return "max"
    if "min" in low:
        return "min"
    return "mean"


def _agreed_names(names: list, group, device) -> list:
    """The union of every rank's metric names.  Ranks may log different optional metrics (diagnostics
    degrade per rank under their time budget); a fingerprint all-reduce confirms the common case of
    identical names, and only a disagreement pays for an object gather."""
    h = float(zlib.crc32("\x00".join(names).encode()))
    n = float(len(names))
    probe = torch.tensor([h, -h, n, -n], dtype=torch.float64, device=device)
    dist.all_reduce(probe, op=dist.ReduceOp.MAX, group=group)
    if probe[0].item() == -probe[1].item() and probe[2].item() == -probe[3].item():
        return names
    gathered = [None] * dist.get_world_size(group)
    dist.all_gather_object(gathered, names, group=group)
    return sorted(set().union(*gathered))


def reduce_scalar_metrics(metrics: dict, *, context=None, group=None) -> dict:
    if context is None or not getattr(context, "initialized", False) or context.world_size <= 1:
        return dict(metrics)
    numeric = {k: float(v) for k, v in metrics.items()
               if isinstance(v, (int, float, bool)) and not isinstance(v, str)}
    out = dict(metrics)
    dev = context.device
    names = _agreed_names(sorted(numeric), group, dev)
    by_kind = {"mean": [], "max": [], "min": []}
    for k in names:
        by_kind[reduction_for(k)].append(k)
    fill = {"mean": 0.0, "max": -math.inf, "min": math.inf}
    for kind, op in (("mean", dist.ReduceOp.SUM), ("max", dist.ReduceOp.MAX), ("min", dist.ReduceOp.MIN)):
        keys = by_kind[kind]
        if not keys:
            continue
        # non-finite values stay non-finite under every reduction (NaN propagates through SUM/MAX/MIN);
        # a metric this rank did not log contributes the reduction's identity
        vals = [numeric.get(k, fill[kind]) for k in keys]
        if kind == "mean":  # averaged over the ranks that logged it
            vals += [1.0 if k in numeric else 0.0 for k in keys]
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op, group=group)
        res = t.tolist()
        if kind == "mean":
            res = [v / max(c, 1.0) for v, c in zip(res[:len(keys)], res[len(keys):])]
        out.update(zip(keys, res))
    return out


__all__ = ["reduce_scalar_metrics", "reduction_for"]
