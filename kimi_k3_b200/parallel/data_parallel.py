"""Data parallelism: bucketed gradient all-reduce over NCCL.

Parity target: the reference wraps the model in ``DistributedDataParallel`` on the DP
group (``training/distributed/wrapping.py:61-88``).  Here gradients are packed into
dtype-homogeneous flat buckets after backward and all-reduced (average) bucket by
bucket with async NCCL ops; parameters with no gradient contribute zeros so every rank
reduces identical layouts (the reference needs ``find_unused_parameters=True`` for
the same reason).  Quantile-Balancing statistics are made global by ``QBReducer``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch._utils import _flatten_dense_tensors, _unflatten_dense_tensors


class QBReducer:
    """Global Quantile-Balancing statistics over the data/expert-parallel group."""

    def __init__(self, group=None):
        self.group = group

    def _world(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    def reduce_histogram(self, balancer) -> None:
        if self._world() == 1:
            return
        packed = torch.cat([balancer.counts.reshape(-1), balancer.underflow, balancer.overflow])
        dist.all_reduce(packed, group=self.group)
        e, b = balancer.counts.shape
        balancer.counts.copy_(packed[: e * b].view(e, b))
        balancer.underflow.copy_(packed[e * b: e * b + e])
        balancer.overflow.copy_(packed[e * b + e:])

    def gather_exact(self, scores, cutoffs):
        if self._world() == 1:
            return scores, cutoffs
        from .collectives import all_gather_variable
        return all_gather_variable(scores, group=self.group), all_gather_variable(cutoffs, group=self.group)


class GradientAllReducer:
    def __init__(self, model: torch.nn.Module, group=None, bucket_bytes: int = 256 << 20):
        self.model = model
        self.group = group
        self.bucket_bytes = bucket_bytes
        self.params = [p for p in model.parameters() if p.requires_grad]
        self._buckets = self._plan()

    def _plan(self):
        buckets, cur, size, cur_dtype = [], [], 0, None
        for p in self.params:
            nbytes = p.numel() * p.element_size()
            if cur and (p.dtype != cur_dtype or size + nbytes > self.bucket_bytes):
                buckets.append(cur)
                cur, size = [], 0
            cur.append(p)
            cur_dtype = p.dtype
            size += nbytes
        if cur:
            buckets.append(cur)
        return buckets

    @property
    def world_size(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    @torch.no_grad()
    def broadcast_parameters(self, src: int = 0) -> None:
        if self.world_size == 1:
            return
        tensors = list(self.model.parameters()) + list(self.model.buffers())
        by_dtype: dict = {}
        for t in tensors:
            by_dtype.setdefault((t.dtype, t.device), []).append(t)
        for ts in by_dtype.values():
            flat = _flatten_dense_tensors([t.data for t in ts])
            dist.broadcast(flat, src=src, group=self.group)
            for t, s in zip(ts, _unflatten_dense_tensors(flat, [t.data for t in ts])):
                t.data.copy_(s)

    @torch.no_grad()
    def all_reduce_gradients(self) -> None:
        world = self.world_size
        if world == 1:
            return
        pending = []
        for bucket in self._buckets:
            grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in bucket]
            flat = _flatten_dense_tensors(grads)
            flat.div_(world)
            work = dist.all_reduce(flat, group=self.group, async_op=True)
            pending.append((bucket, grads, flat, work))
        for bucket, grads, flat, work in pending:
            work.wait()
            for p, g in zip(bucket, _unflatten_dense_tensors(flat, grads)):
                if p.grad is None:
                    p.grad = g.clone()
                else:
                    p.grad.copy_(g)

    def qb_reducer(self) -> QBReducer:
        return QBReducer(self.group)


__all__ = ["GradientAllReducer", "QBReducer"]
