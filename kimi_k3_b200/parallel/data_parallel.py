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

from ..debug import nvtx


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
    """Average gradients over a data-replica group in flat, dtype-homogeneous buckets.

    With ``overlap=True`` each bucket's all-reduce is launched from a post-accumulate-grad
    hook as soon as the last gradient of the bucket has been produced, so communication runs
    under the rest of the backward pass (buckets are filled in reverse parameter order,
    roughly the order backward produces them; with gradient accumulation only the window's last
    backward runs ``armed``). ``all_reduce_gradients()`` then launches any
    bucket that did not complete (parameters without gradients contribute zeros) and waits.
    ``params`` restricts the reducer to a subset (expert-parallel layouts reduce expert and
    replicated parameters over different groups).
    """

    def __init__(self, model: torch.nn.Module, group=None, bucket_bytes: int = 256 << 20, *, params=None,
                 overlap: bool = False, scale: float | None = None):
        self.model = model
        self.group = group
        self.bucket_bytes = int(bucket_bytes)
        self._all_params = params is None
        self.params = [p for p in (params if params is not None else model.parameters()) if p.requires_grad]
        self.scale = scale
        self._buckets = self._plan()
        self.overlap = bool(overlap) and self.world_size > 1
        self._ready = [0] * len(self._buckets)
        self._pending = {}
        self._hooks = []
        self.armed = True  # trainers disarm for all but the last backward of an accumulation window
        if self.overlap:
            where = {}
            for bi, bucket in enumerate(self._buckets):
                for p in bucket:
                    where[id(p)] = bi
            for p in self.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(
                    lambda param, bi=where[id(p)]: self._grad_ready(bi)))

    def _plan(self):
        buckets, cur, size, cur_key = [], [], 0, None
        for p in reversed(self.params):
            nbytes = p.numel() * p.element_size()
            key = (p.dtype, p.device)
            if cur and (key != cur_key or size + nbytes > self.bucket_bytes):
                buckets.append(cur)
                cur, size = [], 0
            cur.append(p)
            cur_key = key
            size += nbytes
        if cur:
            buckets.append(cur)
        return buckets

    @property
    def world_size(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    def _src(self) -> int:
        return dist.get_global_rank(self.group, 0) if self.group is not None else 0

    @torch.no_grad()
    def broadcast_parameters(self, src: int | None = None) -> None:
        """Make every replica start from the group's first rank's parameters and buffers."""
        if self.world_size == 1:
            return
        src = self._src() if src is None else src
        seen, tensors = set(), []
        # a reducer over a parameter subset only owns (and broadcasts) that subset
        owned = list(self.model.parameters()) + list(self.model.buffers()) if self._all_params else list(self.params)
        for t in owned:
            if id(t) not in seen:
                seen.add(id(t))
                tensors.append(t)
        by_key: dict = {}
        for t in tensors:
            by_key.setdefault((t.dtype, t.device), []).append(t)
        for ts in by_key.values():
            flat = _flatten_dense_tensors([t.data for t in ts])
            dist.broadcast(flat, src=src, group=self.group)
            for t, v in zip(ts, _unflatten_dense_tensors(flat, [t.data for t in ts])):
                t.data.copy_(v)

    @torch.no_grad()
    def _launch(self, bi: int) -> None:
        if bi in self._pending:
            return
        bucket = self._buckets[bi]
        grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in bucket]
        with nvtx(f"dp all-reduce bucket {bi}"):
            flat = _flatten_dense_tensors(grads)
            flat.mul_(self.scale if self.scale is not None else 1.0 / self.world_size)
            self._pending[bi] = (grads, flat, dist.all_reduce(flat, group=self.group, async_op=True))

    def _grad_ready(self, bi: int) -> None:
        if not self.armed:  # an earlier micro-batch of an accumulation window
            return
        self._ready[bi] += 1
        if self._ready[bi] == len(self._buckets[bi]):
            self._launch(bi)

    @torch.no_grad()
    def all_reduce_gradients(self) -> None:
        if self.world_size == 1:
            return
        for bi in range(len(self._buckets)):
            self._launch(bi)
        for bi, (grads, flat, work) in sorted(self._pending.items()):
            work.wait()
            for p, v in zip(self._buckets[bi], _unflatten_dense_tensors(flat, grads)):
                if p.grad is None:
                    p.grad = v.clone()
                else:
                    p.grad.copy_(v)
        self._pending.clear()
        self._ready = [0] * len(self._buckets)

    def remove_hooks(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []

    def qb_reducer(self) -> QBReducer:
        return QBReducer(self.group)


__all__ = ["GradientAllReducer", "QBReducer"]
