"""``data_parallel.mode: fsdp`` - sharded gradients and optimizer state with whole-tensor owners.

The reference wraps the model in PyTorch FSDP (``training/distributed/wrapping.py:90-127``)
and leaves Muon's compatibility with flattened shards unverified. Muon's Newton-Schulz needs
whole matrices, so this layout shards by TENSOR instead of by flat slice: every parameter
has one owner rank in the data-parallel group (greedy balance by size); after backward each
owner-bucket of gradients is averaged onto its owner (``reduce``); the owner alone keeps
momentum / Adam state and runs Muon (on whole matrices) and AdamW; updated parameters are
broadcast back from their owners. Parameters stay replicated (HBM holds them easily at these
sizes); gradient and optimizer-state memory is divided by the group size.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
from torch._utils import _flatten_dense_tensors, _unflatten_dense_tensors

from ..train.optimizer import OptimizerStepReport


class ZeroDataParallel:
    def __init__(self, model: torch.nn.Module, optimizer, group=None, *, bucket_mb: float = 64.0):
        self.model, self.optimizer, self.group = model, optimizer, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        params = [p for p in model.parameters() if p.requires_grad]
        load = [0] * self.world
        self.owner = {}
        for p in sorted(params, key=lambda t: -t.numel()):
            r = min(range(self.world), key=lambda i: load[i])
            self.owner[id(p)] = r
            load[r] += p.numel()
        self.params = params
        self.owned = [p for p in params if self.owner[id(p)] == self.rank]
        optimizer.restrict_to({id(p) for p in self.owned})
        cap = int(bucket_mb * (1 << 20))
        self.buckets = []  # (owner, [params]) dtype/device homogeneous
        for r in range(self.world):
            cur, size, key = [], 0, None
            for p in params:
                if self.owner[id(p)] != r:
                    continue
                k = (p.dtype, p.device)
                if cur and (k != key or size + p.numel() * p.element_size() > cap):
                    self.buckets.append((r, cur))
                    cur, size = [], 0
                cur.append(p)
                key = k
                size += p.numel() * p.element_size()
            if cur:
                self.buckets.append((r, cur))

    def _global(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    @torch.no_grad()
    def broadcast_parameters(self) -> None:
        """Start every replica from rank 0's parameters and buffers."""
        if self.world == 1:
            return
        for t in list(self.model.parameters()) + list(self.model.buffers()):
            dist.broadcast(t.data, src=self._global(0), group=self.group)

    @torch.no_grad()
    def reduce_gradients(self) -> None:
        """Average each owner bucket onto its owner; other ranks drop those gradients."""
        if self.world == 1:
            return
        pending = []
        for r, ps in self.buckets:
            grads = [p.grad if p.grad is not None else torch.zeros_like(p) for p in ps]
            flat = _flatten_dense_tensors(grads).mul_(1.0 / self.world)
            pending.append((r, ps, grads, flat, dist.reduce(flat, dst=self._global(r), group=self.group,
                                                             async_op=True)))
        for r, ps, grads, flat, work in pending:
            work.wait()
            if r == self.rank:
                for p, g in zip(ps, _unflatten_dense_tensors(flat, grads)):
                    p.grad = g.clone() if p.grad is None else p.grad.copy_(g)
            else:
                for p in ps:
                    p.grad = None

    @torch.no_grad()
    def grad_norm(self) -> torch.Tensor | None:
        grads = [p.grad for p in self.owned if p.grad is not None]
        dev = self.params[0].device
        sq = (torch.stack([n.float() for n in torch._foreach_norm(grads, 2.0)]).square().sum() if grads
              else torch.zeros((), device=dev))
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
        return sq.sqrt()

    @torch.no_grad()
    def _broadcast_updates(self) -> None:
        for r, ps in self.buckets:
            flat = _flatten_dense_tensors([p.data for p in ps])
            dist.broadcast(flat, src=self._global(r), group=self.group)
            if r != self.rank:
                for p, v in zip(ps, _unflatten_dense_tensors(flat, [p.data for p in ps])):
                    p.data.copy_(v)

    # ---- optimizer facade used by the training loop
    @property
    def param_groups(self):
        return self.optimizer.param_groups

    def zero_grad(self, set_to_none: bool = True) -> None:
        self.optimizer.zero_grad(set_to_none=set_to_none)

    @torch.no_grad()
    def step(self, closure=None):
        self.optimizer.drop_foreign_gradients()
        grads = [p.grad for p in self.owned if p.grad is not None]
        ok = torch.tensor([1 if all(bool(torch.isfinite(g).all()) for g in grads) else 0], dtype=torch.int32,
                          device=self.params[0].device)
        if self.world > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if not bool(ok.item()):
            return OptimizerStepReport(False, 0.0, 0.0, False, 0, 1, {})
        qk = getattr(self.optimizer, "qk_clip", None)
        if qk is not None:
            self.optimizer.qk_clip = None  # applied below on every rank, after the broadcast
        try:
            report = self.optimizer.step(gradients_known_finite=True)
        finally:
            if qk is not None:
                self.optimizer.qk_clip = qk
        if self.world > 1:
            self._broadcast_updates()
        if qk is not None:
            qk.apply(self.optimizer.step_number, materialize=False)
        refresh = getattr(self.optimizer, "refresh_weight_mirror", None)
        if refresh is not None:
            refresh()  # the broadcasts and QK-Clip rewrote masters after the optimizer's own refresh
        return report

    def state_dict(self) -> dict:
        return {"owner_rank": self.rank, "world": self.world, "optimizer": self.optimizer.state_dict()}

    def load_state_dict(self, state: dict, strict: bool = True) -> None:
        if int(state["world"]) != self.world:
            raise ValueError("sharded optimizer state was saved for another data-parallel size")
        self.optimizer.load_state_dict(state["optimizer"], strict=strict)


__all__ = ["ZeroDataParallel"]
