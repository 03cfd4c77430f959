"""One-optimizer-step training engine used by the trainer loop and ``bench.py``.

A step = (optional pinned host -> device copy) -> bf16 autocast forward with the
fused head losses (no ``[N, V]`` logits) -> backward -> global-norm clip on the
device -> hybrid optimizer -> scheduler -> Quantile-Balancing commit.  The clip
coefficient is applied without a host round trip; the only host syncs are the
loss normalisers and the optimizer's single finite-gradient check.

Parity: the step semantics follow ``training/train_one_epoch.py:145-330`` (reference)
for a window of one micro-batch.
"""
from __future__ import annotations

from contextlib import nullcontext
from dataclasses import dataclass

import torch


@dataclass
class StepOutput:
    loss: torch.Tensor          # device scalar (total objective)
    ntp_loss: torch.Tensor
    mtp_loss: torch.Tensor | None
    grad_norm: torch.Tensor     # device scalar, pre-clip
    executed: bool


def move_batch(batch: dict, device, non_blocking: bool = True) -> dict:
    return {k: (v.to(device, non_blocking=non_blocking) if isinstance(v, torch.Tensor) else v)
            for k, v in batch.items()}


@torch.no_grad()
def clip_grad_norm_device(params, max_norm: float | None) -> torch.Tensor:
    """Global L2 norm of the gradients; scales them in place by min(1, max_norm/norm) on device."""
    grads = [p.grad for p in params if p.grad is not None]
    if not grads:
        return torch.zeros(())
    norms = torch._foreach_norm(grads, 2.0)
    total = torch.linalg.vector_norm(torch.stack([n.float() for n in norms]), 2.0)
    if max_norm is not None:
        coef = (max_norm / (total + 1e-6)).clamp(max=1.0)
        torch._foreach_mul_(grads, coef)
    return total


class TrainStepEngine:
    """Runs optimizer steps of a KimiK3 model (single process; the distributed runtime wraps it)."""

    def __init__(self, model, optimizer, *, scheduler=None, grad_clip: float | None = 1.0,
                 amp_dtype: torch.dtype | None = torch.bfloat16, use_mtp: bool = True, moe_controller=None,
                 grad_hook=None):
        self.model = model
        self.optimizer = optimizer
        self.scheduler = scheduler
        self.grad_clip = grad_clip
        self.amp_dtype = amp_dtype
        self.use_mtp = use_mtp
        self.moe_controller = moe_controller
        self.grad_hook = grad_hook  # called after backward (gradient reduction in data parallel)
        self.device = next(model.parameters()).device
        self._params = [p for p in model.parameters() if p.requires_grad]

    def _autocast(self):
        if self.amp_dtype is None or self.device.type != "cuda":
            return nullcontext()
        return torch.autocast("cuda", dtype=self.amp_dtype)

    def forward_loss(self, batch: dict):
        with self._autocast():
            out = self.model(input_ids=batch["input_ids"], attention_mask=batch.get("attention_mask"),
                             labels=batch["labels"], use_mtp=self.use_mtp, compute_logits=False)
        return out

    def step(self, batch: dict) -> StepOutput:
        if batch["input_ids"].device != self.device:
            batch = move_batch(batch, self.device)
        self.model.train()
        if self.moe_controller is not None:
            self.moe_controller.begin()
        try:
            out = self.forward_loss(batch)
            out.loss.backward()
            if self.grad_hook is not None:
                self.grad_hook()
            gnorm = clip_grad_norm_device(self._params, self.grad_clip)
            report = self.optimizer.step()
            executed = bool(getattr(report, "executed", True))
        except BaseException:
            if self.moe_controller is not None:
                self.moe_controller.discard()
            self.optimizer.zero_grad(set_to_none=True)
            raise
        if executed:
            if self.scheduler is not None:
                self.scheduler.step()
            if self.moe_controller is not None:
                self.moe_controller.commit()
        elif self.moe_controller is not None:
            self.moe_controller.discard()
        self.optimizer.zero_grad(set_to_none=True)
        lo = out.loss_output
        return StepOutput(out.loss.detach(), lo.ntp.loss.detach(), None if lo.mtp is None else lo.mtp.loss.detach(),
                          gnorm, executed)


class MoEController:
    """Open / commit / discard Quantile-Balancing windows on every balanced MoE layer.

    Parity: ``training/moe_control.py:10-57`` (reference).  ``reducer`` (expert / data
    parallel) makes the window statistics global before the bias update.
    """

    def __init__(self, model, reducer=None):
        from ..models.moe import StableLatentMoE
        raw = model.module if hasattr(model, "module") else model
        self.layers = tuple(m for m in raw.modules()
                            if isinstance(m, StableLatentMoE) and m.config.enable_quantile_balancing)
        self.reducer = reducer
        self.window_open = False

    def begin(self) -> None:
        if self.window_open:
            raise RuntimeError("a Quantile Balancing window is already open")
        for layer in self.layers:
            layer.begin_balance_accumulation()
        self.window_open = True

    def commit(self):
        if not self.window_open:
            raise RuntimeError("no Quantile Balancing window is open")
        updates = tuple(layer.finalize_and_commit_balance(self.reducer) for layer in self.layers)
        self.window_open = False
        return updates

    def discard(self) -> None:
        if not self.window_open:
            return
        for layer in self.layers:
            layer.discard_balance_accumulation()
        self.window_open = False

    def assert_clean(self) -> None:
        if self.window_open:
            raise RuntimeError("checkpoint requested with an open QB window")
