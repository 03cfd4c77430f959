"""Exponential moving average of the trainable parameters.

Parity: ``training/ema.py:19-334`` (reference): fp32 shadow weights, warmup decay
``min(decay, (1 + n) / (10 + n))``, ``update_after_step`` / ``update_every``, name exclusion,
temporary swap for evaluation, checkpoint-safe state dict with the same keys.

B200 design: the shadow stays in device memory by default (HBM is ample) and one update is a
single multi-tensor ``lerp`` launch over all parameters; with ``device_decay=True`` the decay
is a device scalar so the update can sit inside a captured CUDA graph.
"""
from __future__ import annotations

from contextlib import contextmanager
from typing import Iterable

import torch
import torch.nn as nn


def unwrap_model(model: nn.Module) -> nn.Module:
    return model.module if hasattr(model, "module") else model


class EMA:
    def __init__(self, model: nn.Module, decay: float = 0.999, device=None, use_num_updates: bool = True,
                 update_after_step: int = 0, update_every: int = 1, exclude_names: Iterable[str] | None = None):
        if not 0.0 <= decay < 1.0:
            raise ValueError(f"EMA decay must satisfy 0 <= decay < 1. Got {decay}.")
        if update_after_step < 0:
            raise ValueError(f"update_after_step must be >= 0. Got {update_after_step}.")
        if update_every <= 0:
            raise ValueError(f"update_every must be > 0. Got {update_every}.")
        self.decay = float(decay)
        self.device = torch.device(device) if device is not None else None
        self.use_num_updates = bool(use_num_updates)
        self.update_after_step = int(update_after_step)
        self.update_every = int(update_every)
        self.num_updates = 0
        self.total_steps_seen = 0
        self.exclude_names = tuple(exclude_names or ())
        self.shadow: dict[str, torch.Tensor] = {}
        self.backup: dict[str, torch.Tensor] = {}
        for name, p in unwrap_model(model).named_parameters():
            if p.requires_grad and not self._is_excluded(name):
                s = p.detach().to(torch.float32).clone()
                self.shadow[name] = s.to(self.device) if self.device is not None else s

    def _is_excluded(self, name: str) -> bool:
        return any(pat in name for pat in self.exclude_names)

    def _compute_decay(self) -> float:
        if not self.use_num_updates:
            return self.decay
        return float(min(self.decay, (1.0 + self.num_updates) / (10.0 + self.num_updates)))

    def _pairs(self, model):
        shadows, params = [], []
        for name, p in unwrap_model(model).named_parameters():
            s = self.shadow.get(name)
            if s is not None and p.requires_grad:
                shadows.append(s)
                params.append(p.detach())
        return shadows, params

    @torch.no_grad()
    def update(self, model: nn.Module, step: int | None = None) -> bool:
        if step is None:
            self.total_steps_seen += 1
            cur = self.total_steps_seen
        else:
            cur = int(step)
            self.total_steps_seen = max(self.total_steps_seen, cur)
        if cur < self.update_after_step or (cur - self.update_after_step) % self.update_every:
            return False
        self.num_updates += 1
        d = self._compute_decay()
        shadows, params = self._pairs(model)
        same = [(s, p) for s, p in zip(shadows, params) if s.device == p.device and p.dtype == torch.float32]
        other = [(s, p) for s, p in zip(shadows, params) if not (s.device == p.device and p.dtype == torch.float32)]
        if same:
            # shadow <- d * shadow + (1 - d) * p  ==  lerp(shadow, p, 1 - d)
            torch._foreach_lerp_([s for s, _ in same], [p for _, p in same], 1.0 - d)
        for s, p in other:
            s.lerp_(p.to(device=s.device, dtype=torch.float32), 1.0 - d)
        return True

    @torch.no_grad()
    def copy_to(self, model: nn.Module) -> None:
        for name, p in unwrap_model(model).named_parameters():
            if name in self.shadow:
                p.data.copy_(self.shadow[name].to(device=p.device, dtype=p.dtype))

    @torch.no_grad()
    def store(self, model: nn.Module) -> None:
        self.backup = {name: p.detach().clone() for name, p in unwrap_model(model).named_parameters()
                       if name in self.shadow}

    @torch.no_grad()
    def restore(self, model: nn.Module) -> None:
        for name, p in unwrap_model(model).named_parameters():
            if name in self.backup:
                p.data.copy_(self.backup[name].to(device=p.device, dtype=p.dtype))
        self.backup = {}

    @contextmanager
    def average_parameters(self, model: nn.Module):
        self.store(model)
        self.copy_to(model)
        try:
            yield
        finally:
            self.restore(model)

    @torch.no_grad()
    def to(self, device) -> None:
        self.device = torch.device(device)
        self.shadow = {k: v.to(self.device) for k, v in self.shadow.items()}

    @torch.no_grad()
    def reinit_from_model(self, model: nn.Module) -> None:
        for name, p in unwrap_model(model).named_parameters():
            if name in self.shadow:
                self.shadow[name].copy_(p.detach().to(device=self.shadow[name].device, dtype=torch.float32))

    def state_dict(self) -> dict:
        return {"decay": self.decay, "device": str(self.device) if self.device is not None else None,
                "use_num_updates": self.use_num_updates, "update_after_step": self.update_after_step,
                "update_every": self.update_every, "num_updates": self.num_updates,
                "total_steps_seen": self.total_steps_seen, "exclude_names": self.exclude_names,
                "shadow": {k: v.detach().cpu() for k, v in self.shadow.items()}}

    @torch.no_grad()
    def load_state_dict(self, state: dict, strict: bool = False) -> None:
        self.decay = float(state.get("decay", self.decay))
        self.use_num_updates = bool(state.get("use_num_updates", self.use_num_updates))
        self.update_after_step = int(state.get("update_after_step", self.update_after_step))
        self.update_every = int(state.get("update_every", self.update_every))
        self.num_updates = int(state.get("num_updates", self.num_updates))
        self.total_steps_seen = int(state.get("total_steps_seen", self.total_steps_seen))
        self.exclude_names = tuple(state.get("exclude_names", self.exclude_names))
        loaded = state.get("shadow", {})
        missing = [k for k in self.shadow if k not in loaded]
        unexpected = [k for k in loaded if k not in self.shadow]
        for k, s in self.shadow.items():
            if k in loaded:
                s.copy_(loaded[k].to(device=s.device, dtype=s.dtype))
        if strict and (missing or unexpected):
            raise RuntimeError(f"EMA state mismatch. Missing={missing[:10]}, Unexpected={unexpected[:10]}")

    def __len__(self) -> int:
        return len(self.shadow)


@torch.no_grad()
def ema_health(ema: EMA, model: nn.Module, rel_tol: float = 5.0):
    """``(ok, status, relative_difference)`` comparing EMA and live weights."""
    shadows, params = ema._pairs(model)
    if not shadows:
        return False, "empty_ema", float("inf")
    sn = torch.stack([s.float().norm() for s in shadows]).norm()
    pn = torch.stack([p.float().norm() for p in params]).norm()
    diff = torch.stack([(s.float() - p.to(s.device).float()).norm() for s, p in zip(shadows, params)]).norm()
    if not bool(torch.isfinite(sn)):
        return False, "nan_or_inf_in_ema", float("inf")
    if float(pn) < 1e-12:
        return False, "model_zero_norm", float("inf")
    if float(sn) < 1e-12:
        return False, "ema_zero_norm", float("inf")
    rel = float(diff / (pn + 1e-8))
    if rel > rel_tol:
        return False, "large_rel_diff", rel
    return True, "ok", rel


__all__ = ["EMA", "ema_health", "unwrap_model"]
