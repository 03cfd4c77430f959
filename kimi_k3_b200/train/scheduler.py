"""Linear warmup + cosine decay, separately for the AdamW and Muon halves.

Parity: ``training/scheduler.py:13-324`` (reference): steps 1..warmup ramp linearly
from 0, then cosine to ``min_lr``; ``prepare_first_update`` sets the LR of the first
update at construction; state dicts restore the LR prepared for the next update.
"""
from __future__ import annotations

import math

import torch


class WarmupCosineLR:
    def __init__(self, optimizer, total_steps: int, warmup_steps: int, min_lr: float = 0.0,
                 min_muon_lr: float | None = None, prepare_first_update: bool = False):
        if total_steps <= 0 or warmup_steps < 0 or min_lr < 0 or (min_muon_lr is not None and min_muon_lr < 0):
            raise ValueError("invalid scheduler configuration")
        self.optimizer = optimizer
        self.total_steps, self.warmup_steps = int(total_steps), int(warmup_steps)
        self.min_lr = float(min_lr)
        self.min_muon_lr = None if min_muon_lr is None else float(min_muon_lr)
        self.prepare_first_update = bool(prepare_first_update)
        self.step_num = 0
        self.is_hybrid = hasattr(optimizer, "muon") and hasattr(optimizer, "adamw")
        if self.is_hybrid:
            self.base_adamw_lrs = [float(g["lr"]) for g in optimizer.adamw.param_groups]
            self.base_muon_lrs = [float(g["lr"]) for g in optimizer.muon.param_groups]
            self.base_lrs = self.base_muon_lrs + self.base_adamw_lrs
        else:
            self.base_lrs = [float(g["lr"]) for g in optimizer.param_groups]
            self.base_adamw_lrs = self.base_muon_lrs = None
        if self.prepare_first_update:
            self._set_lr(1)

    def _compute_lr(self, base_lr: float, min_lr: float, step: int) -> float:
        if self.warmup_steps > 0 and step <= self.warmup_steps:
            return base_lr * (step / max(1, self.warmup_steps))
        if self.total_steps <= self.warmup_steps:
            return min_lr
        t = min(max(step, self.warmup_steps), self.total_steps)
        progress = min(1.0, max(0.0, (t - self.warmup_steps) / max(1, self.total_steps - self.warmup_steps)))
        return float(min_lr + (base_lr - min_lr) * 0.5 * (1.0 + math.cos(math.pi * progress)))

    @staticmethod
    def _assign(group: dict, value: float) -> None:
        # Device-resident learning rates (CUDA-graph replay) are updated in place.
        if torch.is_tensor(group["lr"]):
            group["lr"].fill_(value)
        else:
            group["lr"] = value

    def _set_lr(self, step: int) -> None:
        if self.is_hybrid:
            mmin = self.min_lr if self.min_muon_lr is None else self.min_muon_lr
            for g, b in zip(self.optimizer.adamw.param_groups, self.base_adamw_lrs):
                self._assign(g, self._compute_lr(b, self.min_lr, step))
            for g, b in zip(self.optimizer.muon.param_groups, self.base_muon_lrs):
                self._assign(g, self._compute_lr(b, mmin, step))
        else:
            for g, b in zip(self.optimizer.param_groups, self.base_lrs):
                self._assign(g, self._compute_lr(b, self.min_lr, step))

    def step(self) -> None:
        self.step_num += 1
        self._set_lr(self.step_num + 1 if self.prepare_first_update else self.step_num)

    def set_step(self, step: int) -> None:
        if step < 0:
            raise ValueError("step must be >= 0")
        self.step_num = int(step)
        self._set_lr(self.step_num + 1 if self.prepare_first_update else self.step_num)

    def get_last_lr(self) -> list:
        if self.is_hybrid:
            return [g["lr"] for g in self.optimizer.muon.param_groups] + \
                   [g["lr"] for g in self.optimizer.adamw.param_groups]
        return [g["lr"] for g in self.optimizer.param_groups]

    def get_lr_dict(self) -> dict:
        if self.is_hybrid:
            return {"adamw_lr": self.optimizer.adamw.param_groups[0]["lr"],
                    "muon_lr": self.optimizer.muon.param_groups[0]["lr"], "step": self.step_num}
        return {"lr": self.optimizer.param_groups[0]["lr"], "step": self.step_num}

    def state_dict(self) -> dict:
        return {"step_num": self.step_num, "total_steps": self.total_steps, "warmup_steps": self.warmup_steps,
                "min_lr": self.min_lr, "min_muon_lr": self.min_muon_lr, "base_lrs": list(self.base_lrs),
                "base_adamw_lrs": self.base_adamw_lrs, "base_muon_lrs": self.base_muon_lrs,
                "is_hybrid": self.is_hybrid, "prepare_first_update": self.prepare_first_update}

    def load_state_dict(self, state: dict) -> None:
        self.step_num = int(state["step_num"])
        self.total_steps, self.warmup_steps = int(state["total_steps"]), int(state["warmup_steps"])
        self.min_lr = float(state["min_lr"])
        self.min_muon_lr = state.get("min_muon_lr")
        self.prepare_first_update = bool(state.get("prepare_first_update", self.prepare_first_update))
        if self.is_hybrid and state.get("base_adamw_lrs") is not None:
            self.base_adamw_lrs = [float(x) for x in state["base_adamw_lrs"]]
            self.base_muon_lrs = [float(x) for x in state["base_muon_lrs"]]
            self.base_lrs = self.base_muon_lrs + self.base_adamw_lrs
        elif isinstance(state.get("base_lrs"), (list, tuple)):
            self.base_lrs = [float(x) for x in state["base_lrs"]]
        self._set_lr(self.step_num + 1 if self.prepare_first_update else self.step_num)


def build_warmup_cosine_scheduler(optimizer, total_steps: int, warmup_steps: int, min_lr: float = 3e-5,
                                  min_muon_lr: float | None = None, prepare_first_update: bool = False):
    return WarmupCosineLR(optimizer, total_steps, warmup_steps, min_lr, min_muon_lr, prepare_first_update)


__all__ = ["WarmupCosineLR", "build_warmup_cosine_scheduler"]
