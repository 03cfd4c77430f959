"""Trainer state, token-exact loss accounting, JSONL logging and the AMP context.

Parity (reference paths):
  * ``training/state.py``                TrainerState
  * ``training/loss_accounting.py:36-214`` LossContribution, window combination (fp64 all-reduce
    of ``[ntp_norm, mtp_norm, tokens, ntp_sum, mtp_sum]`` over DP x EP)
  * ``training/logger.py:18-44``         JSONL + in-memory loggers
  * ``training/autocast.py:116-265``     bf16/fp16 autocast, GradScaler only for fp16
"""
from __future__ import annotations

import json
import math
from contextlib import nullcontext
from dataclasses import asdict, dataclass, fields
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist


@dataclass
class TrainerState:
    epoch: int = 0
    optimizer_step: int = 0
    micro_step: int = 0
    samples_seen: int = 0
    tokens_seen: int = 0
    valid_ntp_tokens_seen: int = 0
    valid_mtp_tokens_seen: int = 0
    curriculum_stage_index: int = 0
    best_eval_loss: float | None = None
    skipped_optimizer_steps: int = 0

    def state_dict(self) -> dict:
        return asdict(self)

    def load_state_dict(self, values: dict) -> None:
        known = {f.name for f in fields(self)}
        for k, v in values.items():
            if k in known:
                setattr(self, k, v)

    @classmethod
    def from_state_dict(cls, values: dict | None) -> "TrainerState":
        s = cls()
        if values:
            s.load_state_dict(values)
        return s


# --------------------------------------------------------------------------- loss accounting
def get_output_value(output: Any, name: str, default=None):
    return output.get(name, default) if isinstance(output, dict) else getattr(output, name, default)


def count_batch_tokens(batch: dict, ignore_index: int = -100) -> int:
    ids = batch.get("input_ids")
    if not torch.is_tensor(ids):
        return 0
    valid = torch.ones_like(ids, dtype=torch.bool)
    for key, fn in (("attention_mask", lambda t: t.bool()), ("labels", lambda t: t.ne(ignore_index)),
                    ("loss_mask", lambda t: t.bool())):
        t = batch.get(key)
        if torch.is_tensor(t):
            valid &= fn(t)
    return int(valid.sum().item())


@dataclass
class LossContribution:
    ntp_loss_sum: torch.Tensor
    ntp_normalizer: float
    mtp_loss_sum: torch.Tensor | None
    mtp_normalizer: float
    lambda_mtp: float
    reported_loss: float
    batch_tokens: int

    @property
    def ntp_loss(self) -> float:
        return float(self.ntp_loss_sum.detach()) / max(self.ntp_normalizer, 1.0)

    @property
    def mtp_loss(self) -> float | None:
        return None if self.mtp_loss_sum is None else float(self.mtp_loss_sum.detach()) / max(self.mtp_normalizer, 1.0)


def extract_loss_contribution(output: Any, batch: dict) -> LossContribution:
    loss = get_output_value(output, "loss")
    if loss is None or not torch.is_tensor(loss) or loss.ndim != 0:
        raise ValueError("model output must contain a loss scalar")
    lo = get_output_value(output, "loss_output")
    ntp = get_output_value(lo, "ntp") if lo is not None else None
    if ntp is not None:
        mtp = get_output_value(lo, "mtp")
        return LossContribution(get_output_value(ntp, "loss_sum"), float(get_output_value(ntp, "normalizer")),
                                None if mtp is None else get_output_value(mtp, "loss_sum"),
                                0.0 if mtp is None else float(get_output_value(mtp, "normalizer")),
                                float(get_output_value(lo, "lambda_mtp", 0.0)), float(loss.detach()),
                                count_batch_tokens(batch))
    n = float(max(count_batch_tokens(batch), 1))
    return LossContribution(loss * n, n, None, 0.0, 0.0, float(loss.detach()), count_batch_tokens(batch))


def combine_window_loss(contribs: list) -> tuple[torch.Tensor, dict]:
    if not contribs:
        raise ValueError("cannot combine an empty accumulation window")
    ntp_sum = torch.stack([c.ntp_loss_sum for c in contribs]).sum()
    ntp_n = sum(c.ntp_normalizer for c in contribs)
    if ntp_n <= 0:
        raise ValueError("accumulation window contains no valid NTP tokens")
    obj = ntp_sum / ntp_n
    mtp_items = [c for c in contribs if c.mtp_loss_sum is not None]
    mtp_n = sum(c.mtp_normalizer for c in mtp_items)
    mtp_loss = None
    if mtp_items:
        lambdas = {c.lambda_mtp for c in mtp_items}
        if len(lambdas) != 1:
            raise ValueError("lambda_mtp changed inside an accumulation window")
        if mtp_n <= 0:
            raise ValueError("MTP output contains no valid tokens")
        mtp_loss = torch.stack([c.mtp_loss_sum for c in mtp_items]).sum() / mtp_n
        obj = obj + lambdas.pop() * mtp_loss
    return obj, {"loss": float(obj.detach()), "ntp_loss": float((ntp_sum / ntp_n).detach()),
                 "mtp_loss": float("nan") if mtp_loss is None else float(mtp_loss.detach()),
                 "ntp_tokens": float(ntp_n), "mtp_tokens": float(mtp_n),
                 "tokens": float(sum(c.batch_tokens for c in contribs))}


def combine_distributed_window_loss(contribs: list, context) -> tuple[torch.Tensor, dict]:
    """Token-exact objective across DP x EP replicas (TP replicas hold the same tokens)."""
    if context is None or not getattr(context, "initialized", False):
        return combine_window_loss(contribs)
    if not contribs:
        raise ValueError("cannot combine an empty accumulation window")
    ntp_sum = torch.stack([c.ntp_loss_sum for c in contribs]).sum()
    mtp_items = [c for c in contribs if c.mtp_loss_sum is not None]
    mtp_sum = torch.stack([c.mtp_loss_sum for c in mtp_items]).sum() if mtp_items else None
    local = torch.stack([
        torch.tensor(float(sum(c.ntp_normalizer for c in contribs)), dtype=torch.float64),
        torch.tensor(float(sum(c.mtp_normalizer for c in mtp_items)), dtype=torch.float64),
        torch.tensor(float(sum(c.batch_tokens for c in contribs)), dtype=torch.float64)]).to(ntp_sum.device)
    sums = torch.stack([ntp_sum.detach().double(), (mtp_sum.detach().double() if mtp_sum is not None
                                                     else torch.zeros((), dtype=torch.float64,
                                                                      device=ntp_sum.device))])
    packed = torch.cat([local, sums])
    axes = (context.data_replica_groups if hasattr(context, "data_replica_groups") else
            ((getattr(context, "dp_group", None), getattr(context, "dp_size", 1)),
             (getattr(context, "ep_group", None), getattr(context, "ep_size", 1))))
    replicas = 1
    for group, size in axes:
        replicas *= size
        if group is not None and size > 1:
            dist.all_reduce(packed, group=group)
    ntp_n, mtp_n, tokens, g_ntp, g_mtp = packed.tolist()
    if ntp_n <= 0:
        raise ValueError("accumulation window contains no valid NTP tokens")
    obj = ntp_sum * replicas / ntp_n
    mtp_loss = None
    if mtp_items:
        lam = mtp_items[0].lambda_mtp
        mtp_loss = g_mtp / max(mtp_n, 1.0)
        obj = obj + lam * mtp_sum * replicas / max(mtp_n, 1.0)
    total = g_ntp / ntp_n + (0.0 if mtp_loss is None else mtp_items[0].lambda_mtp * mtp_loss)
    return obj, {"loss": total, "ntp_loss": g_ntp / ntp_n, "mtp_loss": float("nan") if mtp_loss is None else mtp_loss,
                 "ntp_tokens": ntp_n, "mtp_tokens": mtp_n, "tokens": tokens}


def compute_loss_metrics(*, total_loss, ntp_loss, mtp_loss, ntp_tokens, mtp_tokens, lambda_mtp) -> dict:
    out = {"train/loss": total_loss, "train/ntp_loss": ntp_loss,
           "train/ntp_ppl": math.exp(min(ntp_loss, 50.0)), "train/ntp_tokens": ntp_tokens,
           "train/lambda_mtp": lambda_mtp}
    if mtp_loss is not None:
        out.update({"train/mtp_loss": mtp_loss, "train/mtp_ppl": math.exp(min(mtp_loss, 50.0)),
                    "train/mtp_tokens": mtp_tokens})
    return out


# --------------------------------------------------------------------------- loggers
class JSONLLogger:
    """Append one JSON object per logged step."""

    def __init__(self, path: str | Path, enabled: bool = True):
        self.path = Path(path)
        self.enabled = enabled
        if enabled:
            self.path.parent.mkdir(parents=True, exist_ok=True)

    def log(self, step: int, metrics: dict) -> None:
        if not self.enabled:
            return
        rec = {"step": int(step)}
        for k, v in metrics.items():
            if isinstance(v, torch.Tensor) and v.numel() == 1:
                v = float(v)
            if isinstance(v, (int, float, str, bool)) or v is None:
                rec[k] = v
        with self.path.open("a", encoding="utf-8") as fh:
            fh.write(json.dumps(rec) + "\n")


class MemoryLogger:
    def __init__(self):
        self.records: list = []

    def log(self, step: int, metrics: dict) -> None:
        self.records.append({"step": int(step), **metrics})


# --------------------------------------------------------------------------- AMP
def resolve_amp_dtype(precision: str, device: torch.device):
    if precision == "fp32" or device.type not in ("cuda", "cpu"):
        return None
    if precision == "bf16":
        if device.type == "cuda" and not torch.cuda.is_bf16_supported():
            return torch.float16
        return torch.bfloat16
    return torch.float16


def autocast_ctx(device, enabled: bool = True, amp_dtype: str = "bf16"):
    device = torch.device(device)
    if not enabled:
        return nullcontext()
    dt = resolve_amp_dtype(amp_dtype, device)
    if dt is None:
        return nullcontext()
    return torch.autocast(device.type, dtype=dt)


def make_grad_scaler(precision: str, device: torch.device):
    if precision == "fp16" and torch.device(device).type == "cuda":
        return torch.amp.GradScaler("cuda")
    return None


__all__ = [
    "TrainerState", "LossContribution", "extract_loss_contribution", "combine_window_loss",
    "combine_distributed_window_loss", "compute_loss_metrics", "count_batch_tokens", "JSONLLogger", "MemoryLogger",
    "autocast_ctx", "resolve_amp_dtype", "make_grad_scaler",
]
