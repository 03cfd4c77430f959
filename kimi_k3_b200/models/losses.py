"""Token losses: NTP, MTP, pretraining composite, SFT, Kimi policy loss, MOPD.

Parity targets (reference paths):
  * ``src/loss/common/reduction.py:10-51``, ``common/validation.py:14-127``
  * ``src/loss/pretraining/cross_entropy.py:13-57``, ``next_token_loss.py``
  * ``src/loss/multi_token_prediction_loss.py:18-105``
  * ``src/loss/pretraining/composite.py:12-77``  (NTP + lambda * MTP, no router loss)
  * ``src/loss/sft_loss.py:22-157``, ``policy_optimization_loss.py:17-176``,
    ``mopd_loss.py:21-216``, ``rl/reward_processing.py``, ``distillation/components.py``
  * ``src/loss/training_objective.py:66-118``, ``common/config.py``

Label alignment: the reference's datasets emit pre-shifted labels and its NTP
loss applies a causal shift again, so logits[t] train against x[t+2].
``label_alignment="causal_shift"`` (default) reproduces that exactly;
``"already_aligned"`` treats ``labels[t]`` as the target of ``logits[t]``.

On CUDA the NTP/MTP heads use :func:`kimi_k3_b200.ops.linear_cross_entropy`,
which fuses the vocabulary projection with an online log-sum-exp and never
materialises ``[N,V]`` fp32 logits.
"""
from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from dataclasses import asdict, dataclass
from enum import Enum, IntEnum

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops as _ops
from ..runtime import host_checks


# --------------------------------------------------------------------------- typed outputs
@dataclass
class LossOutput:
    loss: torch.Tensor
    loss_sum: torch.Tensor
    normalizer: torch.Tensor
    num_valid_tokens: torch.Tensor


@dataclass
class TokenCrossEntropyOutput(LossOutput):
    per_token_nll: torch.Tensor | None = None
    per_sample_loss_sum: torch.Tensor | None = None
    per_sample_num_tokens: torch.Tensor | None = None


@dataclass
class MTPLossOutput(TokenCrossEntropyOutput):
    per_depth_loss_sum: torch.Tensor | None = None
    per_depth_normalizer: torch.Tensor | None = None
    future_offsets: tuple | None = None


@dataclass
class SFTLossOutput(TokenCrossEntropyOutput):
    per_component_loss_sum: dict | None = None
    per_component_num_tokens: dict | None = None
    reduction: str = "token_mean"


@dataclass
class PolicyOptimizationLossOutput(LossOutput):
    policy_objective_sum: torch.Tensor = None
    regularization_sum: torch.Tensor = None
    mean_advantage: torch.Tensor = None
    mean_log_ratio: torch.Tensor = None
    max_abs_log_ratio: torch.Tensor = None
    clipped_fraction: torch.Tensor = None
    mean_reward: torch.Tensor | None = None
    reward_std: torch.Tensor | None = None


@dataclass
class MOPDLossOutput(LossOutput):
    mean_token_reward: torch.Tensor = None
    reward_clip_fraction: torch.Tensor = None
    mean_teacher_logprob: torch.Tensor = None
    mean_student_logprob: torch.Tensor = None
    mean_teacher_student_gap: torch.Tensor = None
    teacher_token_count: torch.Tensor = None
    mode: str = "sampled_token_pg"
    reward_reference: str = "current_detached"
    policy_output: PolicyOptimizationLossOutput | None = None


@dataclass
class KimiPretrainingLossOutput:
    loss: torch.Tensor
    ntp: TokenCrossEntropyOutput
    mtp: MTPLossOutput | None
    lambda_mtp: float
    moe_diagnostics: object | None = None
    moe_aux_loss: None = None


class SFTComponent(IntEnum):
    IGNORE = 0
    REASONING = 1
    TOOL_CALL = 2
    TOOL_ARGUMENT = 3
    ASSISTANT_TEXT = 4
    FINAL_ANSWER = 5
    END_OF_TURN = 6


class KimiTrainingPhase(str, Enum):
    PRETRAIN = "pretrain"
    SFT = "sft"
    RL = "rl"
    MOPD = "mopd"


@dataclass(frozen=True)
class RewardWeights:
    verifier: float | None = None
    generative: float | None = None
    task_specific: float | None = None


@dataclass
class KimiLossBundle:
    phase: KimiTrainingPhase
    loss: torch.Tensor
    output: object


# --------------------------------------------------------------------------- helpers
def connected_zero(source: torch.Tensor) -> torch.Tensor:
    """fp32 scalar zero that keeps ``source`` in the autograd graph."""
    return source.float().reshape(-1)[:0].sum()


def boolean_mask(name, value, shape, device, *, default=True):
    if value is None:
        return torch.full(shape, default, dtype=torch.bool, device=device)
    if tuple(value.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}")
    if value.device != device:
        raise ValueError(f"{name} must share the logits device")
    return value.to(torch.bool)


def require_finite(name, values, valid):
    bad = valid & ~torch.isfinite(values)
    if torch.any(bad):
        raise FloatingPointError(f"{name} contains {int(bad.sum().item())} non-finite valid values")


def validate_token_ids(labels, valid, vocab_size, *, name="labels"):
    if labels.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"{name} must use int32 or int64")
    if host_checks() and torch.any(valid & ((labels < 0) | (labels >= vocab_size))):
        raise ValueError(f"{name} contains IDs outside [0, {vocab_size})")


def validate_zero_policy(value):
    if value not in ("raise", "connected_zero"):
        raise ValueError("zero_valid_policy must be 'raise' or 'connected_zero'")
    return value


def align_token_inputs(logits_shape_source, labels, *, alignment, attention_mask, loss_mask, boundary_mask,
                       token_weights, ignore_index, logits=None):
    """Return ``(time_slice, aligned_labels, valid, weights)`` for the chosen alignment.

    ``logits_shape_source`` is any ``[B,T,...]`` tensor on the loss device.
    """
    b, t = labels.shape
    dev = logits_shape_source.device
    if alignment not in ("causal_shift", "already_aligned"):
        raise ValueError("unsupported alignment")
    src = boolean_mask("attention_mask", attention_mask, (b, t), dev)
    sem = boolean_mask("loss_mask", loss_mask, (b, t), dev)
    bnd = boolean_mask("boundary_mask", boundary_mask, (b, t), dev)
    if token_weights is None:
        w = torch.ones((b, t), device=dev)
    else:
        if tuple(token_weights.shape) != (b, t):
            raise ValueError(f"token_weights must have shape {(b, t)}")
        w = token_weights.float()
        if not torch.isfinite(w).all() or torch.any(w < 0):
            raise ValueError("token_weights must be finite and non-negative")
    if alignment == "causal_shift":
        sl = slice(0, t - 1)
        al = labels[:, 1:]
        valid = src[:, :-1] & src[:, 1:] & sem[:, 1:] & bnd[:, 1:]
        w = w[:, 1:]
    else:
        sl = slice(0, t)
        al = labels
        valid = src & sem & bnd
    return sl, al, valid & al.ne(ignore_index), w


def reduce_token_losses(per_token, valid, weights, *, source, zero_valid_policy, return_per_token):
    eff = weights.float() * valid.float()
    normalizer = eff.sum(dtype=torch.float32)
    weighted = torch.where(valid, per_token.float() * weights.float(), torch.zeros_like(per_token, dtype=torch.float32))
    loss_sum = weighted.sum(dtype=torch.float32)
    if normalizer.item() == 0:
        if zero_valid_policy == "raise":
            raise ValueError("loss batch contains no valid tokens")
        loss = loss_sum = connected_zero(source)
    else:
        loss = loss_sum / normalizer
    return TokenCrossEntropyOutput(loss, loss_sum, normalizer.detach(), valid.sum().float().detach(),
                                   per_token.detach() if return_per_token else None, weighted.sum(-1).detach(),
                                   valid.sum(-1).detach())


def head_vocab_size(weight) -> int:
    """Full vocabulary of an LM-head weight (a tensor-parallel shard records the full size)."""
    meta = getattr(weight, "_kimi_vocab_parallel", None)
    return int(meta[2]) if meta is not None else int(weight.shape[0])


def fused_head_loss(hidden, weight, labels, valid, *, label_smoothing=0.0):
    """Per-row CE of ``hidden @ weight^T`` against ``labels`` for valid rows.

    Returns ``(loss_sum, per_row)``; on CUDA the projection + log-sum-exp run
    fused and ``per_row`` is ``None``. A vocabulary-sharded head weight (tensor parallel)
    goes through the fused vocabulary-parallel CE: logits are never gathered.
    """
    flat_h = hidden.reshape(-1, hidden.shape[-1])
    flat_t = labels.reshape(-1).long()
    flat_v = valid.reshape(-1)
    meta = getattr(weight, "_kimi_vocab_parallel", None)
    if meta is not None:
        if label_smoothing:
            raise ValueError("label smoothing is not supported with a vocabulary-parallel head")
        from ..parallel.tensor_parallel import vocab_parallel_linear_cross_entropy
        return vocab_parallel_linear_cross_entropy(flat_h, weight, flat_t, flat_v, vocab_start=meta[0],
                                                   group=meta[3]), None
    if _ops.use_kernels(hidden) and label_smoothing == 0.0:
        return _ops.linear_cross_entropy(flat_h, weight, flat_t, flat_v), None
    logits = F.linear(flat_h, weight).float()
    safe = flat_t.masked_fill(~flat_v, 0)
    per = F.cross_entropy(logits, safe, reduction="none", label_smoothing=label_smoothing)
    return torch.where(flat_v, per, torch.zeros_like(per)).sum(), per


def resolve_component_weights(component_ids, component_weights):
    weights = torch.ones_like(component_ids, dtype=torch.float32)
    if component_weights is None:
        return weights
    if isinstance(component_weights, torch.Tensor):
        return component_weights.float()[component_ids.long()]
    for ident, value in component_weights.items():
        if value < 0 or not math.isfinite(value):
            raise ValueError("component weights must be finite and non-negative")
        weights = torch.where(component_ids.eq(int(ident)), torch.full_like(weights, float(value)), weights)
    return weights


def group_mean_advantages(rewards, group_ids, *, expected_group_size, require_complete_groups):
    """Reward minus its prompt-group mean."""
    if rewards.ndim != 1 or group_ids.shape != rewards.shape:
        raise ValueError("rewards and prompt_group_ids must have shape [B]")
    if group_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("prompt_group_ids must use int32 or int64")
    if not torch.isfinite(rewards).all():
        raise FloatingPointError("rewards contain non-finite values")
    _, inverse, counts = torch.unique(group_ids, sorted=False, return_inverse=True, return_counts=True)
    if require_complete_groups and expected_group_size is not None:
        if expected_group_size <= 0:
            raise ValueError("expected_group_size must be > 0")
        if torch.any(counts != expected_group_size):
            raise ValueError("prompt group is incomplete")
    sums = torch.zeros(counts.numel(), device=rewards.device, dtype=torch.float32)
    sums.scatter_add_(0, inverse, rewards.detach().float())
    return rewards.detach().float() - (sums / counts.float())[inverse]


# --------------------------------------------------------------------------- NTP / MTP
def compute_aligned_cross_entropy(logits, labels, *, alignment, ignore_index, label_smoothing, zero_valid_policy,
                                  attention_mask=None, loss_mask=None, boundary_mask=None, token_weights=None,
                                  return_per_token=False):
    if logits.ndim != 3 or not logits.dtype.is_floating_point or labels.shape != logits.shape[:2]:
        raise ValueError("logits must be floating point [B,T,V] and labels [B,T]")
    sl, al, valid, w = align_token_inputs(logits, labels, alignment=alignment, attention_mask=attention_mask,
                                          loss_mask=loss_mask, boundary_mask=boundary_mask,
                                          token_weights=token_weights, ignore_index=ignore_index)
    validate_token_ids(al, valid, logits.shape[-1])
    safe = al.masked_fill(~valid, 0).long()
    per = F.cross_entropy(logits[:, sl].float().reshape(-1, logits.shape[-1]), safe.reshape(-1), reduction="none",
                          label_smoothing=label_smoothing).reshape_as(safe)
    if torch.any(valid & ~torch.isfinite(per)):
        raise FloatingPointError("cross-entropy produced non-finite valid values")
    return reduce_token_losses(per, valid, w, source=logits, zero_valid_policy=zero_valid_policy,
                               return_per_token=return_per_token)


class NextTokenCrossEntropyLoss(nn.Module):
    def __init__(self, *, ignore_index=-100, label_smoothing=0.0, zero_valid_policy="raise",
                 label_alignment="causal_shift"):
        super().__init__()
        if label_alignment not in ("causal_shift", "already_aligned"):
            raise ValueError("label_alignment must be 'causal_shift' or 'already_aligned'")
        self.ignore_index, self.label_smoothing = ignore_index, float(label_smoothing)
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)
        self.label_alignment = label_alignment

    def forward(self, logits, labels, *, attention_mask=None, loss_mask=None, boundary_mask=None,
                token_weights=None, return_per_token=False) -> TokenCrossEntropyOutput:
        return compute_aligned_cross_entropy(logits, labels, alignment=self.label_alignment,
                                             ignore_index=self.ignore_index, label_smoothing=self.label_smoothing,
                                             zero_valid_policy=self.zero_valid_policy, attention_mask=attention_mask,
                                             loss_mask=loss_mask, boundary_mask=boundary_mask,
                                             token_weights=token_weights, return_per_token=return_per_token)

    def forward_hidden(self, hidden, head_weight, labels, *, attention_mask=None, loss_mask=None,
                       boundary_mask=None, token_weights=None) -> TokenCrossEntropyOutput:
        """Same loss computed from the final hidden state and the LM-head weight."""
        sl, al, valid, w = align_token_inputs(hidden, labels, alignment=self.label_alignment,
                                              attention_mask=attention_mask, loss_mask=loss_mask,
                                              boundary_mask=boundary_mask, token_weights=token_weights,
                                              ignore_index=self.ignore_index)
        validate_token_ids(al, valid, head_vocab_size(head_weight))
        weighted_valid = valid if token_weights is None else valid & (w > 0)
        h = hidden[:, sl]
        if token_weights is not None:
            # Per-token weights: fall back to explicit logits (rare path).
            logits = F.linear(h, head_weight)
            per = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]),
                                  al.masked_fill(~valid, 0).reshape(-1).long(), reduction="none",
                                  label_smoothing=self.label_smoothing).reshape_as(al)
            return reduce_token_losses(per, valid, w, source=hidden, zero_valid_policy=self.zero_valid_policy,
                                       return_per_token=False)
        loss_sum, _ = fused_head_loss(h, head_weight, al, weighted_valid, label_smoothing=self.label_smoothing)
        normalizer = valid.sum().float()
        if not host_checks():
            loss = loss_sum / normalizer.clamp_min(1.0)  # an empty batch gives a connected zero
        elif normalizer.item() == 0:
            if self.zero_valid_policy == "raise":
                raise ValueError("loss batch contains no valid tokens")
            loss = loss_sum = connected_zero(hidden)
        else:
            loss = loss_sum / normalizer
        return TokenCrossEntropyOutput(loss, loss_sum, normalizer.detach(), normalizer.detach())


def canonicalize_mtp_inputs(mtp_logits, mtp_labels, mtp_loss_mask, future_offsets):
    """Accept ``[B,T,V]`` (one depth) or ``[B,D,T,V]``; return the 4-D form."""
    if mtp_logits.ndim == 3:
        mtp_logits = mtp_logits[:, None]
        mtp_labels = mtp_labels[:, None]
        if mtp_loss_mask is not None:
            mtp_loss_mask = mtp_loss_mask[:, None]
    if mtp_logits.ndim != 4 or mtp_labels.shape != mtp_logits.shape[:3]:
        raise ValueError("mtp_logits must be [B,D,T,V] with labels [B,D,T]")
    mask = (torch.ones(mtp_labels.shape, dtype=torch.bool, device=mtp_logits.device) if mtp_loss_mask is None
            else mtp_loss_mask.to(torch.bool))
    depth = mtp_logits.shape[1]
    offsets = tuple(range(2, 2 + depth)) if future_offsets is None else tuple(int(x) for x in
                                                                              (future_offsets.tolist() if isinstance(
                                                                                  future_offsets, torch.Tensor)
                                                                               else future_offsets))
    if len(offsets) != depth:
        raise ValueError("future_offsets must match the number of MTP depths")
    return mtp_logits, mtp_labels, mask, offsets, depth


class MultiTokenPredictionLoss(nn.Module):
    """CE over already-aligned future targets (no shift applied here)."""

    def __init__(self, *, ignore_index=-100, depth_weights: Sequence[float] | None = None,
                 zero_valid_policy="connected_zero"):
        super().__init__()
        if depth_weights is not None and (not depth_weights or any(not math.isfinite(x) or x < 0
                                                                   for x in depth_weights)):
            raise ValueError("depth_weights must be finite and non-negative")
        self.ignore_index = ignore_index
        self.depth_weights = None if depth_weights is None else tuple(float(x) for x in depth_weights)
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)

    def forward(self, mtp_logits, mtp_labels, *, mtp_loss_mask=None, future_offsets=None,
                return_per_depth=False) -> MTPLossOutput:
        logits, labels, mask, offsets, depth = canonicalize_mtp_inputs(mtp_logits, mtp_labels, mtp_loss_mask,
                                                                       future_offsets)
        valid = mask & labels.ne(self.ignore_index)
        validate_token_ids(labels, valid, logits.shape[-1], name="mtp_labels")
        safe = labels.masked_fill(~valid, 0).long()
        per = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), safe.reshape(-1),
                              reduction="none").reshape_as(labels)
        if torch.any(valid & ~torch.isfinite(per)):
            raise FloatingPointError("MTP cross-entropy produced non-finite values")
        if self.depth_weights is not None and len(self.depth_weights) != depth:
            raise ValueError("depth_weights must match the number of MTP depths")
        dw = torch.tensor(self.depth_weights or (1.0,) * depth, dtype=torch.float32, device=logits.device)
        wmask = valid.float() * dw.view(1, depth, 1)
        wl = torch.where(valid, per * dw.view(1, depth, 1), torch.zeros_like(per))
        pds, pdn = wl.sum(dim=(0, 2)), wmask.sum(dim=(0, 2))
        loss_sum, normalizer = pds.sum(), pdn.sum()
        if normalizer.item() == 0:
            if self.zero_valid_policy == "raise":
                raise ValueError("MTP batch contains no valid future targets")
            loss = loss_sum = connected_zero(mtp_logits)
        else:
            loss = loss_sum / normalizer
        return MTPLossOutput(loss, loss_sum, normalizer.detach(), valid.sum().float().detach(),
                             per.detach() if return_per_depth else None, wl.sum((1, 2)).detach(),
                             valid.sum((1, 2)).detach(), pds.detach() if return_per_depth else None,
                             pdn.detach() if return_per_depth else None, offsets)

    def forward_hidden(self, hidden, head_weight, labels, valid_mask, future_offsets=None) -> MTPLossOutput:
        """Single-depth MTP loss from the MTP hidden state (fused head on CUDA)."""
        valid = valid_mask & labels.ne(self.ignore_index)
        validate_token_ids(labels, valid, head_vocab_size(head_weight), name="mtp_labels")
        loss_sum, _ = fused_head_loss(hidden, head_weight, labels, valid)
        normalizer = valid.sum().float()
        if not host_checks():
            loss = loss_sum / normalizer.clamp_min(1.0)
        elif normalizer.item() == 0:
            if self.zero_valid_policy == "raise":
                raise ValueError("MTP batch contains no valid future targets")
            loss = loss_sum = connected_zero(hidden)
        else:
            loss = loss_sum / normalizer
        offsets = (2,) if future_offsets is None else tuple(future_offsets)
        return MTPLossOutput(loss, loss_sum, normalizer.detach(), normalizer.detach(), future_offsets=offsets)


class KimiPretrainingLoss(nn.Module):
    """``NTP + lambda_mtp * MTP``; Stable LatentMoE has no router auxiliary loss."""

    def __init__(self, *, lambda_mtp=0.0, ignore_index=-100, label_smoothing=0.0, label_alignment="causal_shift"):
        super().__init__()
        if lambda_mtp < 0:
            raise ValueError("lambda_mtp must be >= 0")
        self.lambda_mtp = float(lambda_mtp)
        self.ntp_loss = NextTokenCrossEntropyLoss(ignore_index=ignore_index, label_smoothing=label_smoothing,
                                                  label_alignment=label_alignment)
        self.mtp_loss = MultiTokenPredictionLoss(ignore_index=ignore_index)

    def forward(self, *, logits, labels, attention_mask=None, loss_mask=None, boundary_mask=None,
                token_weights=None, mtp_logits=None, mtp_labels=None, mtp_loss_mask=None, future_offsets=None,
                moe_diagnostics=None) -> KimiPretrainingLossOutput:
        ntp = self.ntp_loss(logits, labels, attention_mask=attention_mask, loss_mask=loss_mask,
                            boundary_mask=boundary_mask, token_weights=token_weights)
        if (mtp_logits is None) != (mtp_labels is None):
            raise ValueError("mtp_logits and mtp_labels must be supplied together")
        mtp = (self.mtp_loss(mtp_logits, mtp_labels, mtp_loss_mask=mtp_loss_mask, future_offsets=future_offsets)
               if mtp_logits is not None else None)
        total = ntp.loss if mtp is None else ntp.loss + self.lambda_mtp * mtp.loss
        return KimiPretrainingLossOutput(total, ntp, mtp, self.lambda_mtp, moe_diagnostics)

    def forward_hidden(self, *, hidden, head_weight, labels, attention_mask=None, loss_mask=None,
                       boundary_mask=None, token_weights=None, mtp_hidden=None, mtp_labels=None, mtp_loss_mask=None,
                       future_offsets=None) -> KimiPretrainingLossOutput:
        ntp = self.ntp_loss.forward_hidden(hidden, head_weight, labels, attention_mask=attention_mask,
                                           loss_mask=loss_mask, boundary_mask=boundary_mask,
                                           token_weights=token_weights)
        mtp = (self.mtp_loss.forward_hidden(mtp_hidden, head_weight, mtp_labels, mtp_loss_mask, future_offsets)
               if mtp_hidden is not None else None)
        total = ntp.loss if mtp is None else ntp.loss + self.lambda_mtp * mtp.loss
        return KimiPretrainingLossOutput(total, ntp, mtp, self.lambda_mtp)


# --------------------------------------------------------------------------- SFT / RL / MOPD
class SFTTrajectoryCrossEntropyLoss(nn.Module):
    """Assistant-token CE over trajectories (token- or sequence-mean)."""

    def __init__(self, *, ignore_index=-100, alignment="causal_shift", reduction="token_mean",
                 zero_valid_policy="raise"):
        super().__init__()
        if alignment not in ("causal_shift", "already_aligned") or reduction not in ("token_mean", "sequence_mean"):
            raise ValueError("unsupported SFT alignment or reduction")
        self.ignore_index, self.alignment, self.reduction = ignore_index, alignment, reduction
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)

    def forward(self, logits, labels, *, assistant_mask, attention_mask=None, component_ids=None,
                component_weights=None, boundary_mask=None, sample_weights=None,
                return_per_component=False) -> SFTLossOutput:
        if assistant_mask.shape != labels.shape:
            raise ValueError("assistant_mask must match labels")
        amask = assistant_mask.to(torch.bool)
        weights = torch.ones_like(labels, dtype=torch.float32)
        if component_ids is not None:
            if component_ids.shape != labels.shape:
                raise ValueError("component_ids must match labels")
            weights = resolve_component_weights(component_ids, component_weights)
            amask = amask & component_ids.ne(0)
        elif component_weights is not None:
            raise ValueError("component_weights require component_ids")
        sl, al, valid, aw = align_token_inputs(logits, labels, alignment=self.alignment,
                                               attention_mask=attention_mask, loss_mask=amask,
                                               boundary_mask=boundary_mask, token_weights=weights,
                                               ignore_index=self.ignore_index)
        validate_token_ids(al, valid, logits.shape[-1])
        safe = al.masked_fill(~valid, 0).long()
        per = F.cross_entropy(logits[:, sl].float().reshape(-1, logits.shape[-1]), safe.reshape(-1),
                              reduction="none").reshape_as(al)
        if torch.any(valid & ~torch.isfinite(per)):
            raise FloatingPointError("SFT cross-entropy produced non-finite values")
        tw = aw * valid.float()
        weighted = torch.where(valid, per * aw, torch.zeros_like(per))
        count = valid.sum().float()
        ps, pdn = weighted.sum(-1), tw.sum(-1)
        if sample_weights is None:
            samples = torch.ones(logits.shape[0], dtype=torch.float32, device=logits.device)
        else:
            if tuple(sample_weights.shape) != (logits.shape[0],):
                raise ValueError("sample_weights must have shape [B]")
            samples = sample_weights.float().to(logits.device)
            if not torch.isfinite(samples).all() or torch.any(samples < 0):
                raise ValueError("sample_weights must be finite and non-negative")
        if self.reduction == "token_mean":
            loss_sum = (weighted * samples[:, None]).sum()
            normalizer = (tw * samples[:, None]).sum()
        else:
            active = pdn > 0
            loss_sum = (ps / pdn.clamp_min(1) * samples * active).sum()
            normalizer = (samples * active).sum()
        if normalizer.item() == 0:
            if self.zero_valid_policy == "raise":
                raise ValueError("SFT batch contains no assistant targets")
            loss = loss_sum = connected_zero(logits)
        else:
            loss = loss_sum / normalizer
        csum = ccnt = None
        if return_per_component:
            if component_ids is None:
                raise ValueError("component diagnostics require component_ids")
            ac = component_ids[:, 1:] if self.alignment == "causal_shift" else component_ids
            csum, ccnt = {}, {}
            for ident in torch.unique(ac[valid]).tolist():
                sel = valid & ac.eq(ident)
                csum[int(ident)] = per[sel].sum().detach()
                ccnt[int(ident)] = sel.sum().detach()
        return SFTLossOutput(loss, loss_sum, normalizer.detach(), count.detach(), None, ps.detach(),
                             valid.sum(-1).detach(), csum, ccnt, self.reduction)


class KimiPolicyOptimizationLoss(nn.Module):
    """``-clip(exp(delta), a, b) * A + tau * delta^2`` token-normalised (no critic)."""

    def __init__(self, *, ratio_clip_min, ratio_clip_max, log_ratio_l2_coef, normalize_advantages=False,
                 require_complete_groups=True, zero_valid_policy="raise"):
        super().__init__()
        if not 0 < ratio_clip_min <= ratio_clip_max:
            raise ValueError("ratio bounds must satisfy 0 < min <= max")
        if log_ratio_l2_coef < 0:
            raise ValueError("log_ratio_l2_coef must be >= 0")
        self.ratio_clip_min, self.ratio_clip_max = float(ratio_clip_min), float(ratio_clip_max)
        self.log_ratio_l2_coef = float(log_ratio_l2_coef)
        self.normalize_advantages, self.require_complete_groups = normalize_advantages, require_complete_groups
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)

    def forward(self, *, current_logprobs, old_logprobs, action_mask, rewards=None, prompt_group_ids=None,
                advantages=None, sample_weights=None, expected_group_size=None) -> PolicyOptimizationLossOutput:
        if current_logprobs.ndim != 2 or old_logprobs.shape != current_logprobs.shape:
            raise ValueError("current_logprobs and old_logprobs must have shape [B,T]")
        b, t = current_logprobs.shape
        valid = boolean_mask("action_mask", action_mask, (b, t), current_logprobs.device)
        reward_mode = rewards is not None or prompt_group_ids is not None
        if reward_mode == (advantages is not None):
            raise ValueError("provide exactly rewards+prompt_group_ids or explicit advantages")
        mean_reward = reward_std = None
        if reward_mode:
            if rewards is None or prompt_group_ids is None:
                raise ValueError("rewards and prompt_group_ids are required together")
            adv = group_mean_advantages(rewards, prompt_group_ids, expected_group_size=expected_group_size,
                                        require_complete_groups=self.require_complete_groups)
            mean_reward, reward_std = rewards.detach().float().mean(), rewards.detach().float().std(unbiased=False)
            tok_adv = adv[:, None].expand(b, t)
        else:
            if advantages.shape not in ((b,), (b, t)):
                raise ValueError("advantages must have shape [B] or [B,T]")
            tok_adv = (advantages[:, None].expand(b, t) if advantages.ndim == 1 else advantages).detach().float()
        if self.normalize_advantages:
            sel = tok_adv[valid]
            if sel.numel():
                tok_adv = (tok_adv - sel.mean()) / sel.std(unbiased=False).clamp_min(1e-6)
        if sample_weights is None:
            w = torch.ones((b, 1), device=current_logprobs.device)
        else:
            if tuple(sample_weights.shape) != (b,):
                raise ValueError("sample_weights must have shape [B]")
            w = sample_weights.detach().float()[:, None]
            if not torch.isfinite(w).all() or torch.any(w < 0):
                raise ValueError("sample_weights must be finite and non-negative")
        normalizer = (valid.float() * w).sum(dtype=torch.float32)
        cur, old = current_logprobs.float(), old_logprobs.detach().float()
        require_finite("current_logprobs", cur, valid)
        require_finite("old_logprobs", old, valid)
        require_finite("advantages", tok_adv, valid)
        lr = cur - old
        lo, hi = math.log(self.ratio_clip_min), math.log(self.ratio_clip_max)
        pterm = torch.exp(lr.clamp(lo, hi)) * tok_adv
        rterm = self.log_ratio_l2_coef * lr.square()
        psum = torch.where(valid, pterm * w, torch.zeros_like(pterm)).sum()
        rsum = torch.where(valid, rterm * w, torch.zeros_like(rterm)).sum()
        loss_sum = -psum + rsum
        if normalizer.item() == 0:
            if self.zero_valid_policy == "raise":
                raise ValueError("RL batch contains no action tokens")
            loss = loss_sum = connected_zero(current_logprobs)
        else:
            loss = loss_sum / normalizer
        sr, sa = lr[valid], tok_adv[valid]
        zero = cur.detach().new_zeros(())
        clipped = valid & ((lr < lo) | (lr > hi))
        return PolicyOptimizationLossOutput(
            loss, loss_sum, normalizer.detach(), valid.sum().float().detach(), psum.detach(), rsum.detach(),
            sa.mean().detach() if sa.numel() else zero, sr.mean().detach() if sr.numel() else zero,
            sr.abs().max().detach() if sr.numel() else zero,
            clipped[valid].float().mean().detach() if torch.any(valid) else zero,
            None if mean_reward is None else mean_reward.detach(), None if reward_std is None else reward_std.detach())


def validate_teacher_ids(teacher_ids, batch_size, device):
    if teacher_ids.device != device:
        raise ValueError("teacher_ids must share the student device")
    if teacher_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("teacher_ids must use int32 or int64")
    if tuple(teacher_ids.shape) == (batch_size,):
        if torch.any((teacher_ids < 0) | (teacher_ids >= 9)):
            raise ValueError("flat teacher IDs must be in [0, 9)")
        return
    if tuple(teacher_ids.shape) == (batch_size, 2):
        if torch.any((teacher_ids < 0) | (teacher_ids >= 3)):
            raise ValueError("domain/effort IDs must each be in [0, 3)")
        return
    raise ValueError("teacher_ids must have shape [B] or [B,2]")


def clipped_teacher_student_reward(teacher_logprobs, student_reference_logprobs, reward_clip_max):
    raw = teacher_logprobs.detach().float() - student_reference_logprobs.detach().float()
    return raw.clamp(-reward_clip_max, reward_clip_max).detach(), raw.abs() > reward_clip_max


def corrected_topk_reverse_kl(teacher_logprobs, student_logprobs):
    t, s = teacher_logprobs.detach().float(), student_logprobs.float()
    sp = s.exp()
    return (sp * (s - t) - sp + t.exp()).sum(-1)


class MultiTeacherOnPolicyDistillationLoss(nn.Module):
    """Multi-teacher on-policy distillation: sampled-token PG, Kimi-regularised, or corrected Top-k RKL."""

    MODES = ("sampled_token_pg", "kimi_rl_regularized", "topk_reverse_kl")

    def __init__(self, *, reward_clip_max, mode="sampled_token_pg", policy_loss=None, zero_valid_policy="raise"):
        super().__init__()
        if reward_clip_max <= 0:
            raise ValueError("reward_clip_max must be > 0")
        if mode not in self.MODES:
            raise ValueError("unsupported MOPD mode")
        if mode == "kimi_rl_regularized" and policy_loss is None:
            raise ValueError("regularized MOPD requires KimiPolicyOptimizationLoss")
        self.reward_clip_max, self.mode, self.policy_loss = float(reward_clip_max), mode, policy_loss
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)

    def forward(self, *, current_student_logprobs, teacher_sampled_token_logprobs, action_mask, teacher_ids,
                student_logprobs_for_reward=None, old_student_logprobs=None, teacher_topk_token_ids=None,
                teacher_topk_logprobs=None, student_topk_logprobs=None, sampled_token_ids=None,
                teacher_sampled_token_ids=None) -> MOPDLossOutput:
        if current_student_logprobs.ndim != 2:
            raise ValueError("current_student_logprobs must have shape [B,T]")
        b, t = current_student_logprobs.shape
        dev = current_student_logprobs.device
        valid = boolean_mask("action_mask", action_mask, (b, t), dev)
        validate_teacher_ids(teacher_ids, b, dev)
        if (sampled_token_ids is None) != (teacher_sampled_token_ids is None):
            raise ValueError("both sampled-token metadata tensors are required")
        if sampled_token_ids is not None and (tuple(sampled_token_ids.shape) != (b, t)
                                              or tuple(teacher_sampled_token_ids.shape) != (b, t)
                                              or torch.any(sampled_token_ids[valid] != teacher_sampled_token_ids[valid])):
            raise ValueError("teacher/student tokenization metadata mismatch")
        normalizer = valid.sum().float()
        if normalizer.item() == 0 and self.zero_valid_policy == "raise":
            raise ValueError("MOPD batch contains no sampled action tokens")
        cur = current_student_logprobs.float()
        require_finite("current_student_logprobs", cur, valid)
        policy_output = None
        if self.mode == "topk_reverse_kl":
            if any(v is None for v in (teacher_topk_token_ids, teacher_topk_logprobs, student_topk_logprobs)):
                raise ValueError("Top-k mode requires token IDs and both logprobs")
            if (teacher_topk_token_ids.shape[:2] != (b, t) or teacher_topk_logprobs.shape != teacher_topk_token_ids.shape
                    or student_topk_logprobs.shape != teacher_topk_token_ids.shape):
                raise ValueError("Top-k tensors must have shape [B,T,K]")
            srt = teacher_topk_token_ids.sort(-1).values
            if torch.any(srt[..., 1:] == srt[..., :-1]):
                raise ValueError("teacher Top-k token IDs must be unique per token")
            per = corrected_topk_reverse_kl(teacher_topk_logprobs, student_topk_logprobs)
            require_finite("topk_reverse_kl", per, valid)
            loss_sum = torch.where(valid, per, torch.zeros_like(per)).sum()
            loss = loss_sum / normalizer if normalizer.item() else connected_zero(student_topk_logprobs)
            tv, sv = teacher_topk_logprobs.detach().float(), student_topk_logprobs.detach().float()
            reward, clipped = torch.zeros_like(cur), torch.zeros_like(valid)
            ref = "topk_distribution"
            mt = tv.mean(-1)[valid].mean() if torch.any(valid) else tv.new_zeros(())
            ms = sv.mean(-1)[valid].mean() if torch.any(valid) else sv.new_zeros(())
        else:
            if teacher_sampled_token_logprobs is None or tuple(teacher_sampled_token_logprobs.shape) != (b, t):
                raise ValueError("sampled MOPD requires teacher logprobs [B,T]")
            tv = teacher_sampled_token_logprobs.detach().float()
            require_finite("teacher_logprobs", tv, valid)
            if student_logprobs_for_reward is None:
                sv, ref = cur.detach(), "current_detached"
            else:
                if tuple(student_logprobs_for_reward.shape) != (b, t):
                    raise ValueError("stored student logprobs must have shape [B,T]")
                sv, ref = student_logprobs_for_reward.detach().float(), "rollout_stored"
            require_finite("student_reward_reference", sv, valid)
            reward, clipped = clipped_teacher_student_reward(tv, sv, self.reward_clip_max)
            if self.mode == "sampled_token_pg":
                loss_sum = -torch.where(valid, reward * cur, torch.zeros_like(cur)).sum()
                loss = loss_sum / normalizer if normalizer.item() else connected_zero(current_student_logprobs)
            else:
                if old_student_logprobs is None:
                    raise ValueError("regularized MOPD requires old_student_logprobs")
                policy_output = self.policy_loss(current_logprobs=current_student_logprobs,
                                                 old_logprobs=old_student_logprobs, action_mask=valid,
                                                 advantages=reward)
                loss, loss_sum = policy_output.loss, policy_output.loss_sum
            mt = tv[valid].mean() if torch.any(valid) else tv.new_zeros(())
            ms = sv[valid].mean() if torch.any(valid) else sv.new_zeros(())
        zero = cur.detach().new_zeros(())
        return MOPDLossOutput(loss, loss_sum, normalizer.detach(), normalizer.detach(),
                              reward[valid].mean().detach() if torch.any(valid) else zero,
                              clipped[valid].float().mean().detach() if torch.any(valid) else zero,
                              mt.detach(), ms.detach(), (mt - ms).detach(), normalizer.detach(), self.mode, ref,
                              policy_output)


class KimiRewardComposer:
    """Explicitly weighted, detached sum of verifier / generative / task rewards."""

    def __call__(self, *, verifier_reward, generative_reward, task_specific_reward, weights: RewardWeights):
        sources = (("verifier", verifier_reward, weights.verifier), ("generative", generative_reward, weights.generative),
                   ("task_specific", task_specific_reward, weights.task_specific))
        present = [s for s in sources if s[1] is not None]
        if not present:
            raise ValueError("at least one reward source is required")
        shape = present[0][1].shape
        if len(shape) != 1:
            raise ValueError("reward sources must have shape [B]")
        out = torch.zeros_like(present[0][1], dtype=torch.float32)
        for name, value, weight in sources:
            if value is None:
                if weight is not None:
                    raise ValueError(f"{name} weight was supplied without its reward")
                continue
            if weight is None:
                raise ValueError(f"{name} reward requires an explicit weight")
            if value.shape != shape:
                raise ValueError("all reward sources must share shape and device")
            if not torch.isfinite(value).all():
                raise FloatingPointError(f"{name} reward contains non-finite values")
            out = out + float(weight) * value.detach().float()
        return out.detach()


def apply_reasoning_budget_override(reward, used_tokens, base_budget, budget_multiplier, penalty_reward=-1.0):
    if reward.ndim != 1 or used_tokens.shape != reward.shape or base_budget.shape != reward.shape:
        raise ValueError("reward, used_tokens and base_budget must have shape [B]")
    if budget_multiplier <= 0:
        raise ValueError("budget_multiplier must be > 0")
    if torch.any(used_tokens < 0) or torch.any(base_budget < 0):
        raise ValueError("token counts and budgets must be non-negative")
    exceeded = used_tokens.float() > float(budget_multiplier) * base_budget.float()
    return torch.where(exceeded, torch.full_like(reward.float(), float(penalty_reward)), reward.detach().float()).detach()


def apply_verbosity_binary_rule(wins, output_length, initial_verbosity, sigma):
    if wins.dtype != torch.bool:
        raise TypeError("wins must be boolean")
    if output_length.shape != wins.shape or initial_verbosity.shape != wins.shape:
        raise ValueError("verbosity inputs must share shape")
    if sigma <= 0:
        raise ValueError("sigma must be > 0")
    return (wins & ~(output_length.float() > sigma * initial_verbosity.float())).detach()


# --------------------------------------------------------------------------- objective
@dataclass(frozen=True)
class KimiLossConfig:
    ignore_index: int = -100
    label_smoothing: float = 0.0
    lambda_mtp: float = 0.0
    sft_reduction: str = "token_mean"
    rl_ratio_clip_min: float | None = None
    rl_ratio_clip_max: float | None = None
    rl_log_ratio_l2_coef: float | None = None
    rl_normalize_advantages: bool = False
    mopd_reward_clip_max: float | None = None
    mopd_mode: str = "sampled_token_pg"
    compute_loss_in_fp32: bool = True

    def __post_init__(self) -> None:
        if self.ignore_index >= 0:
            raise ValueError("ignore_index must be outside the non-negative vocabulary")
        if not 0.0 <= self.label_smoothing < 1.0 or self.lambda_mtp < 0:
            raise ValueError("invalid label_smoothing or lambda_mtp")
        if self.sft_reduction not in ("token_mean", "sequence_mean"):
            raise ValueError("unsupported SFT reduction")
        if self.rl_log_ratio_l2_coef is not None and self.rl_log_ratio_l2_coef < 0:
            raise ValueError("rl_log_ratio_l2_coef must be >= 0")
        if self.mopd_reward_clip_max is not None and self.mopd_reward_clip_max <= 0:
            raise ValueError("mopd_reward_clip_max must be > 0")
        if (self.rl_ratio_clip_min is None) != (self.rl_ratio_clip_max is None):
            raise ValueError("both RL ratio bounds must be provided together")
        if self.rl_ratio_clip_min is not None and not 0 < self.rl_ratio_clip_min <= self.rl_ratio_clip_max:
            raise ValueError("RL ratio bounds must satisfy 0 < min <= max")
        if self.mopd_mode not in MultiTeacherOnPolicyDistillationLoss.MODES:
            raise ValueError("unsupported MOPD mode")
        if not self.compute_loss_in_fp32:
            raise ValueError("losses are computed in fp32")

    def require_posttraining_values(self) -> None:
        if any(v is None for v in (self.rl_ratio_clip_min, self.rl_ratio_clip_max, self.rl_log_ratio_l2_coef,
                                   self.mopd_reward_clip_max)):
            raise ValueError("RL and MOPD values must be provided explicitly before building post-training objectives")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "KimiLossConfig":
        return cls(**values)


_PHASE_KEYS = {
    KimiTrainingPhase.PRETRAIN: {"logits", "labels", "attention_mask", "loss_mask", "boundary_mask", "token_weights",
                                 "mtp_logits", "mtp_labels", "mtp_loss_mask", "future_offsets", "moe_diagnostics"},
    KimiTrainingPhase.SFT: {"logits", "labels", "assistant_mask", "attention_mask", "component_ids",
                            "component_weights", "boundary_mask", "sample_weights", "return_per_component"},
    KimiTrainingPhase.RL: {"current_logprobs", "old_logprobs", "action_mask", "rewards", "prompt_group_ids",
                           "advantages", "sample_weights", "expected_group_size"},
    KimiTrainingPhase.MOPD: {"current_student_logprobs", "teacher_sampled_token_logprobs", "action_mask",
                             "teacher_ids", "student_logprobs_for_reward", "old_student_logprobs",
                             "teacher_topk_token_ids", "teacher_topk_logprobs", "student_topk_logprobs",
                             "sampled_token_ids", "teacher_sampled_token_ids"},
}


class KimiTrainingObjective(nn.Module):
    """Strict per-phase dispatcher; unknown keys for a phase raise."""

    def __init__(self, config: KimiLossConfig):
        super().__init__()
        self.config = config
        self.pretrain = KimiPretrainingLoss(lambda_mtp=config.lambda_mtp, ignore_index=config.ignore_index,
                                            label_smoothing=config.label_smoothing)
        self.sft = SFTTrajectoryCrossEntropyLoss(ignore_index=config.ignore_index, reduction=config.sft_reduction)
        self.rl = self.mopd = None
        if config.rl_ratio_clip_min is not None and config.rl_log_ratio_l2_coef is not None:
            self.rl = KimiPolicyOptimizationLoss(ratio_clip_min=config.rl_ratio_clip_min,
                                                 ratio_clip_max=config.rl_ratio_clip_max,
                                                 log_ratio_l2_coef=config.rl_log_ratio_l2_coef,
                                                 normalize_advantages=config.rl_normalize_advantages)
        if config.mopd_reward_clip_max is not None:
            self.mopd = MultiTeacherOnPolicyDistillationLoss(reward_clip_max=config.mopd_reward_clip_max,
                                                             mode=config.mopd_mode, policy_loss=self.rl)

    def forward(self, phase, **inputs) -> KimiLossBundle:
        phase = KimiTrainingPhase(phase)
        unknown = set(inputs) - _PHASE_KEYS[phase]
        if unknown:
            raise ValueError(f"unexpected inputs for phase {phase.value}: {sorted(unknown)}")
        module = {KimiTrainingPhase.PRETRAIN: self.pretrain, KimiTrainingPhase.SFT: self.sft,
                  KimiTrainingPhase.RL: self.rl, KimiTrainingPhase.MOPD: self.mopd}[phase]
        if module is None:
            self.config.require_posttraining_values()
        if phase == KimiTrainingPhase.SFT:
            out = module(inputs.pop("logits"), inputs.pop("labels"), **inputs)
        elif phase == KimiTrainingPhase.PRETRAIN:
            out = module(**inputs)
        else:
            out = module(**inputs)
        return KimiLossBundle(phase, out.loss, out)


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "math", "torch", "nn", "F")]
