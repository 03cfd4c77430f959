"""Token losses: NTP, MTP and the pretraining composite, with the shared token helpers.

Parity targets (reference paths):
  * ``src/loss/common/reduction.py:10-51``, ``common/validation.py:14-127``
  * ``src/loss/pretraining/cross_entropy.py:13-57``, ``next_token_loss.py``
  * ``src/loss/multi_token_prediction_loss.py:18-105``
  * ``src/loss/pretraining/composite.py:12-77``  (NTP + lambda * MTP, no router loss)
  (the post-training objectives -- SFT, the Kimi policy loss, MOPD, rewards and the per-phase
  dispatcher -- live in ``posttrain.py``)

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
                 label_alignment="causal_shift", alignment=None):
        """``alignment`` is the reference's name for ``label_alignment`` and may be used instead."""
        super().__init__()
        if alignment is not None:
            if label_alignment not in ("causal_shift", alignment):
                raise ValueError("alignment and label_alignment disagree")
            label_alignment = alignment
        if label_alignment not in ("causal_shift", "already_aligned"):
            raise ValueError("label_alignment must be 'causal_shift' or 'already_aligned'")
        if not 0.0 <= float(label_smoothing) < 1.0:
            raise ValueError("label_smoothing must be in [0, 1)")
        self.ignore_index, self.label_smoothing = ignore_index, float(label_smoothing)
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)
        self.label_alignment = label_alignment

    @property
    def alignment(self) -> str:
        return self.label_alignment

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


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "math", "torch", "nn", "F")]
