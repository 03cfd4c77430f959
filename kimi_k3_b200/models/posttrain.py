"""Post-training objectives: SFT trajectory cross-entropy, the Kimi policy loss, multi-teacher
on-policy distillation (MOPD), reward shaping, and the per-phase objective dispatcher.

Written from the loss contract (the equations and modes below), not from an implementation:

* SFT: mean negative log-likelihood of the assistant-selected target tokens, weighted per
  trajectory component, reduced per token (default) or per sequence.
* Kimi policy loss, per action token with ``d = log pi - log pi_old``:
  ``-exp(clamp(d, log a, log b)) * A + tau * d^2`` (the ratio is clipped in log space before
  ``exp``; the L2 penalty sees the unclipped ``d``); advantages are rewards minus their exact
  prompt-group mean.  No critic, no PPO minimum.
* MOPD reward per sampled token: ``clamp(stopgrad(log p_teacher - log p_student_ref), -R, R)``;
  modes: sampled-token policy gradient ``-r * log pi``, the Kimi policy loss with ``A = r``
  (regularised stale rollouts), and a corrected Top-k reverse KL
  ``sum_k p_s (log p_s - log p_t) - p_s + p_t`` (the KL between the unnormalised restrictions of
  both distributions to the teacher's Top-k tokens).
* Every loss returns ``loss``, ``loss_sum``, ``normalizer`` and ``num_valid_tokens`` so a data
  parallel trainer can re-normalise sums globally; none performs a collective.

The class names, constructor arguments and output fields are the reference's public interface
(``src/loss/sft_loss.py``, ``policy_optimization_loss.py``, ``mopd_loss.py``,
``rl/reward_processing.py``, ``training_objective.py``, ``common/config.py``), kept so callers
switch without edits.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass

import torch
import torch.nn as nn

from .losses import (KimiLossBundle, KimiPretrainingLoss, KimiTrainingPhase, MOPDLossOutput,
                     PolicyOptimizationLossOutput, RewardWeights, SFTLossOutput, align_token_inputs, boolean_mask,
                     connected_zero, group_mean_advantages, resolve_component_weights, validate_token_ids,
                     validate_zero_policy)


# --------------------------------------------------------------------------- shared pieces
class _TokenSelection:
    """The valid action/target tokens of a ``[B, T]`` batch and each token's weight."""

    def __init__(self, valid: torch.Tensor, weight: torch.Tensor):
        self.valid = valid
        self.weight = torch.where(valid, weight.float(), torch.zeros_like(weight, dtype=torch.float32))

    def weighted_sum(self, per_token: torch.Tensor) -> torch.Tensor:
        return torch.where(self.valid, per_token * self.weight, torch.zeros_like(per_token)).sum()

    def normalizer(self) -> torch.Tensor:
        return self.weight.sum()

    def count(self) -> torch.Tensor:
        return self.valid.sum().float()

    def mean(self, per_token: torch.Tensor) -> torch.Tensor:
        """Unweighted mean over the valid tokens (a detached zero when there are none)."""
        picked = per_token.detach()[self.valid]
        return picked.mean() if picked.numel() else per_token.detach().new_zeros(())


def _row_weights(sample_weights, batch: int, device) -> torch.Tensor:
    if sample_weights is None:
        return torch.ones(batch, dtype=torch.float32, device=device)
    if tuple(sample_weights.shape) != (batch,):
        raise ValueError("sample_weights must have shape [B]")
    w = sample_weights.detach().float().to(device)
    if not bool(torch.isfinite(w).all()) or bool((w < 0).any()):
        raise ValueError("sample_weights must be finite and non-negative")
    return w


def _finite_where_valid(name: str, values: torch.Tensor, valid: torch.Tensor) -> None:
    n_bad = int((valid & ~torch.isfinite(values)).sum())
    if n_bad:
        raise FloatingPointError(f"{name}: {n_bad} valid entries are not finite")


def _normalise(loss_sum, normalizer, policy: str, empty_message: str, anchor: torch.Tensor):
    """``loss_sum / normalizer``; an empty batch raises or yields a graph-connected zero."""
    if float(normalizer) == 0.0:
        if policy == "raise":
            raise ValueError(empty_message)
        zero = connected_zero(anchor)
        return zero, zero
    return loss_sum / normalizer, loss_sum


# --------------------------------------------------------------------------- SFT
class SFTTrajectoryCrossEntropyLoss(nn.Module):
    """Cross-entropy on the assistant-selected tokens of agentic trajectories."""

    def __init__(self, *, ignore_index=-100, alignment="causal_shift", reduction="token_mean",
                 zero_valid_policy="raise"):
        super().__init__()
        if alignment not in ("causal_shift", "already_aligned"):
            raise ValueError(f"unsupported SFT alignment {alignment!r}")
        if reduction not in ("token_mean", "sequence_mean"):
            raise ValueError(f"unsupported SFT reduction {reduction!r}")
        self.ignore_index, self.alignment, self.reduction = ignore_index, alignment, reduction
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)

    def forward(self, logits, labels, *, assistant_mask, attention_mask=None, component_ids=None,
                component_weights=None, boundary_mask=None, sample_weights=None,
                return_per_component=False) -> SFTLossOutput:
        if assistant_mask.shape != labels.shape:
            raise ValueError("assistant_mask must have the shape of labels")
        selected = assistant_mask.to(torch.bool)
        if component_ids is None:
            if component_weights is not None:
                raise ValueError("component_weights need component_ids")
            comp_w = torch.ones(labels.shape, dtype=torch.float32, device=labels.device)
        else:
            if component_ids.shape != labels.shape:
                raise ValueError("component_ids must have the shape of labels")
            comp_w = resolve_component_weights(component_ids, component_weights)
            selected = selected & (component_ids != 0)  # component 0 is context
        cols, targets, valid, tok_w = align_token_inputs(
            logits, labels, alignment=self.alignment, attention_mask=attention_mask, loss_mask=selected,
            boundary_mask=boundary_mask, token_weights=comp_w, ignore_index=self.ignore_index)
        validate_token_ids(targets, valid, logits.shape[-1])
        logp = torch.log_softmax(logits[:, cols].float(), dim=-1)
        nll = -logp.gather(-1, targets.masked_fill(~valid, 0).long().unsqueeze(-1)).squeeze(-1)
        _finite_where_valid("SFT token losses", nll, valid)
        rows = _row_weights(sample_weights, logits.shape[0], logits.device)
        tokens = _TokenSelection(valid, tok_w)
        per_row_sum = torch.where(valid, nll * tokens.weight, torch.zeros_like(nll)).sum(-1)
        per_row_norm = tokens.weight.sum(-1)
        if self.reduction == "token_mean":
            loss_sum = (per_row_sum * rows).sum()
            normalizer = (per_row_norm * rows).sum()
        else:  # each sequence with targets counts once
            has_targets = (per_row_norm > 0).float()
            loss_sum = (per_row_sum / per_row_norm.clamp_min(1) * rows * has_targets).sum()
            normalizer = (rows * has_targets).sum()
        loss, loss_sum = _normalise(loss_sum, normalizer, self.zero_valid_policy,
                                    "SFT batch has no assistant target tokens", logits)
        comp_sum = comp_cnt = None
        if return_per_component:
            if component_ids is None:
                raise ValueError("per-component diagnostics need component_ids")
            aligned = component_ids[:, 1:] if self.alignment == "causal_shift" else component_ids
            comp_sum, comp_cnt = {}, {}
            for ident in sorted(set(aligned[valid].tolist())):
                where = valid & (aligned == ident)
                comp_sum[int(ident)] = nll[where].sum().detach()
                comp_cnt[int(ident)] = where.sum().detach()
        return SFTLossOutput(loss, loss_sum, normalizer.detach(), tokens.count().detach(), None,
                             per_row_sum.detach(), valid.sum(-1).detach(), comp_sum, comp_cnt, self.reduction)


# --------------------------------------------------------------------------- Kimi policy loss
class KimiPolicyOptimizationLoss(nn.Module):
    """Clipped-ratio policy gradient with a log-ratio L2 penalty, token normalised."""

    def __init__(self, *, ratio_clip_min, ratio_clip_max, log_ratio_l2_coef, normalize_advantages=False,
                 require_complete_groups=True, zero_valid_policy="raise"):
        super().__init__()
        if not (0 < ratio_clip_min <= ratio_clip_max):
            raise ValueError("ratio clip bounds need 0 < min <= max")
        if log_ratio_l2_coef < 0:
            raise ValueError("log_ratio_l2_coef must be non-negative")
        self.ratio_clip_min, self.ratio_clip_max = float(ratio_clip_min), float(ratio_clip_max)
        self.log_ratio_l2_coef = float(log_ratio_l2_coef)
        self.normalize_advantages, self.require_complete_groups = normalize_advantages, require_complete_groups
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)

    def _token_advantages(self, b, t, rewards, prompt_group_ids, advantages, expected_group_size):
        from_rewards = rewards is not None or prompt_group_ids is not None
        if from_rewards == (advantages is not None):
            raise ValueError("give either rewards with prompt_group_ids, or explicit advantages")
        if not from_rewards:
            if advantages.shape not in ((b,), (b, t)):
                raise ValueError("advantages must have shape [B] or [B,T]")
            adv = advantages.detach().float()
            return (adv[:, None].expand(b, t) if adv.ndim == 1 else adv), None, None
        if rewards is None or prompt_group_ids is None:
            raise ValueError("rewards and prompt_group_ids go together")
        per_sample = group_mean_advantages(rewards, prompt_group_ids, expected_group_size=expected_group_size,
                                           require_complete_groups=self.require_complete_groups)
        r = rewards.detach().float()
        return per_sample[:, None].expand(b, t), r.mean(), r.std(unbiased=False)

    def forward(self, *, current_logprobs, old_logprobs, action_mask, rewards=None, prompt_group_ids=None,
                advantages=None, sample_weights=None, expected_group_size=None) -> PolicyOptimizationLossOutput:
        if current_logprobs.ndim != 2 or old_logprobs.shape != current_logprobs.shape:
            raise ValueError("current_logprobs and old_logprobs must both be [B,T]")
        b, t = current_logprobs.shape
        dev = current_logprobs.device
        valid = boolean_mask("action_mask", action_mask, (b, t), dev)
        adv, reward_mean, reward_std = self._token_advantages(b, t, rewards, prompt_group_ids, advantages,
                                                              expected_group_size)
        if self.normalize_advantages and bool(valid.any()):
            chosen = adv[valid]
            adv = (adv - chosen.mean()) / chosen.std(unbiased=False).clamp_min(1e-6)
        rows = _row_weights(sample_weights, b, dev)
        tokens = _TokenSelection(valid, rows[:, None].expand(b, t))
        logp, logp_old = current_logprobs.float(), old_logprobs.detach().float()
        for name, val in (("current_logprobs", logp), ("old_logprobs", logp_old), ("advantages", adv)):
            _finite_where_valid(name, val, valid)
        delta = logp - logp_old
        lo, hi = math.log(self.ratio_clip_min), math.log(self.ratio_clip_max)
        surrogate = delta.clamp(lo, hi).exp() * adv
        penalty = self.log_ratio_l2_coef * delta.square()
        surrogate_sum, penalty_sum = tokens.weighted_sum(surrogate), tokens.weighted_sum(penalty)
        loss, loss_sum = _normalise(penalty_sum - surrogate_sum, tokens.normalizer(), self.zero_valid_policy,
                                    "RL batch has no action tokens", current_logprobs)
        outside = ((delta < lo) | (delta > hi)).float()
        chosen_delta = delta.detach()[valid]
        max_abs = chosen_delta.abs().max() if chosen_delta.numel() else delta.detach().new_zeros(())
        return PolicyOptimizationLossOutput(
            loss, loss_sum, tokens.normalizer().detach(), tokens.count().detach(), surrogate_sum.detach(),
            penalty_sum.detach(), tokens.mean(adv), tokens.mean(delta), max_abs, tokens.mean(outside),
            None if reward_mean is None else reward_mean.detach(), None if reward_std is None else reward_std.detach())


# --------------------------------------------------------------------------- MOPD
_DOMAINS, _EFFORTS = 3, 3


def validate_teacher_ids(teacher_ids, batch_size, device):
    """One teacher per sample: a flat id in [0, 9) or a (domain, effort) pair, each in [0, 3)."""
    if teacher_ids.device != device:
        raise ValueError("teacher IDs must live on the student device")
    if teacher_ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("teacher IDs must be int32 or int64")
    shape = tuple(teacher_ids.shape)
    if shape == (batch_size,):
        upper = _DOMAINS * _EFFORTS
    elif shape == (batch_size, 2):
        upper = _DOMAINS
    else:
        raise ValueError("teacher IDs must have shape [B] or [B,2]")
    if bool(((teacher_ids < 0) | (teacher_ids >= upper)).any()):
        raise ValueError(f"teacher IDs out of range [0, {upper})")


def clipped_teacher_student_reward(teacher_logprobs, student_reference_logprobs, reward_clip_max):
    """The MOPD token reward (no gradient) and where the clamp bit."""
    gap = (teacher_logprobs.detach().float() - student_reference_logprobs.detach().float())
    return gap.clamp(-reward_clip_max, reward_clip_max), gap.abs() > reward_clip_max


def corrected_topk_reverse_kl(teacher_logprobs, student_logprobs):
    """``sum_k p_s (log p_s - log p_t) - p_s + p_t`` over the Top-k tokens (teacher side detached)."""
    log_t, log_s = teacher_logprobs.detach().float(), student_logprobs.float()
    p_s, p_t = log_s.exp(), log_t.exp()
    return (p_s * (log_s - log_t) + p_t - p_s).sum(-1)


class MultiTeacherOnPolicyDistillationLoss(nn.Module):
    """On-policy distillation from one teacher per sample (sampled-token PG, Kimi-regularised, or
    corrected Top-k reverse KL)."""

    MODES = ("sampled_token_pg", "kimi_rl_regularized", "topk_reverse_kl")

    def __init__(self, *, reward_clip_max, mode="sampled_token_pg", policy_loss=None, zero_valid_policy="raise"):
        super().__init__()
        if reward_clip_max <= 0:
            raise ValueError("reward_clip_max must be positive")
        if mode not in self.MODES:
            raise ValueError(f"unsupported MOPD mode {mode!r}")
        if mode == "kimi_rl_regularized" and policy_loss is None:
            raise ValueError("the regularized mode needs a KimiPolicyOptimizationLoss")
        self.reward_clip_max, self.mode, self.policy_loss = float(reward_clip_max), mode, policy_loss
        self.zero_valid_policy = validate_zero_policy(zero_valid_policy)

    def _topk(self, tokens, logp, ids, teacher_lp, student_lp):
        b, t = logp.shape
        if ids is None or teacher_lp is None or student_lp is None:
            raise ValueError("Top-k mode needs the Top-k token IDs and both Top-k logprobs")
        if ids.shape[:2] != (b, t) or teacher_lp.shape != ids.shape or student_lp.shape != ids.shape:
            raise ValueError("Top-k tensors must all have shape [B,T,K]")
        ordered = ids.sort(-1).values
        if bool((ordered[..., 1:] == ordered[..., :-1]).any()):
            raise ValueError("teacher Top-k token IDs repeat within a token")
        per_token = corrected_topk_reverse_kl(teacher_lp, student_lp)
        _finite_where_valid("Top-k reverse KL", per_token, tokens.valid)
        loss, loss_sum = _normalise(tokens.weighted_sum(per_token), tokens.normalizer(), "connected_zero", "",
                                    student_lp)
        zeros = torch.zeros_like(logp)
        stats = (zeros, torch.zeros_like(tokens.valid), tokens.mean(teacher_lp.float().mean(-1)),
                 tokens.mean(student_lp.float().mean(-1)))
        return loss, loss_sum, None, "topk_distribution", stats

    def _sampled(self, tokens, logp, teacher_lp, stored_student_lp, old_student_lp, current):
        b, t = logp.shape
        if teacher_lp is None or tuple(teacher_lp.shape) != (b, t):
            raise ValueError("sampled-token MOPD needs teacher logprobs of shape [B,T]")
        teacher = teacher_lp.detach().float()
        _finite_where_valid("teacher logprobs", teacher, tokens.valid)
        if stored_student_lp is None:
            reference, source = logp.detach(), "current_detached"
        else:
            if tuple(stored_student_lp.shape) != (b, t):
                raise ValueError("stored student logprobs must have shape [B,T]")
            reference, source = stored_student_lp.detach().float(), "rollout_stored"
        _finite_where_valid("student reward reference", reference, tokens.valid)
        reward, clipped = clipped_teacher_student_reward(teacher, reference, self.reward_clip_max)
        policy_out = None
        if self.mode == "sampled_token_pg":
            loss, loss_sum = _normalise(-tokens.weighted_sum(reward * logp), tokens.normalizer(), "connected_zero",
                                        "", current)
        else:
            if old_student_lp is None:
                raise ValueError("the regularized mode needs old_student_logprobs")
            policy_out = self.policy_loss(current_logprobs=current, old_logprobs=old_student_lp,
                                          action_mask=tokens.valid, advantages=reward)
            loss, loss_sum = policy_out.loss, policy_out.loss_sum
        stats = (reward, clipped, tokens.mean(teacher), tokens.mean(reference))
        return loss, loss_sum, policy_out, source, stats

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
            raise ValueError("sampled-token tokenization check needs both id tensors")
        if sampled_token_ids is not None:
            if tuple(sampled_token_ids.shape) != (b, t) or tuple(teacher_sampled_token_ids.shape) != (b, t) or \
                    bool((sampled_token_ids[valid] != teacher_sampled_token_ids[valid]).any()):
                raise ValueError("teacher and student tokenization disagree on sampled tokens")
        tokens = _TokenSelection(valid, torch.ones((b, t), dtype=torch.float32, device=dev))
        if float(tokens.normalizer()) == 0.0 and self.zero_valid_policy == "raise":
            raise ValueError("MOPD batch has no sampled action tokens")
        logp = current_student_logprobs.float()
        _finite_where_valid("current student logprobs", logp, valid)
        if self.mode == "topk_reverse_kl":
            loss, loss_sum, policy_out, source, stats = self._topk(tokens, logp, teacher_topk_token_ids,
                                                                   teacher_topk_logprobs, student_topk_logprobs)
        else:
            loss, loss_sum, policy_out, source, stats = self._sampled(
                tokens, logp, teacher_sampled_token_logprobs, student_logprobs_for_reward, old_student_logprobs,
                current_student_logprobs)
        reward, clipped, mean_teacher, mean_student = stats
        n = tokens.count().detach()
        return MOPDLossOutput(loss, loss_sum, n, n, tokens.mean(reward), tokens.mean(clipped.float()),
                              mean_teacher, mean_student, (mean_teacher - mean_student).detach(), n, self.mode,
                              source, policy_out)


# --------------------------------------------------------------------------- rewards
class KimiRewardComposer:
    """Detached, explicitly weighted sum of the verifier, generative and task-specific rewards."""

    SOURCES = ("verifier", "generative", "task_specific")

    def __call__(self, *, verifier_reward, generative_reward, task_specific_reward, weights: RewardWeights):
        given = {"verifier": verifier_reward, "generative": generative_reward, "task_specific": task_specific_reward}
        present = [name for name in self.SOURCES if given[name] is not None]
        if not present:
            raise ValueError("no reward source was given")
        shape = given[present[0]].shape
        if len(shape) != 1:
            raise ValueError("rewards must have shape [B]")
        total = torch.zeros(shape, dtype=torch.float32, device=given[present[0]].device)
        for name in self.SOURCES:
            value, weight = given[name], getattr(weights, name)
            if value is None and weight is not None:
                raise ValueError(f"weight for {name} given without its reward")
            if value is None:
                continue
            if weight is None:
                raise ValueError(f"{name} reward needs an explicit weight")
            if value.shape != shape:
                raise ValueError("reward sources must share one shape")
            if not bool(torch.isfinite(value).all()):
                raise FloatingPointError(f"{name} reward has non-finite entries")
            total = total + float(weight) * value.detach().float()
        return total


def apply_reasoning_budget_override(reward, used_tokens, base_budget, budget_multiplier, penalty_reward=-1.0):
    """A sample that used more than ``budget_multiplier`` times its base reasoning budget gets the
    penalty reward instead of its own."""
    if reward.ndim != 1 or used_tokens.shape != reward.shape or base_budget.shape != reward.shape:
        raise ValueError("reward, used_tokens and base_budget must all have shape [B]")
    if budget_multiplier <= 0:
        raise ValueError("budget_multiplier must be positive")
    if bool((used_tokens < 0).any()) or bool((base_budget < 0).any()):
        raise ValueError("token counts and budgets must be non-negative")
    over = used_tokens.float() > base_budget.float() * float(budget_multiplier)
    return reward.detach().float().masked_fill(over, float(penalty_reward))


def apply_verbosity_binary_rule(wins, output_length, initial_verbosity, sigma):
    """A win survives only when the output is at most ``sigma`` times the initial verbosity."""
    if wins.dtype != torch.bool:
        raise TypeError("wins must be a boolean tensor")
    if output_length.shape != wins.shape or initial_verbosity.shape != wins.shape:
        raise ValueError("wins, output_length and initial_verbosity must share a shape")
    if sigma <= 0:
        raise ValueError("sigma must be positive")
    return wins.detach() & (output_length.float() <= float(sigma) * initial_verbosity.float())


# --------------------------------------------------------------------------- configuration and dispatch
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
        checks = (
            (self.ignore_index < 0, "ignore_index must be negative (outside the vocabulary)"),
            (0.0 <= self.label_smoothing < 1.0, "label_smoothing must lie in [0, 1)"),
            (self.lambda_mtp >= 0, "lambda_mtp must be non-negative"),
            (self.sft_reduction in ("token_mean", "sequence_mean"), "unsupported SFT reduction"),
            (self.rl_log_ratio_l2_coef is None or self.rl_log_ratio_l2_coef >= 0,
             "rl_log_ratio_l2_coef must be non-negative"),
            (self.mopd_reward_clip_max is None or self.mopd_reward_clip_max > 0,
             "mopd_reward_clip_max must be positive"),
            ((self.rl_ratio_clip_min is None) == (self.rl_ratio_clip_max is None),
             "the two RL ratio bounds go together"),
            (self.rl_ratio_clip_min is None or 0 < self.rl_ratio_clip_min <= self.rl_ratio_clip_max,
             "RL ratio bounds need 0 < min <= max"),
            (self.mopd_mode in MultiTeacherOnPolicyDistillationLoss.MODES, "unsupported MOPD mode"),
            (self.compute_loss_in_fp32, "losses are always computed in fp32"),
        )
        for ok, message in checks:
            if not ok:
                raise ValueError(message)

    def require_posttraining_values(self) -> None:
        needed = (self.rl_ratio_clip_min, self.rl_ratio_clip_max, self.rl_log_ratio_l2_coef, self.mopd_reward_clip_max)
        if any(v is None for v in needed):
            raise ValueError("RL and MOPD values are unpublished project choices and must be set explicitly")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "KimiLossConfig":
        return cls(**values)


# inputs each phase accepts (anything else raises: it belongs to another phase)
_PHASE_INPUTS = {
    KimiTrainingPhase.PRETRAIN: frozenset({"logits", "labels", "attention_mask", "loss_mask", "boundary_mask",
                                           "token_weights", "mtp_logits", "mtp_labels", "mtp_loss_mask",
                                           "future_offsets", "moe_diagnostics"}),
    KimiTrainingPhase.SFT: frozenset({"logits", "labels", "assistant_mask", "attention_mask", "component_ids",
                                      "component_weights", "boundary_mask", "sample_weights",
                                      "return_per_component"}),
    KimiTrainingPhase.RL: frozenset({"current_logprobs", "old_logprobs", "action_mask", "rewards",
                                     "prompt_group_ids", "advantages", "sample_weights", "expected_group_size"}),
    KimiTrainingPhase.MOPD: frozenset({"current_student_logprobs", "teacher_sampled_token_logprobs", "action_mask",
                                       "teacher_ids", "student_logprobs_for_reward", "old_student_logprobs",
                                       "teacher_topk_token_ids", "teacher_topk_logprobs", "student_topk_logprobs",
                                       "sampled_token_ids", "teacher_sampled_token_ids"}),
}


class KimiTrainingObjective(nn.Module):
    """One objective per training phase; a phase receiving another phase's inputs raises."""

    def __init__(self, config: KimiLossConfig):
        super().__init__()
        self.config = config
        self.pretrain = KimiPretrainingLoss(lambda_mtp=config.lambda_mtp, ignore_index=config.ignore_index,
                                            label_smoothing=config.label_smoothing)
        self.sft = SFTTrajectoryCrossEntropyLoss(ignore_index=config.ignore_index, reduction=config.sft_reduction)
        have_rl = config.rl_ratio_clip_min is not None and config.rl_log_ratio_l2_coef is not None
        self.rl = (KimiPolicyOptimizationLoss(ratio_clip_min=config.rl_ratio_clip_min,
                                              ratio_clip_max=config.rl_ratio_clip_max,
                                              log_ratio_l2_coef=config.rl_log_ratio_l2_coef,
                                              normalize_advantages=config.rl_normalize_advantages)
                   if have_rl else None)
        self.mopd = (MultiTeacherOnPolicyDistillationLoss(reward_clip_max=config.mopd_reward_clip_max,
                                                          mode=config.mopd_mode, policy_loss=self.rl)
                     if config.mopd_reward_clip_max is not None else None)

    def forward(self, phase, **inputs) -> KimiLossBundle:
        phase = KimiTrainingPhase(phase)
        stray = sorted(set(inputs) - _PHASE_INPUTS[phase])
        if stray:
            raise ValueError(f"inputs {stray} belong to another phase than {phase.value}")
        objective = getattr(self, phase.value)
        if objective is None:
            self.config.require_posttraining_values()
        if phase is KimiTrainingPhase.SFT:
            out = objective(inputs.pop("logits"), inputs.pop("labels"), **inputs)
        else:
            out = objective(**inputs)
        return KimiLossBundle(phase, out.loss, out)


__all__ = ["SFTTrajectoryCrossEntropyLoss", "KimiPolicyOptimizationLoss", "MultiTeacherOnPolicyDistillationLoss",
           "KimiRewardComposer", "KimiLossConfig", "KimiTrainingObjective", "validate_teacher_ids",
           "clipped_teacher_student_reward", "corrected_topk_reverse_kl", "apply_reasoning_budget_override",
           "apply_verbosity_binary_rule"]
