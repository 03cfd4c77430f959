"""Next-token sampling on the device.

Parity: ``inference/sampling.py:10-91`` (reference): repetition penalty (divide positive,
multiply negative logits of seen tokens), top-k, top-p (keep the smallest prefix whose mass
reaches p, always the top token), temperature, seeded multinomial, NaN-safe argmax; an
all-invalid distribution falls back to argmax.  Both filters here cut at a per-row logit
threshold, so tokens tied with the last kept one are all kept (as in the fused device sampler);
the reference's cut among equal values depends on its sort order.

The reference's repetition penalty loops over rows in Python with ``torch.unique``; here it
is one scatter over a ``[B, V]`` seen-mask. The validity fallback is decided on the device
(``torch.where``) instead of a host branch, so a decode step issues no synchronisation.
"""
from __future__ import annotations

import torch

from .config import GenerationConfig


def apply_repetition_penalty(logits: torch.Tensor, token_ids: torch.Tensor, penalty: float | None) -> torch.Tensor:
    if penalty is None or penalty == 1:
        return logits
    if penalty <= 0:
        raise ValueError("repetition penalty must be positive")
    seen = torch.zeros_like(logits, dtype=torch.bool)
    seen.scatter_(1, token_ids.long().to(logits.device), True)
    adjusted = torch.where(logits < 0, logits * penalty, logits / penalty)
    return torch.where(seen, adjusted, logits)


def top_k_filter(logits: torch.Tensor, top_k: int | None) -> torch.Tensor:
    """Keep the logits at or above each row's k-th largest value (ties with it are kept)."""
    v = logits.shape[-1]
    if top_k is None or top_k >= v:
        return logits
    # the k-th largest is the (v - k + 1)-th smallest
    threshold = torch.kthvalue(logits, v - int(top_k) + 1, dim=-1, keepdim=True).values
    return torch.where(logits >= threshold, logits, torch.full_like(logits, float("-inf")))


def top_p_filter(logits: torch.Tensor, top_p: float | None) -> torch.Tensor:
    """Nucleus filter: a token survives when the probability mass strictly ahead of it (in
    descending order) is at most ``top_p``, so the top token always survives and the kept set is
    the shortest prefix whose mass reaches ``top_p``.  Applied as a per-row logit threshold (the
    smallest surviving logit), which also keeps ties with the last surviving token."""
    if top_p is None or top_p >= 1:
        return logits
    ordered = logits.sort(dim=-1, descending=True).values
    p = torch.softmax(ordered, dim=-1)
    mass_ahead = p.cumsum(dim=-1) - p
    survivors = (mass_ahead <= top_p).sum(dim=-1, keepdim=True).clamp_min(1)
    threshold = ordered.gather(-1, survivors - 1)
    return torch.where(logits >= threshold, logits, torch.full_like(logits, float("-inf")))


def safe_argmax(logits: torch.Tensor) -> torch.Tensor:
    return torch.nan_to_num(logits, nan=float("-inf"), posinf=1e30, neginf=-1e30).argmax(dim=-1, keepdim=True)


def sample_next_token(logits: torch.Tensor, config: GenerationConfig, *, previous_token_ids=None,
                      generator: torch.Generator | None = None) -> torch.Tensor:
    """``[B, V]`` logits -> ``[B, 1]`` token ids."""
    if logits.ndim != 2:
        raise ValueError("sampling logits must have shape [B,V]")
    if previous_token_ids is not None:
        logits = apply_repetition_penalty(logits, previous_token_ids, config.repetition_penalty)
    greedy = safe_argmax(logits)
    if not config.do_sample:
        return greedy
    filt = top_p_filter(top_k_filter(logits.float() / config.temperature, config.top_k), config.top_p)
    probs = torch.softmax(filt, dim=-1)
    ok = torch.isfinite(probs).all(-1) & probs.sum(-1).gt(0) & torch.isfinite(logits).all(-1)
    safe_probs = torch.where(ok[:, None], torch.nan_to_num(probs, nan=0.0), torch.ones_like(probs))
    drawn = torch.multinomial(safe_probs, num_samples=1, generator=generator)
    return torch.where(ok[:, None], drawn, safe_argmax(filt))


__all__ = ["apply_repetition_penalty", "top_k_filter", "top_p_filter", "safe_argmax", "sample_next_token"]
