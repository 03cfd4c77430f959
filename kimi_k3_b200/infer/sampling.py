"""Next-token sampling on the device.

Parity: ``inference/sampling.py:10-91`` (reference): repetition penalty (divide positive,
multiply negative logits of seen tokens), top-k, top-p (keep the smallest prefix whose mass
reaches p, always the top token), temperature, seeded multinomial, NaN-safe argmax; an
all-invalid distribution falls back to argmax.

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
    if top_k is None or top_k >= logits.shape[-1]:
        return logits
    cutoff = torch.topk(logits, int(top_k), dim=-1).values[..., -1, None]
    return logits.masked_fill(logits < cutoff, float("-inf"))


def top_p_filter(logits: torch.Tensor, top_p: float | None) -> torch.Tensor:
    if top_p is None or top_p >= 1:
        return logits
    srt, idx = torch.sort(logits, descending=True, dim=-1)
    cum = torch.softmax(srt, dim=-1).cumsum(dim=-1)
    drop = cum > top_p
    drop[..., 1:] = drop[..., :-1].clone()
    drop[..., 0] = False
    return torch.empty_like(logits).scatter(-1, idx, srt.masked_fill(drop, float("-inf")))


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
