"""Batch summaries for data validation (reference: ``data/inspection.py:12-97``)."""
from __future__ import annotations

import torch


def summarize_tensor(t: torch.Tensor) -> dict:
    out = {"shape": tuple(t.shape), "dtype": str(t.dtype), "device": str(t.device), "numel": int(t.numel())}
    if t.numel() and (t.is_floating_point() or t.dtype in (torch.int32, torch.int64, torch.int16, torch.uint8)):
        f = t.detach().float()
        out.update({"min": float(f.min()), "max": float(f.max()), "mean": float(f.mean())})
    if t.dtype == torch.bool:
        out["true_fraction"] = float(t.float().mean()) if t.numel() else 0.0
    return out


def summarize_lm_batch(batch) -> dict:
    from ..train.loop import normalize_lm_batch
    b = normalize_lm_batch(batch)
    out = {k: summarize_tensor(v) for k, v in b.items() if torch.is_tensor(v)}
    ids, labels = b["input_ids"], b.get("labels")
    mask = b.get("attention_mask")
    out["batch_size"] = int(ids.shape[0])
    out["sequence_length"] = int(ids.shape[1]) if ids.ndim > 1 else 1
    out["valid_tokens"] = int(mask.sum()) if mask is not None else int(ids.numel())
    if torch.is_tensor(labels):
        out["ignored_labels"] = int((labels == -100).sum())
        out["labels_shifted"] = bool(ids.ndim == 2 and ids.shape[1] > 1 and torch.equal(ids[:, 1:], labels[:, :-1]))
    return out


__all__ = ["summarize_tensor", "summarize_lm_batch"]
