"""Cache accounting and validation (reference: ``inference/cache.py:13-80``)."""
from __future__ import annotations

from dataclasses import fields, is_dataclass
from typing import Any

import torch

from ..models.backbone import HybridBackboneCache


def _tensors(value: Any, seen: set):
    if torch.is_tensor(value):
        if id(value) not in seen:
            seen.add(id(value))
            yield value
        return
    if is_dataclass(value):
        for f in fields(value):
            yield from _tensors(getattr(value, f.name), seen)
    elif isinstance(value, dict):
        for v in value.values():
            yield from _tensors(v, seen)
    elif isinstance(value, (list, tuple)):
        for v in value:
            yield from _tensors(v, seen)


def cache_memory_bytes(cache) -> int:
    return 0 if cache is None else sum(t.numel() * t.element_size() for t in _tensors(cache, set()))


def cache_summary(cache) -> dict:
    if cache is None:
        return {}
    if not isinstance(cache, HybridBackboneCache):
        raise TypeError("expected Kimi HybridBackboneCache")
    kinds = [c.attention_type for c in cache.layer_caches]
    return {"sequence_length": int(cache.sequence_length),
            "sequence_lengths": cache.sequence_lengths.detach().cpu().tolist(), "num_layers": len(kinds),
            "num_kda_layers": kinds.count("kda"), "num_mla_layers": kinds.count("gated_mla"),
            "kda_elements": int(cache.kda_elements), "mla_elements": int(cache.mla_elements),
            "total_elements": int(cache.total_elements), "memory_bytes": cache_memory_bytes(cache)}


def validate_kimi_cache(model, cache) -> None:
    if not isinstance(cache, HybridBackboneCache):
        raise TypeError("model did not return HybridBackboneCache")
    raw = model.module if hasattr(model, "module") else model
    expected = tuple("gated_mla" if n == "gated_mla_final" else n for n in raw.backbone.attention_types)
    if tuple(c.attention_type for c in cache.layer_caches) != expected:
        raise ValueError("cache attention layout does not match Kimi backbone")
    if cache.sequence_lengths.numel() == 0:
        raise ValueError("cache must contain at least one sequence")


__all__ = ["cache_memory_bytes", "cache_summary", "validate_kimi_cache"]
