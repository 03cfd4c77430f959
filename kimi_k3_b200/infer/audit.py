"""Full-forward vs prefill + per-token decode audit (reference: ``inference/audit.py:13-62``)."""
from __future__ import annotations

import torch

from .cache import cache_summary
from .generation import decode_one_token, prefill_prompt


@torch.no_grad()
def compare_full_vs_cached_logits(model, input_ids, *, split: int | None = None, atol: float = 1e-5,
                                  rtol: float = 1e-5) -> dict:
    if input_ids.ndim != 2 or input_ids.shape[1] < 2:
        raise ValueError("audit requires input_ids [B,T] with T >= 2")
    split = int(split or max(1, input_ids.shape[1] // 2))
    if not 1 <= split < input_ids.shape[1]:
        raise ValueError("split must lie inside the sequence")
    dev = next(model.parameters()).device
    ids = input_ids.to(dev)
    mask = torch.ones_like(ids, dtype=torch.bool)
    was = model.training
    model.eval()
    try:
        full = model(input_ids=ids, attention_mask=mask, return_dict=True).logits
        pre = prefill_prompt(model, ids[:, :split], mask[:, :split])
        pieces, cache = [pre.logits], pre.cache
        for i in range(split, ids.shape[1]):
            d = decode_one_token(model, ids[:, i:i + 1], cache, mask[:, i:i + 1])
            pieces.append(d.logits)
            cache = d.cache
        inc = torch.cat(pieces, 1)
        return {"allclose": bool(torch.allclose(inc.float(), full.float(), atol=atol, rtol=rtol)),
                "max_abs_diff": float((inc.float() - full.float()).abs().max()), "atol": float(atol),
                "rtol": float(rtol), "cache_stats": cache_summary(cache)}
    finally:
        if was:
            model.train()


__all__ = ["compare_full_vs_cached_logits"]
