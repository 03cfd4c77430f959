"""Prompt encoding / decoding helpers (reference: ``inference/tokenization.py:10-117``)."""
from __future__ import annotations

from typing import Any

import torch

_SPECIAL = ("<pad>", "<bos>", "<eos>", "<unk>")


def tokenizer_token_id(tokenizer: Any, token: str) -> int | None:
    attr = {"<bos>": "bos_token_id", "<eos>": "eos_token_id", "<pad>": "pad_token_id"}.get(token)
    if attr is not None and getattr(tokenizer, attr, None) is not None:
        return int(getattr(tokenizer, attr))
    legacy = {"<bos>": "bos_id", "<eos>": "eos_id", "<pad>": "pad_id"}.get(token)
    if legacy is not None and getattr(tokenizer, legacy, None) is not None:
        return int(getattr(tokenizer, legacy))
    if hasattr(tokenizer, "token_to_id"):
        v = tokenizer.token_to_id(token)
        return None if v is None else int(v)
    return None


def encode_prompt(prompt, *, tokenizer=None, add_bos_token: bool = True) -> torch.Tensor:
    """One prompt -> ``[1, T]`` ids (a ``[B, T]`` tensor passes through)."""
    if torch.is_tensor(prompt):
        ids = prompt.detach().clone().long()
        ids = ids.unsqueeze(0) if ids.ndim == 1 else ids
        if ids.ndim != 2 or ids.shape[1] == 0:
            raise ValueError("prompt tensor must have shape [T] or [B,T] with T > 0")
        return ids
    if isinstance(prompt, list):
        if not prompt or not all(isinstance(v, int) for v in prompt):
            raise ValueError("prompt ID list must contain integers")
        return torch.tensor(prompt, dtype=torch.long).unsqueeze(0)
    if not isinstance(prompt, str) or not prompt.strip():
        raise ValueError("text prompt must be a non-empty string")
    if tokenizer is None:
        raise ValueError("a tokenizer is required for text prompts")
    if callable(tokenizer) and not hasattr(tokenizer, "encode"):
        ids = tokenizer(prompt, return_tensors="pt")["input_ids"]
    else:
        enc = tokenizer.encode(prompt)
        ids = torch.as_tensor(enc.ids if hasattr(enc, "ids") else enc, dtype=torch.long).unsqueeze(0)
    if ids.ndim != 2:
        raise ValueError("tokenizer must produce token IDs with shape [1,T]")
    bos = tokenizer_token_id(tokenizer, "<bos>")
    if add_bos_token and bos is not None and (ids.shape[1] == 0 or int(ids[0, 0]) != bos):
        ids = torch.cat((torch.tensor([[bos]], dtype=torch.long), ids), dim=1)
    return ids


def decode_token_ids(ids, *, tokenizer=None, skip_special_tokens: bool = True):
    """``[T]`` or ``[B, T]`` ids -> text (list for batches)."""
    t = ids.detach().cpu() if torch.is_tensor(ids) else torch.as_tensor(ids)
    rows = t.tolist() if t.ndim == 2 else [t.tolist()]
    special = {tokenizer_token_id(tokenizer, s) for s in _SPECIAL} if tokenizer is not None else set()
    out = []
    for row in rows:
        if skip_special_tokens:
            row = [i for i in row if i not in special]
        if tokenizer is None:
            out.append(" ".join(map(str, row)))
        elif hasattr(tokenizer, "decode"):
            try:
                out.append(tokenizer.decode(row, skip_special_tokens=skip_special_tokens))
            except TypeError:
                out.append(tokenizer.decode(row))
        else:
            out.append(" ".join(map(str, row)))
    return out if t.ndim == 2 else out[0]


__all__ = ["tokenizer_token_id", "encode_prompt", "decode_token_ids"]
