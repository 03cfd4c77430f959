"""Prefill + cached decode generation.

Parity: ``inference/generation.py:54-266``, ``prefill.py``, ``decode.py``, ``outputs.py``
(reference): one prefill over the prompt, then one cached decode step per token (KDA recurrent
state + MLA latent cache), sampling per step, EOS bookkeeping (finished rows emit the pad id),
TTFT as ``prefill_seconds`` and ``tokens_per_second = generated_per_sequence / decode_seconds``.

Differences: sampling runs fully on the device (no per-step host branch) and the EOS test is
read on the host every ``eos_check_every`` steps (default 1 = reference behaviour); prompts of
different lengths are allowed (right padding; the KDA state and MLA latent cache are
per-row), while the reference requires equal prompt lengths; ``batch_tokens_per_second``
reports the batch throughput beside the reference's per-sequence rate.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, replace
from typing import Any

import torch

from .config import GenerationConfig
from .sampling import sample_next_token
from .session import cache_summary, decode_token_ids, encode_prompt, tokenizer_token_id


@dataclass
class GenerationOutput:
    prompt_ids: torch.Tensor
    sequences: torch.Tensor
    generated_ids: torch.Tensor
    text: Any
    completion_text: Any
    finish_reason: str
    cache: Any
    cache_stats: dict
    scores: tuple | None
    prompt_tokens: int
    generated_tokens: int
    prefill_seconds: float
    decode_seconds: float
    total_seconds: float
    tokens_per_second: float
    batch_tokens_per_second: float = 0.0

    def to_dict(self) -> dict:
        return {name: getattr(self, name) for name in self.__dataclass_fields__}


def _model_device(model) -> torch.device:
    p = next(iter(model.parameters()), None)
    return p.device if p is not None else torch.device("cpu")


def resolve_generation_device(model, requested: str) -> torch.device:
    if requested == "auto":
        return _model_device(model)
    dev = torch.device(requested)
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("CUDA generation requested but unavailable")
    return dev


def _sync(device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


@torch.no_grad()
def prefill_prompt(model, input_ids, attention_mask=None, **kwargs):
    return model(input_ids=input_ids, attention_mask=attention_mask, use_cache=True, return_dict=True, **kwargs)


@torch.no_grad()
def decode_one_token(model, input_ids, cache, attention_mask=None, **kwargs):
    return model(input_ids=input_ids, attention_mask=attention_mask, cache=cache, use_cache=True, return_dict=True,
                 **kwargs)


def last_prompt_logits(logits: torch.Tensor, attention_mask: torch.Tensor) -> torch.Tensor:
    idx = attention_mask.long().sum(dim=1).clamp_min(1) - 1
    return logits[torch.arange(logits.shape[0], device=logits.device), idx]


@torch.no_grad()
def generate_tokens(model, input_ids, *, generation_config: GenerationConfig | None = None, attention_mask=None,
                    prefill_kwargs: dict | None = None) -> GenerationOutput:
    cfg = generation_config or GenerationConfig()
    device = resolve_generation_device(model, cfg.device)
    if _model_device(model) != device:
        model.to(device)
    input_ids = input_ids.to(device=device, dtype=torch.long)
    if input_ids.ndim != 2 or input_ids.shape[1] == 0:
        raise ValueError("input_ids must have shape [B,T], T > 0")
    if attention_mask is None:
        attention_mask = (torch.ones_like(input_ids, dtype=torch.bool) if cfg.pad_token_id is None
                          else input_ids.ne(cfg.pad_token_id))
    attention_mask = attention_mask.to(device)
    if attention_mask.dtype != torch.bool:
        raise TypeError("attention_mask must be boolean")
    width = int(input_ids.shape[1])
    steps, reason = cfg.max_new_tokens, "length"
    if cfg.max_total_tokens is not None and max(cfg.max_total_tokens - width, 0) < steps:
        steps, reason = max(cfg.max_total_tokens - width, 0), "max_total_tokens"
    was_training = model.training
    model.eval()
    gen = torch.Generator(device=device).manual_seed(cfg.seed) if cfg.seed is not None else None
    seqs, out_tokens, scores = input_ids, [], []
    finished = torch.zeros(input_ids.shape[0], dtype=torch.bool, device=device)
    eos = cfg.eos_token_id
    pad = cfg.pad_token_id if cfg.pad_token_id is not None else eos
    _sync(device)
    t_all = time.perf_counter()
    try:
        out = prefill_prompt(model, input_ids, attention_mask, **(prefill_kwargs or {}))
        _sync(device)
        prefill_s = time.perf_counter() - t_all
        cache = out.cache
        logits = last_prompt_logits(out.logits, attention_mask)
        t_dec = time.perf_counter()
        for step in range(steps):
            if cfg.return_scores:
                scores.append(logits.detach().float().cpu())
            nxt = sample_next_token(logits, cfg, previous_token_ids=seqs, generator=gen)
            active = ~finished
            if pad is not None:
                nxt = torch.where(active[:, None], nxt, torch.full_like(nxt, int(pad)))
            out_tokens.append(nxt)
            seqs = torch.cat((seqs, nxt), dim=1)
            if eos is not None:
                finished |= active & nxt[:, 0].eq(int(eos))
            # Every row decodes its token: a finished row feeds the pad id and its outputs are
            # ignored.  (Masking finished rows out would hand the model a row with no valid token,
            # which it rejects; the reference's loop raises there once one row ends before the rest.)
            dec = decode_one_token(model, nxt, cache, torch.ones_like(active)[:, None])
            cache = dec.cache
            logits = dec.logits[:, -1, :]
            if eos is not None and (step + 1) % cfg.eos_check_every == 0 and bool(finished.all()):
                reason = "eos"
                break
        _sync(device)
        decode_s = time.perf_counter() - t_dec
    finally:
        if was_training:
            model.train()
    total_s = time.perf_counter() - t_all
    gen_ids = torch.cat(out_tokens, 1) if out_tokens else input_ids.new_empty((input_ids.shape[0], 0))
    n = int(gen_ids.shape[1])
    return GenerationOutput(input_ids, seqs, gen_ids, None, None, reason, cache if cfg.return_cache else None,
                            cache_summary(cache), tuple(scores) if cfg.return_scores else None, width, n, prefill_s,
                            decode_s, total_s, n / decode_s if decode_s > 0 else 0.0,
                            n * input_ids.shape[0] / decode_s if decode_s > 0 else 0.0)


@torch.inference_mode()
def inference_autoregressive(model, prompt, *, tokenizer=None, generation_config: GenerationConfig | None = None,
                             attention_mask=None, prefill_kwargs: dict | None = None,
                             **overrides) -> GenerationOutput:
    """Master API: encode a prompt, generate with the cache, decode the text."""
    if generation_config is not None and overrides:
        raise ValueError("pass generation_config or keyword overrides, not both")
    cfg = generation_config or GenerationConfig(**overrides)
    mc = getattr(model, "config", None)
    if cfg.eos_token_id is None:
        e = tokenizer_token_id(tokenizer, "<eos>") if tokenizer is not None else getattr(mc, "eos_token_id", None)
        if e is not None:
            cfg = replace(cfg, eos_token_id=int(e))
    if cfg.pad_token_id is None:
        p = tokenizer_token_id(tokenizer, "<pad>") if tokenizer is not None else getattr(mc, "pad_token_id", None)
        if p is not None:
            cfg = replace(cfg, pad_token_id=int(p))
    ids = encode_prompt(prompt, tokenizer=tokenizer, add_bos_token=cfg.add_bos_token)
    out = generate_tokens(model, ids, generation_config=cfg, attention_mask=attention_mask,
                          prefill_kwargs=prefill_kwargs)
    if tokenizer is not None:
        out.text = decode_token_ids(out.sequences, tokenizer=tokenizer, skip_special_tokens=cfg.skip_special_tokens)
        out.completion_text = decode_token_ids(out.generated_ids, tokenizer=tokenizer,
                                               skip_special_tokens=cfg.skip_special_tokens)
    return out


__all__ = ["GenerationOutput", "prefill_prompt", "decode_one_token", "generate_tokens", "inference_autoregressive",
           "resolve_generation_device", "last_prompt_logits"]
