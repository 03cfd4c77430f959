"""Inference session: checkpoint restore, prompt codec, cache accounting and the cache audit.

One object owns what a serving caller needs around the generation loops:

* :class:`TextCodec` resolves a tokenizer's special ids once, at construction, from the
  attribute spellings tokenizers use (``bos_token_id`` / ``bos_id`` / ``token_to_id("<bos>")``),
  and encodes / decodes prompts with them.
* :class:`InferenceSession` builds the model from its YAML, restores weights from a
  checkpoint payload, places it, and offers :meth:`InferenceSession.audit` (full forward vs
  prefill + per-token decode, compared as the pieces stream in, without concatenating them) and
  :meth:`InferenceSession.cache_report`.
* Cache accounting walks the cache object graph iteratively and counts every distinct span of
  device memory once (identity by address and size, so two views of one buffer count once).

The module-level functions keep the reference's public names and return shapes (an interface kept
alike on purpose: callers of ``inference/loading.py``, ``inference/audit.py``, ``inference/cache.py``
and ``inference/tokenization.py`` of the reference switch without edits).
"""
from __future__ import annotations

from dataclasses import dataclass, fields, is_dataclass
from pathlib import Path
from typing import Any, Iterator

import torch

from .config import ModelLoadConfig

# --------------------------------------------------------------------------- prompt codec
_SPECIAL_NAMES = {"<bos>": "bos", "<eos>": "eos", "<pad>": "pad", "<unk>": "unk"}


def _lookup_special(tokenizer: Any, kind: str) -> int | None:
    for attr in (f"{kind}_token_id", f"{kind}_id"):
        value = getattr(tokenizer, attr, None)
        if value is not None and not callable(value):
            return int(value)
    to_id = getattr(tokenizer, "token_to_id", None)
    if callable(to_id):
        value = to_id(f"<{kind}>")
        return None if value is None else int(value)
    return None


class TextCodec:
    """Prompt encoding and id decoding against one tokenizer (or none: id lists and tensors only)."""

    def __init__(self, tokenizer: Any = None):
        self.tokenizer = tokenizer
        self.special = ({} if tokenizer is None else
                        {kind: _lookup_special(tokenizer, kind) for kind in ("bos", "eos", "pad", "unk")})

    def special_id(self, token: str) -> int | None:
        kind = _SPECIAL_NAMES.get(token)
        if kind is not None:
            return self.special.get(kind)
        to_id = getattr(self.tokenizer, "token_to_id", None)
        if callable(to_id):
            value = to_id(token)
            return None if value is None else int(value)
        return None

    def _tokenize(self, text: str) -> list[int]:
        tok = self.tokenizer
        if hasattr(tok, "encode"):
            enc = tok.encode(text)
            return list(getattr(enc, "ids", enc))
        return torch.as_tensor(tok(text, return_tensors="pt")["input_ids"]).reshape(-1).tolist()

    def encode(self, prompt, *, add_bos: bool = True) -> torch.Tensor:
        """A prompt (text, list of ids, ``[T]`` or ``[B, T]`` tensor) as int64 ``[B, T]`` ids."""
        if torch.is_tensor(prompt):
            ids = prompt.detach().long().clone()
            if ids.ndim == 1:
                ids = ids[None]
            if ids.ndim != 2 or ids.shape[1] == 0:
                raise ValueError("prompt tensor must have shape [T] or [B,T] with T > 0")
            return ids
        if isinstance(prompt, list):
            if not prompt or any(not isinstance(v, int) for v in prompt):
                raise ValueError("prompt ID list must contain integers")
            return torch.tensor([prompt], dtype=torch.long)
        if not isinstance(prompt, str) or not prompt.strip():
            raise ValueError("text prompt must be a non-empty string")
        if self.tokenizer is None:
            raise ValueError("a tokenizer is required for text prompts")
        body = self._tokenize(prompt)
        bos = self.special.get("bos")
        if add_bos and bos is not None and (not body or body[0] != bos):
            body = [bos] + body
        if not body:
            raise ValueError("tokenizer produced an empty prompt")
        return torch.tensor([body], dtype=torch.long)

    def decode(self, ids, *, skip_special: bool = True):
        """``[T]`` ids, or a batch of one row, -> one string; ``[B, T]`` -> a list of strings.  The
        tokenizer's own ``decode`` applies ``skip_special``; without a tokenizer the ids are joined."""
        t = ids.detach().cpu().long() if torch.is_tensor(ids) else torch.as_tensor(ids, dtype=torch.long)
        if t.ndim not in (1, 2):
            raise ValueError("token IDs must have shape [T] or [B,T]")
        rows = t.reshape(-1, t.shape[-1]).tolist()
        texts = [self._render(row, skip_special) for row in rows]
        return texts[0] if len(texts) == 1 else texts

    def _render(self, row: list[int], skip_special: bool) -> str:
        dec = getattr(self.tokenizer, "decode", None)
        if dec is None:
            return " ".join(str(i) for i in row)
        try:
            return dec(row, skip_special_tokens=skip_special)
        except TypeError:
            return dec(row)


def tokenizer_token_id(tokenizer: Any, token: str) -> int | None:
    return TextCodec(tokenizer).special_id(token)


def encode_prompt(prompt, *, tokenizer=None, add_bos_token: bool = True) -> torch.Tensor:
    return TextCodec(tokenizer).encode(prompt, add_bos=add_bos_token)


def decode_token_ids(ids, *, tokenizer=None, skip_special_tokens: bool = True):
    return TextCodec(tokenizer).decode(ids, skip_special=skip_special_tokens)


class TokenizerModelMetadata:
    """Vocabulary size and special ids of a tokenizer, in the form the model YAML builder asks for."""

    def __init__(self, tokenizer):
        self.codec = TextCodec(tokenizer)

    @property
    def vocab_size(self) -> int:
        tok = self.codec.tokenizer
        size = getattr(tok, "vocab_size", None)
        if size is None and callable(getattr(tok, "get_vocab_size", None)):
            size = tok.get_vocab_size()
        if size is None:
            raise ValueError("tokenizer does not expose a vocabulary size")
        return int(size)

    def token_id(self, token: str):
        return self.codec.special_id(token)


# --------------------------------------------------------------------------- cache accounting
def _device_spans(root) -> Iterator[torch.Tensor]:
    """Every tensor reachable from ``root`` once per (address, bytes) span; iterative walk."""
    stack, seen_obj, seen_span = [root], set(), set()
    while stack:
        node = stack.pop()
        if node is None or isinstance(node, (int, float, str, bool)):
            continue
        if torch.is_tensor(node):
            span = (node.device, node.data_ptr(), node.numel() * node.element_size())
            if span not in seen_span:
                seen_span.add(span)
                yield node
            continue
        if id(node) in seen_obj:
            continue
        seen_obj.add(id(node))
        if isinstance(node, dict):
            stack.extend(node.values())
        elif isinstance(node, (list, tuple)):
            stack.extend(node)
        elif is_dataclass(node):
            stack.extend(getattr(node, f.name) for f in fields(node))


def cache_memory_bytes(cache) -> int:
    return sum(t.numel() * t.element_size() for t in _device_spans(cache))


@dataclass
class CacheReport:
    sequence_length: int
    sequence_lengths: list
    num_layers: int
    num_kda_layers: int
    num_mla_layers: int
    kda_elements: int
    mla_elements: int
    total_elements: int
    memory_bytes: int

    @classmethod
    def of(cls, cache) -> "CacheReport":
        from ..models.backbone import HybridBackboneCache
        if not isinstance(cache, HybridBackboneCache):
            raise TypeError("expected Kimi HybridBackboneCache")
        counts = {"kda": 0, "gated_mla": 0}
        for layer in cache.layer_caches:
            counts[layer.attention_type] = counts.get(layer.attention_type, 0) + 1
        return cls(int(cache.sequence_length), cache.sequence_lengths.detach().cpu().tolist(),
                   len(cache.layer_caches), counts["kda"], counts["gated_mla"], int(cache.kda_elements),
                   int(cache.mla_elements), int(cache.total_elements), cache_memory_bytes(cache))

    def as_dict(self) -> dict:
        return {f.name: getattr(self, f.name) for f in fields(self)}


def cache_summary(cache) -> dict:
    return {} if cache is None else CacheReport.of(cache).as_dict()


def validate_kimi_cache(model, cache) -> None:
    """The cache's per-layer kinds follow the backbone's attention layout (the final global layer
    stores an ordinary gated-MLA latent cache)."""
    from ..models.backbone import HybridBackboneCache
    if not isinstance(cache, HybridBackboneCache):
        raise TypeError("model did not return HybridBackboneCache")
    backbone = (model.module if hasattr(model, "module") else model).backbone
    want = [kind[: -len("_final")] if kind.endswith("_final") else kind for kind in backbone.attention_types]
    if [layer.attention_type for layer in cache.layer_caches] != want:
        raise ValueError("cache attention layout does not match Kimi backbone")
    if cache.sequence_lengths.numel() == 0:
        raise ValueError("cache must contain at least one sequence")


# --------------------------------------------------------------------------- checkpoints and sessions
_WEIGHT_KEYS = ("model_state_dict", "state_dict", "model")
_PRECISIONS = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}


def state_dict_from_payload(payload) -> dict:
    """The model weights inside a checkpoint payload (one of the usual keys, or a bare state dict)."""
    if not isinstance(payload, dict):
        raise ValueError("checkpoint must contain a mapping")
    found = next((payload[k] for k in _WEIGHT_KEYS if isinstance(payload.get(k), dict) and payload[k]), None)
    if found is not None:
        return found
    if payload and all(torch.is_tensor(v) for v in payload.values()):
        return payload
    raise ValueError("checkpoint does not contain model weights")


def resolve_load_device(requested: str) -> torch.device:
    if requested == "auto":
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    device = torch.device(requested)
    if device.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("CUDA model loading requested but unavailable")
    return device


@dataclass
class LoadedKimiCheckpoint:
    model: Any
    checkpoint_path: Path
    format_version: int
    global_step: int
    epoch: int
    metadata: dict
    missing_keys: tuple
    unexpected_keys: tuple


class InferenceSession:
    """A model placed for inference, its prompt codec, and the tools around generation."""

    def __init__(self, model, *, tokenizer=None, checkpoint: LoadedKimiCheckpoint | None = None):
        self.model = model
        self.codec = TextCodec(tokenizer)
        self.checkpoint = checkpoint

    @property
    def device(self) -> torch.device:
        p = next(iter(self.model.parameters()), None)
        return p.device if p is not None else torch.device("cpu")

    @classmethod
    def from_files(cls, model_config_path, checkpoint_path, *, tokenizer=None,
                   load_config: ModelLoadConfig | None = None) -> "InferenceSession":
        from ..config.model_yaml import build_model_from_yaml
        cfg = load_config or ModelLoadConfig()
        path = Path(checkpoint_path).expanduser().resolve()
        if not path.is_file():
            raise FileNotFoundError(f"checkpoint not found: {path}")
        device = resolve_load_device(cfg.device)
        dtype = _PRECISIONS.get(cfg.precision)
        if dtype is torch.float16 and device.type == "cpu":
            raise RuntimeError("FP16 inference is unsupported on CPU")
        model = build_model_from_yaml(model_config_path,
                                      data_bundle=None if tokenizer is None else TokenizerModelMetadata(tokenizer))
        payload = torch.load(path, map_location="cpu", weights_only=False)
        result = model.load_state_dict(state_dict_from_payload(payload), strict=cfg.strict)
        if callable(getattr(model, "tie_weights", None)):
            model.tie_weights()
        model.to(device=device, dtype=dtype) if dtype is not None else model.to(device=device)
        model.requires_grad_(False).eval()
        info = payload if isinstance(payload, dict) else {}
        record = LoadedKimiCheckpoint(model, path, int(info.get("format_version", 0)),
                                      int(info.get("global_step", 0)), int(info.get("epoch", 0)),
                                      dict(info.get("metadata") or {}), tuple(result.missing_keys),
                                      tuple(result.unexpected_keys))
        return cls(model, tokenizer=tokenizer, checkpoint=record)

    def cache_report(self, cache) -> dict:
        return cache_summary(cache)

    @torch.no_grad()
    def audit(self, input_ids, *, split: int | None = None, atol: float = 1e-5, rtol: float = 1e-5) -> dict:
        """Logits of one full forward against prefill (first ``split`` tokens) + one cached decode
        step per remaining token.  Pieces are compared as they are produced."""
        from .generation import decode_one_token, prefill_prompt
        if input_ids.ndim != 2 or input_ids.shape[1] < 2:
            raise ValueError("audit requires input_ids [B,T] with T >= 2")
        total = input_ids.shape[1]
        split = int(split or max(1, total // 2))
        if not 1 <= split < total:
            raise ValueError("split must lie inside the sequence")
        model, ids = self.model, input_ids.to(self.device)
        mask = torch.ones_like(ids, dtype=torch.bool)
        restore = model.training
        model.eval()
        try:
            reference = model(input_ids=ids, attention_mask=mask, return_dict=True).logits.float()
            worst, close = 0.0, True
            step = prefill_prompt(model, ids[:, :split], mask[:, :split])
            start = 0
            while True:
                piece = step.logits.float()
                want = reference[:, start:start + piece.shape[1]]
                worst = max(worst, float((piece - want).abs().max()))
                close = close and bool(torch.allclose(piece, want, atol=atol, rtol=rtol))
                start += piece.shape[1]
                if start >= total:
                    break
                step = decode_one_token(model, ids[:, start:start + 1], step.cache, mask[:, start:start + 1])
            return {"allclose": close, "max_abs_diff": worst, "atol": float(atol), "rtol": float(rtol),
                    "cache_stats": cache_summary(step.cache)}
        finally:
            if restore:
                model.train()


def load_kimi_checkpoint(model_config_path, checkpoint_path, *, tokenizer=None,
                         load_config: ModelLoadConfig | None = None) -> LoadedKimiCheckpoint:
    return InferenceSession.from_files(model_config_path, checkpoint_path, tokenizer=tokenizer,
                                       load_config=load_config).checkpoint


def compare_full_vs_cached_logits(model, input_ids, *, split: int | None = None, atol: float = 1e-5,
                                  rtol: float = 1e-5) -> dict:
    return InferenceSession(model).audit(input_ids, split=split, atol=atol, rtol=rtol)


__all__ = ["TextCodec", "InferenceSession", "CacheReport", "LoadedKimiCheckpoint", "TokenizerModelMetadata",
           "tokenizer_token_id", "encode_prompt", "decode_token_ids", "cache_memory_bytes", "cache_summary",
           "validate_kimi_cache", "state_dict_from_payload", "resolve_load_device", "load_kimi_checkpoint",
           "compare_full_vs_cached_logits"]
