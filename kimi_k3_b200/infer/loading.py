"""Build a model from its YAML and restore checkpoint weights for inference.

Parity: ``inference/loading.py:38-133`` (reference): weights from ``model_state_dict`` /
``state_dict`` / ``model`` (or a bare state dict), tied weights re-tied, precision and device
applied, gradients disabled, eval mode. A distributed checkpoint directory is accepted when
it was exported with the full un-sharded state.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch

from ..config.model_yaml import build_model_from_yaml
from .config import ModelLoadConfig


class TokenizerModelMetadata:
    """Exposes ``vocab_size`` / ``token_id`` of a tokenizer to the model YAML builder."""

    def __init__(self, tokenizer):
        self.tokenizer = tokenizer

    @property
    def vocab_size(self) -> int:
        v = getattr(self.tokenizer, "vocab_size", None)
        if v is None and hasattr(self.tokenizer, "get_vocab_size"):
            v = self.tokenizer.get_vocab_size()
        if v is None:
            raise ValueError("tokenizer does not expose a vocabulary size")
        return int(v)

    def token_id(self, token: str):
        from .tokenization import tokenizer_token_id
        return tokenizer_token_id(self.tokenizer, token)


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


def resolve_load_device(requested: str) -> torch.device:
    if requested == "auto":
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    dev = torch.device(requested)
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("CUDA model loading requested but unavailable")
    return dev


def state_dict_from_payload(payload) -> dict:
    if not isinstance(payload, dict):
        raise ValueError("checkpoint must contain a mapping")
    for key in ("model_state_dict", "state_dict", "model"):
        st = payload.get(key)
        if isinstance(st, dict) and st:
            return st
    if payload and all(torch.is_tensor(v) for v in payload.values()):
        return payload
    raise ValueError("checkpoint does not contain model weights")


def load_kimi_checkpoint(model_config_path, checkpoint_path, *, tokenizer=None,
                         load_config: ModelLoadConfig | None = None) -> LoadedKimiCheckpoint:
    cfg = load_config or ModelLoadConfig()
    ckpt = Path(checkpoint_path).expanduser().resolve()
    if not ckpt.is_file():
        raise FileNotFoundError(f"checkpoint not found: {ckpt}")
    meta = None if tokenizer is None else TokenizerModelMetadata(tokenizer)
    model = build_model_from_yaml(model_config_path, data_bundle=meta)
    payload = torch.load(ckpt, map_location="cpu", weights_only=False)
    inc = model.load_state_dict(state_dict_from_payload(payload), strict=cfg.strict)
    if hasattr(model, "tie_weights"):
        model.tie_weights()
    dev = resolve_load_device(cfg.device)
    dtype = {"fp32": torch.float32, "bf16": torch.bfloat16, "fp16": torch.float16}.get(cfg.precision)
    if dtype is torch.float16 and dev.type == "cpu":
        raise RuntimeError("FP16 inference is unsupported on CPU")
    model.to(device=dev) if dtype is None else model.to(device=dev, dtype=dtype)
    model.requires_grad_(False)
    model.eval()
    m = payload if isinstance(payload, dict) else {}
    return LoadedKimiCheckpoint(model, ckpt, int(m.get("format_version", 0)), int(m.get("global_step", 0)),
                                int(m.get("epoch", 0)), dict(m.get("metadata") or {}), tuple(inc.missing_keys),
                                tuple(inc.unexpected_keys))


__all__ = ["LoadedKimiCheckpoint", "TokenizerModelMetadata", "resolve_load_device", "state_dict_from_payload",
           "load_kimi_checkpoint"]
