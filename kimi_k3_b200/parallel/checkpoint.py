"""Distributed checkpoints: one file per rank, committed atomically as a directory.

Parity: ``training/distributed/checkpoint.py:109-303`` (reference): a temporary directory
receives ``rank_%05d.pt`` from every rank, rank 0 adds ``metadata.json`` (topology and
sha256 fingerprints of the model / data / training configs and the optimizer parameter
registry) and a ``SUCCESS`` marker, then renames the directory into place; loading requires
the marker and the same topology. The on-disk layout is kept identical.

Addition: :func:`export_rank0_full_checkpoint` also un-shards tensor-parallel heads,
vocabulary shards and expert-parallel experts (all-gathers along the recorded shard
dimensions), so a TP/EP run exports an ordinary single-process checkpoint; the reference
supports data parallelism only.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
import torch.nn as nn

from ..train.checkpoints import restore_rng_state, rng_state, save_checkpoint, to_host

FORMAT_VERSION = 1
SUCCESS_MARKER = "SUCCESS"


def fingerprint(value: Any) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, default=str, separators=(",", ":")).encode()).hexdigest()


def _barrier(context) -> None:
    if context.initialized and context.world_size > 1:
        context.barrier()


def _unwrap(model):
    return model.module if hasattr(model, "module") else model


def checkpoint_metadata(context, *, step: int, model_config=None, data_config=None, training_config=None,
                        registry_fingerprint: str | None = None) -> dict:
    from ..train.checkpoints import config_to_dict
    return {"format_version": FORMAT_VERSION, "step": int(step),
            "topology": {"world_size": context.world_size, "dp_size": context.dp_size, "tp_size": context.tp_size,
                         "ep_size": context.ep_size, "backend": context.backend,
                         "ep_overlays_tp": bool(getattr(context, "ep_overlays_tp", False))},
            "model_fingerprint": fingerprint(config_to_dict(model_config)),
            "data_fingerprint": fingerprint(config_to_dict(data_config)),
            "training_fingerprint": fingerprint(config_to_dict(training_config)),
            "parameter_registry_fingerprint": registry_fingerprint, "cache_schema_version": 1}


def save_distributed_checkpoint(path, *, model: nn.Module, context, step: int, optimizer=None, scheduler=None,
                                scaler=None, ema=None, trainer_state=None, curriculum=None, diagnostics=None,
                                sampler=None, model_config=None, data_config=None, training_config=None,
                                registry_fingerprint: str | None = None, extra: dict | None = None,
                                save_rng: bool = True) -> Path:
    target = Path(path)
    tmp = target.with_name(target.name + ".tmp")
    if context.is_global_zero:
        if target.exists():
            raise FileExistsError(f"checkpoint already exists: {target}")
        if tmp.exists():
            shutil.rmtree(tmp)
        tmp.mkdir(parents=True)
    _barrier(context)

    def st(obj):
        return None if obj is None else to_host(obj.state_dict())
    payload = {"model": to_host(_unwrap(model).state_dict()), "optimizer": st(optimizer), "scheduler": st(scheduler),
               "scaler": st(scaler), "ema": st(ema), "trainer_state": st(trainer_state), "curriculum": st(curriculum),
               "diagnostics": st(diagnostics), "sampler": st(sampler), "rng": rng_state() if save_rng else None,
               "extra": extra or {}}
    torch.save(payload, tmp / f"rank_{context.global_rank:05d}.pt")
    _barrier(context)
    if context.is_global_zero:
        meta = checkpoint_metadata(context, step=step, model_config=model_config, data_config=data_config,
                                   training_config=training_config, registry_fingerprint=registry_fingerprint)
        (tmp / "metadata.json").write_text(json.dumps(meta, indent=2, sort_keys=True) + "\n", encoding="utf-8")
        (tmp / SUCCESS_MARKER).write_text("ok\n", encoding="utf-8")
        os.replace(tmp, target)
    _barrier(context)
    return target


def load_distributed_checkpoint(path, *, model: nn.Module, context, optimizer=None, scheduler=None, scaler=None,
                                ema=None, trainer_state=None, curriculum=None, diagnostics=None, sampler=None,
                                restore_rng: bool = True, strict: bool = True) -> dict:
    src = Path(path)
    if not (src / SUCCESS_MARKER).is_file():
        raise ValueError(f"{src} is incomplete: missing {SUCCESS_MARKER} marker")
    meta = json.loads((src / "metadata.json").read_text(encoding="utf-8"))
    expected = {"world_size": context.world_size, "dp_size": context.dp_size, "tp_size": context.tp_size,
                "ep_size": context.ep_size}
    actual = {k: meta["topology"][k] for k in expected}
    if actual != expected:
        raise ValueError(f"distributed checkpoint topology change is unsupported: saved={actual}, current={expected}")
    payload = torch.load(src / f"rank_{context.global_rank:05d}.pt", map_location="cpu", weights_only=False)
    incompatible = _unwrap(model).load_state_dict(payload["model"], strict=strict)
    if optimizer is not None and payload.get("optimizer") is not None:
        optimizer.load_state_dict(payload["optimizer"])
    for owner, key in ((scheduler, "scheduler"), (scaler, "scaler"), (ema, "ema"), (trainer_state, "trainer_state"),
                       (curriculum, "curriculum"), (diagnostics, "diagnostics"), (sampler, "sampler")):
        if owner is not None and payload.get(key) is not None:
            owner.load_state_dict(payload[key])
    if restore_rng:
        restore_rng_state(payload.get("rng"))
    return {"metadata": meta, "extra": payload.get("extra", {}), "sampler_state": payload.get("sampler"),
            "missing_keys": list(incompatible.missing_keys), "unexpected_keys": list(incompatible.unexpected_keys)}


@torch.no_grad()
def _gather(t: torch.Tensor, dim: int, group) -> torch.Tensor:
    n = dist.get_world_size(group)
    parts = [torch.empty_like(t) for _ in range(n)]
    dist.all_gather(parts, t.contiguous(), group=group)
    return torch.cat(parts, dim=dim)


@torch.no_grad()
def full_state_dict(model: nn.Module, context) -> dict:
    """Single-process (unsharded) state dict, identical on every rank; collective."""
    from ..models.moe import GroupedRoutedExperts
    from .kimi_tp import TensorParallelKDA, TensorParallelMLA
    from .tensor_parallel import VocabParallelEmbedding, VocabParallelLMHead
    raw = _unwrap(model)
    sd = raw.state_dict(keep_vars=False)
    out = {}
    handled = set()
    for name, mod in raw.named_modules():
        prefix = name + "." if name else ""
        if isinstance(mod, (TensorParallelKDA, TensorParallelMLA)):
            for pname, dim in mod.shard_dims.items():
                key = f"{prefix}inner.{pname}"
                if key not in sd:
                    continue
                v = sd[key]
                out[f"{prefix}{pname}"] = v if dim is None else _gather(v, dim, mod.group)
                handled.add(key)
            for key in [k for k in sd if k.startswith(prefix + "inner.") and k not in handled]:
                out[key.replace(prefix + "inner.", prefix, 1)] = sd[key]
                handled.add(key)
        elif isinstance(mod, (VocabParallelEmbedding, VocabParallelLMHead)) and prefix + "weight" in sd:
            key = prefix + "weight"
            if key not in handled:
                out[key] = _gather(sd[key], 0, mod.group)
                handled.add(key)
            if isinstance(mod, VocabParallelLMHead) and prefix + "bias" in sd:
                out[prefix + "bias"] = _gather(sd[prefix + "bias"], 0, mod.group)
                handled.add(prefix + "bias")
        elif isinstance(mod, GroupedRoutedExperts) and getattr(mod, "_kimi_expert_parallel", None) is not None:
            group = getattr(mod, "_kimi_ep_group", None)
            for e_key in [k for k in sd if k.startswith(prefix) and ".transform." in k]:
                handled.add(e_key)
            stacked = {n: _gather(getattr(mod, n).detach(), 0, group) for n in ("gate_proj", "up_proj", "down_proj")}
            for n, full in stacked.items():
                for e in range(full.shape[0]):
                    out[f"{prefix}{e}.transform.{n}.weight"] = full[e]
    for k, v in sd.items():
        if k not in handled and k not in out:
            out[k] = v
    return out


def export_rank0_full_checkpoint(path, *, model: nn.Module, context, model_config=None, **kw) -> Path | None:
    """Write an ordinary single-process checkpoint (format v2) from a sharded run (rank 0)."""
    sd = full_state_dict(model, context) if context.initialized else _unwrap(model).state_dict()

    class _Holder(nn.Module):
        def state_dict(self, *a, **k):
            return sd
    target = None
    if context.is_global_zero:
        target = save_checkpoint(path, _Holder(), model_config=model_config, **kw)
    _barrier(context)
    return target


__all__ = ["FORMAT_VERSION", "SUCCESS_MARKER", "fingerprint", "checkpoint_metadata", "save_distributed_checkpoint",
           "load_distributed_checkpoint", "full_state_dict", "export_rank0_full_checkpoint"]
