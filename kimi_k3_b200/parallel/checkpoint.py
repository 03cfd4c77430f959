"""Distributed checkpoints: one file per rank, committed atomically as a directory.

Parity: ``training/distributed/checkpoint.py:109-303`` (reference): a temporary directory
receives ``rank_%05d.pt`` from every rank, rank 0 adds ``metadata.json`` (topology and
sha256 fingerprints of the model / data / training configs and the optimizer parameter
registry) and a ``SUCCESS`` marker, then renames the directory into place; loading requires
the marker and the same topology. The on-disk layout is kept identical.

Sharded data parallelism (``data_parallel.mode: fsdp``): every rank's file holds its own shards
(:class:`LocalShard`) of the DTensor parameters and optimizer states; loading rebuilds the DTensors
around the live parameters' meshes, so a sharded run resumes on the same topology.

Addition: :func:`export_rank0_full_checkpoint` also un-shards tensor-parallel heads,
vocabulary shards and expert-parallel experts (all-gathers along the recorded shard
dimensions) and gathers fully sharded parameters, so a TP / EP / FSDP run exports an ordinary
single-process checkpoint; the reference supports data parallelism only.
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
from .fsdp import reshard_all

FORMAT_VERSION = 1
SUCCESS_MARKER = "SUCCESS"


def fingerprint(value: Any) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, default=str, separators=(",", ":")).encode()).hexdigest()


def _barrier(context) -> None:
    if context.initialized and context.world_size > 1:
        context.barrier()


def _unwrap(model):
    return model.module if hasattr(model, "module") else model


# --------------------------------------------------------------------------- sharded (FSDP) values
class LocalShard:
    """This rank's shard of a sharded (DTensor) value, as stored in its per-rank file.  Loading
    rebuilds the DTensor around it with the mesh and placements of the live parameter."""

    __slots__ = ("tensor",)

    def __init__(self, tensor: torch.Tensor):
        self.tensor = tensor

    def __reduce__(self):
        return (LocalShard, (self.tensor,))


def _dtensor_type():
    try:
        from torch.distributed.tensor import DTensor
    except ImportError:  # pragma: no cover - every supported torch has it
        return None
    return DTensor


def _to_local_shards(obj):
    dt = _dtensor_type()
    if dt is not None and isinstance(obj, dt):
        return LocalShard(obj.to_local().detach().cpu())
    if isinstance(obj, dict):
        return {k: _to_local_shards(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [_to_local_shards(v) for v in obj]
    if isinstance(obj, tuple):
        return tuple(_to_local_shards(v) for v in obj)
    return obj


def _as_dtensor(local: torch.Tensor, like, dtype=None):
    dt = _dtensor_type()
    return dt.from_local(local.to(device=like.device, dtype=dtype or local.dtype), like.device_mesh, like.placements,
                         shape=like.shape, stride=like.stride(), run_check=False)


def _model_state_for_load(model: nn.Module, saved: dict) -> dict:
    """Rebuild the DTensor entries of a saved model state around the live parameters' meshes."""
    dt = _dtensor_type()
    live = model.state_dict()
    out = dict(saved)
    for k, v in saved.items():
        if isinstance(v, LocalShard):
            cur = live.get(k)
            if dt is None or not isinstance(cur, dt):
                raise ValueError(f"checkpoint holds a shard of {k}, but the model's {k} is not sharded")
            out[k] = _as_dtensor(v.tensor, cur, dtype=cur.dtype)
    return out


def _restore_optimizer_shards(optimizer) -> None:
    """After ``load_state_dict``: optimizer states saved as shards become DTensors of their parameter."""
    inner = [o for o in (getattr(optimizer, "muon", None), getattr(optimizer, "adamw", None)) if o is not None]
    for opt in inner or [optimizer]:
        for p, st in getattr(opt, "state", {}).items():
            for key, val in list(st.items()):
                if isinstance(val, LocalShard):
                    st[key] = _as_dtensor(val.tensor, p)


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
        return None if obj is None else to_host(_to_local_shards(obj.state_dict()))
    reshard_all(_unwrap(model))
    payload = {"model": st(_unwrap(model)), "optimizer": st(optimizer), "scheduler": st(scheduler),
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
    raw = _unwrap(model)
    incompatible = raw.load_state_dict(_model_state_for_load(raw, payload["model"]), strict=strict)
    if optimizer is not None and payload.get("optimizer") is not None:
        optimizer.load_state_dict(payload["optimizer"])
        _restore_optimizer_shards(optimizer)
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
    reshard_all(raw)
    sd = raw.state_dict(keep_vars=False)
    dt = _dtensor_type()
    if dt is not None:  # sharded data parallelism: gather every shard (same key order on all ranks)
        sd = {k: (v.full_tensor() if isinstance(v, dt) else v) for k, v in sd.items()}
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


__all__ = ["FORMAT_VERSION", "SUCCESS_MARKER", "LocalShard", "fingerprint", "checkpoint_metadata", "save_distributed_checkpoint",
           "load_distributed_checkpoint", "full_state_dict", "export_rank0_full_checkpoint"]
