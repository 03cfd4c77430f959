"""Single-process training checkpoints (``format_version`` 2), written atomically.

Parity: ``training/checkpoints.py:43-165`` (reference). The payload keys are the reference's,
so checkpoints move between the two implementations: model/optimizer/scheduler/scaler state,
epoch and global step, model and training configs, history, RNG state (python, numpy, torch,
every CUDA device), EMA, trainer state, curriculum (under both of its key names), metadata and
diagnostics. The file is written next to its destination and moved into place with
``os.replace``, so a crash never leaves a truncated checkpoint.

B200 notes: state dicts are copied to host memory before pickling (device tensors would pin
the GPU in the serialised file and make loads device-dependent); ``keep_last`` pruning and a
``latest`` pointer file support long runs.
"""
from __future__ import annotations

import os
import random
import re
from dataclasses import asdict, is_dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch
import torch.nn as nn

FORMAT_VERSION = 2


def rng_state() -> dict:
    return {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state(),
            "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None}


def restore_rng_state(state: dict | None) -> None:
    if not state:
        return
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"].cpu())
    if torch.cuda.is_available() and state.get("cuda") is not None:
        torch.cuda.set_rng_state_all(state["cuda"])


def config_to_dict(config: Any) -> Any:
    if config is None or isinstance(config, (str, int, float, bool, list, dict)):
        return config
    if is_dataclass(config):
        return asdict(config)
    if hasattr(config, "to_dict"):
        return config.to_dict()
    return dict(vars(config)) if hasattr(config, "__dict__") else str(config)


def to_host(obj):
    """Recursively copy tensors of a state structure to host memory."""
    if torch.is_tensor(obj):
        return obj.detach().cpu() if obj.device.type != "cpu" else obj
    if isinstance(obj, dict):
        return {k: to_host(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [to_host(v) for v in obj]
    if isinstance(obj, tuple):
        return tuple(to_host(v) for v in obj)
    return obj


def unwrap(model: nn.Module) -> nn.Module:
    return model.module if hasattr(model, "module") else model


def _state(obj):
    return None if obj is None else to_host(obj.state_dict())


def save_checkpoint(path, model, *, optimizer=None, scheduler=None, scaler=None, epoch: int = 0,
                    global_step: int = 0, model_config=None, training_config=None, history=None, ema=None,
                    trainer_state=None, curriculum=None, metadata=None, save_rng_state: bool = True,
                    diagnostics=None) -> Path:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    curriculum_state = _state(curriculum)
    payload = {
        "format_version": FORMAT_VERSION,
        "model_state_dict": to_host(unwrap(model).state_dict()),
        "optimizer_state_dict": _state(optimizer),
        "scheduler_state_dict": _state(scheduler),
        "scaler_state_dict": _state(scaler),
        "epoch": int(epoch),
        "global_step": int(global_step),
        "model_config": config_to_dict(model_config),
        "training_config": config_to_dict(training_config),
        "history": history or {},
        "rng_state": rng_state() if save_rng_state else None,
        "ema_state_dict": _state(ema),
        "trainer_state_dict": _state(trainer_state),
        "curriculum_state_dict": curriculum_state,
        "context_curriculum": curriculum_state,
        "metadata": metadata or {},
        "diagnostics_state_dict": _state(diagnostics),
    }
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(payload, tmp)
    os.replace(tmp, path)
    return path


def load_checkpoint(path, model, *, optimizer=None, scheduler=None, scaler=None, map_location="cpu",
                    strict: bool = True, restore_rng: bool = False, ema=None, trainer_state=None, curriculum=None,
                    diagnostics=None) -> dict:
    payload = torch.load(Path(path), map_location=map_location, weights_only=False)
    incompatible = unwrap(model).load_state_dict(payload["model_state_dict"], strict=strict)
    for obj, key in ((optimizer, "optimizer_state_dict"), (scheduler, "scheduler_state_dict"),
                     (scaler, "scaler_state_dict")):
        if obj is not None and payload.get(key) is not None:
            obj.load_state_dict(payload[key])
    if restore_rng:
        restore_rng_state(payload.get("rng_state"))
    if ema is not None and payload.get("ema_state_dict") is not None:
        ema.load_state_dict(payload["ema_state_dict"], strict=strict)
    if trainer_state is not None and payload.get("trainer_state_dict") is not None:
        trainer_state.load_state_dict(payload["trainer_state_dict"])
    cur = payload.get("context_curriculum") or payload.get("curriculum_state_dict")
    if curriculum is not None and cur is not None:
        curriculum.load_state_dict(cur)
    if diagnostics is not None and payload.get("diagnostics_state_dict") is not None:
        diagnostics.load_state_dict(payload["diagnostics_state_dict"])
    return {"format_version": payload.get("format_version", 1), "epoch": payload.get("epoch", 0),
            "global_step": payload.get("global_step", 0), "model_config": payload.get("model_config"),
            "training_config": payload.get("training_config"), "history": payload.get("history", {}),
            "trainer_state": payload.get("trainer_state_dict"), "curriculum_state": cur,
            "metadata": payload.get("metadata", {}), "diagnostics_state": payload.get("diagnostics_state_dict"),
            "missing_keys": list(incompatible.missing_keys), "unexpected_keys": list(incompatible.unexpected_keys)}


_STEP_RE = re.compile(r"step_(\d+)")


def checkpoint_step(path) -> int:
    m = _STEP_RE.search(Path(path).name)
    return int(m.group(1)) if m else -1


def list_checkpoints(directory, pattern: str = "*.pt") -> list:
    """Checkpoints in ``directory`` ordered by the step number in their name (then mtime)."""
    d = Path(directory)
    if not d.is_dir():
        return []
    files = [p for p in d.glob(pattern) if p.is_file() and not p.name.endswith(".tmp")]
    return sorted(files, key=lambda p: (checkpoint_step(p), p.stat().st_mtime))


def prune_checkpoints(directory, keep_last: int, *, protect=(), pattern: str = "step_*.pt") -> list:
    """Delete all but the newest ``keep_last`` step checkpoints; ``protect`` names survive."""
    if keep_last is None or keep_last <= 0:
        return []
    protected = {Path(p).resolve() for p in protect}
    files = [p for p in list_checkpoints(directory, pattern) if p.resolve() not in protected]
    removed = files[:-keep_last] if len(files) > keep_last else []
    for p in removed:
        p.unlink(missing_ok=True)
    return removed


def write_latest_pointer(directory, path) -> Path:
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    ptr = d / "latest"
    tmp = d / "latest.tmp"
    tmp.write_text(Path(path).name + "\n")
    os.replace(tmp, ptr)
    return ptr


def resolve_resume_path(value, directory=None):
    """``value`` may be a file, ``"latest"`` (pointer file or newest checkpoint) or None."""
    if value in (None, "", False):
        return None
    if value == "latest":
        if directory is None:
            raise ValueError("resume='latest' needs a checkpoint directory")
        ptr = Path(directory) / "latest"
        if ptr.is_file():
            cand = Path(directory) / ptr.read_text().strip()
            if cand.is_file():
                return cand
        found = list_checkpoints(directory)
        return found[-1] if found else None
    p = Path(value)
    if not p.is_file():
        raise FileNotFoundError(f"checkpoint {p} does not exist")
    return p


__all__ = ["FORMAT_VERSION", "save_checkpoint", "load_checkpoint", "rng_state", "restore_rng_state",
           "config_to_dict", "to_host", "list_checkpoints", "prune_checkpoints", "write_latest_pointer",
           "resolve_resume_path", "checkpoint_step"]
