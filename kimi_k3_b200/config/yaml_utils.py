"""Strict YAML helpers shared by every configuration loader.

Behaviour parity: ``configuration/yaml_utils.py`` (reference) rejects unknown
keys loudly and requires mapping roots; these helpers keep that contract so
reference profile YAMLs parse unchanged.
"""
from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import yaml


class ConfigError(ValueError):
    """A YAML document violates the public configuration schema."""


def load_yaml_mapping(path: str | Path) -> tuple[Path, dict[str, Any]]:
    resolved = Path(path).expanduser().resolve()
    if not resolved.is_file():
        raise FileNotFoundError(f"configuration file does not exist: {resolved}")
    with resolved.open("r", encoding="utf-8") as handle:
        values = yaml.safe_load(handle)
    if not isinstance(values, Mapping):
        raise ConfigError(f"{resolved} must contain a YAML mapping")
    return resolved, dict(values)


def expect_mapping(values: dict, key: str, *, path: str, required: bool = True) -> dict:
    """Pop ``key`` from ``values`` and require it to be a mapping."""
    if key not in values:
        if required:
            raise ConfigError(f"{path}.{key} is required")
        return {}
    nested = values.pop(key)
    if nested is None and not required:
        return {}
    if not isinstance(nested, Mapping):
        raise ConfigError(f"{path}.{key} must be a mapping")
    return dict(nested)


def reject_unknown_keys(values: Mapping, *, path: str) -> None:
    if values:
        raise ConfigError(
            f"unknown keys in {path}: " + ", ".join(sorted(map(str, values)))
        )


def dataclass_kwargs(values: Mapping, dataclass_type, *, path: str) -> dict:
    """Check ``values`` against the fields of ``dataclass_type``."""
    fields = dataclass_type.__dataclass_fields__
    unknown = {k: values[k] for k in values if k not in fields}
    reject_unknown_keys(unknown, path=path)
    return dict(values)


@dataclass(frozen=True)
class KimiPipelinePaths:
    root: Path
    data: Path
    model: Path
    training: Path


def resolve_kimi_pipeline_profile(profile: str | Path) -> KimiPipelinePaths:
    """Resolve a profile directory holding ``data/model/training.yaml``."""
    root = Path(profile).expanduser().resolve()
    if not root.is_dir():
        raise ConfigError(f"Kimi pipeline profile is not a directory: {root}")
    paths = KimiPipelinePaths(root, root / "data.yaml", root / "model.yaml", root / "training.yaml")
    missing = [p.name for p in (paths.data, paths.model, paths.training) if not p.is_file()]
    if missing:
        raise ConfigError(f"incomplete Kimi pipeline profile {root}: missing " + ", ".join(missing))
    return paths


__all__ = [
    "ConfigError", "load_yaml_mapping", "expect_mapping", "reject_unknown_keys",
    "dataclass_kwargs", "KimiPipelinePaths", "resolve_kimi_pipeline_profile",
]
