"""``inference.yaml``: ``inference:`` generation settings + optional ``distributed:`` (TP / EP
only; DDP/FSDP have no role at inference). Reference: ``inference/yaml_config.py:23-60``."""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

from ..config.yaml_utils import dataclass_kwargs, expect_mapping, load_yaml_mapping, reject_unknown_keys
from ..parallel.config import DistributedConfig, distributed_config_from_dict
from .config import GenerationConfig


@dataclass(frozen=True)
class InferenceYamlConfig:
    generation: GenerationConfig
    distributed: DistributedConfig
    source_path: Path


def load_inference_yaml_config(path) -> InferenceYamlConfig:
    source, root = load_yaml_mapping(path)
    root = dict(root)
    values = dict(expect_mapping(root, "inference", path="root"))
    dist_values = root.pop("distributed", None) or {}
    reject_unknown_keys(root, path="root")
    dist = distributed_config_from_dict(dist_values)
    if dist.data_parallel.mode != "none":
        raise ValueError("distributed inference does not use DDP/FSDP")
    return InferenceYamlConfig(GenerationConfig(**dataclass_kwargs(values, GenerationConfig, path="inference")), dist,
                               source)


def load_generation_config(path) -> GenerationConfig:
    return load_inference_yaml_config(path).generation


__all__ = ["InferenceYamlConfig", "load_inference_yaml_config", "load_generation_config"]
