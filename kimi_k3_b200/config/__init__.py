"""Strict YAML configuration (data / model / training / inference profiles)."""
from .yaml_utils import (ConfigError, KimiPipelinePaths, dataclass_kwargs, expect_mapping,  # noqa: F401
                         load_yaml_mapping, reject_unknown_keys, resolve_kimi_pipeline_profile)
