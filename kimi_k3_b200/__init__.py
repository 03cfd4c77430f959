"""kimi_k3_b200: a Blackwell (sm_100a) native Kimi-K3 training and inference framework.

Public API (mirrors the reference project's entry points):
  * models:   ``KimiK3``, ``KimiK3Config``, ``build_model_from_yaml``, ``load_model_config``
  * training: ``train_kimiK3``, ``train_kimi_from_yaml``, ``train_one_epoch``, ``build_kimi_optimizer``,
    ``build_muon_adamw_optimizer``, ``build_adamw_optimizer``
  * inference: ``inference_autoregressive``, ``generate_tokens``, ``load_kimi_checkpoint``
  * distributed: ``parallelize_kimi_model``, ``setup_distributed``
"""
from .models import (KimiK3, KimiK3Config, KimiK3Output, kimi_k3_canonical_config,  # noqa: F401
                     kimi_k3_cpu_tiny_config)

__version__ = "0.1.0"


def __getattr__(name):  # lazy access to the heavier subsystems
    if name in ("build_model_from_yaml", "load_model_config", "build_model_config_from_mapping"):
        from .config import model_yaml
        return getattr(model_yaml, name)
    if name in ("train_kimiK3", "train_kimi_from_yaml"):
        from .train import trainer
        return getattr(trainer, name)
    if name == "build_kimi_optimizer":
        from .train.optimizer import build_kimi_optimizer
        return build_kimi_optimizer
    if name == "train_one_epoch":
        from .train.loop import train_one_epoch
        return train_one_epoch
    if name in ("build_muon_adamw_optimizer", "build_adamw_optimizer"):
        from .train import legacy
        return getattr(legacy, name)
    if name == "parallelize_kimi_model":
        from .parallel.parallelize import parallelize_kimi_model
        return parallelize_kimi_model
    if name == "setup_distributed":
        from .parallel.environment import setup_distributed
        return setup_distributed
    if name in ("inference_autoregressive", "generate_tokens", "load_kimi_checkpoint"):
        from . import infer
        return getattr(infer, name)
    raise AttributeError(name)
