"""Device ops: the sm_100a CUDA kernels behind the model's hot paths.

Every public function here takes CUDA tensors and runs the extension built from
``csrc/`` (``kimi_k3_b200/_C*.so``).  ``use_kernels(x)`` is the single switch the
model uses: True for CUDA tensors unless ``KIMI_K3_KERNELS=0``.  When it is True
and the extension cannot be loaded, the call raises -- there is no silent
fallback on the GPU.  CPU tensors never reach this module (the modules keep
their PyTorch math, which doubles as the numerical oracle for the kernels).
"""
from __future__ import annotations

import os

import torch

from . import _loader
from .functional import (attnres_mix, conv_silu_norm, conv_silu_norm_step, flash_attention, kda_chunk, kda_decay,
                         kda_decode_step, linear, linear_cross_entropy, linear_group, linear_group_supported,
                         linear_supported, mark_seen, mla_absorbed_decode, mla_decode_supported,
                         moe_grouped_experts, qb_histogram, rms_norm, router_topk, sample_tokens, sigmoid_mul,
                         situ_glu)


def kernels_enabled() -> bool:
    return os.environ.get("KIMI_K3_KERNELS", "1") != "0"


def use_kernels(x: torch.Tensor) -> bool:
    """True when ``x`` lives on CUDA and the native kernels are enabled."""
    if not (isinstance(x, torch.Tensor) and x.is_cuda and kernels_enabled()):
        return False
    _loader.require()
    return True


__all__ = [
    "kernels_enabled", "use_kernels", "linear", "linear_supported", "linear_group", "linear_group_supported", "rms_norm", "situ_glu", "sigmoid_mul", "kda_chunk", "kda_decode_step",
    "conv_silu_norm", "kda_decay", "flash_attention", "mla_absorbed_decode", "router_topk", "qb_histogram",
    "moe_grouped_experts", "attnres_mix", "linear_cross_entropy", "conv_silu_norm_step", "mla_decode_supported",
    "sample_tokens", "mark_seen",
]
