"""The projection layer of every model in this package.

``Linear`` is ``nn.Linear`` (same parameters, state-dict keys and initialisation) whose CUDA
forward under bf16 compute runs :func:`kimi_k3_b200.ops.linear`: the tcgen05 GEMM reading the
weight's bf16 mirror, with the weight gradient produced in fp32 by the same kernel.  On the CPU,
in fp32, or with ``KIMI_K3_KERNELS=0`` it is exactly ``nn.Linear``.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops as _ops


class Linear(nn.Linear):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if _ops.use_kernels(x) and _ops.linear_supported(x, self.weight):
            return _ops.linear(x, self.weight, self.bias)
        return F.linear(x, self.weight, self.bias)


__all__ = ["Linear"]
