"""L0 primitives: short causal conv, SiTU-GLU, head-wise and plain RMSNorm, gates.

Parity targets (reference paths):
  * ``src/kimi_primitives/short_conv.py:12-98``  CausalShortConv1D (lag-ordered weights)
  * ``src/kimi_primitives/situ_glu.py:9-98``     softcap / SiTU-GLU
  * ``src/kimi_primitives/headwise_rmsnorm.py:7-65``
  * ``src/kimi_primitives/output_gate.py:9-74``  FullRankOutputGate
  * ``src/transformer_modules/rms_norm.py:6-72`` RMSNorm

Parameter names and initialisation match the reference so state dicts load
unchanged.  On CUDA tensors the hot paths (RMSNorm, SiTU activation) route to the
sm_100a kernels in :mod:`kimi_k3_b200.ops`; CPU tensors use the PyTorch math below,
which is also the numerical oracle for the kernels.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops as _ops
from .linear import Linear


# --------------------------------------------------------------------------- states
@dataclass
class ShortConvState:
    """Convolution history ``[B, K-1, C]`` (the last K-1 inputs)."""

    buffer: torch.Tensor

    def __post_init__(self) -> None:
        if not isinstance(self.buffer, torch.Tensor) or self.buffer.ndim != 3:
            raise ValueError("ShortConvState.buffer must have shape [B, K-1, C]")

    def clone(self) -> "ShortConvState":
        return ShortConvState(self.buffer.clone())


# --------------------------------------------------------------------------- heads
def split_heads(hidden_states: torch.Tensor, num_heads: int) -> torch.Tensor:
    if hidden_states.ndim != 3:
        raise ValueError("hidden_states must have shape [B,T,D]")
    b, t, d = hidden_states.shape
    if num_heads <= 0 or d % num_heads:
        raise ValueError(f"model width {d} must be divisible by num_heads={num_heads}")
    return hidden_states.reshape(b, t, num_heads, d // num_heads)


def combine_heads(head_states: torch.Tensor) -> torch.Tensor:
    if head_states.ndim != 4:
        raise ValueError("head_states must have shape [B,T,H,Dh]")
    b, t, h, dh = head_states.shape
    return head_states.reshape(b, t, h * dh)


def _low_to_fp32(x: torch.Tensor) -> torch.Tensor:
    return x.float() if x.dtype in (torch.float16, torch.bfloat16) else x


# --------------------------------------------------------------------------- norms
def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    """fp32-accumulated RMSNorm; output cast back before the affine multiply."""
    work = _low_to_fp32(x)
    y = work * torch.rsqrt(work.pow(2).mean(dim=-1, keepdim=True) + eps)
    if y.dtype != x.dtype:
        y = y.to(x.dtype)
    if weight is not None:
        y = y * weight.to(x.dtype)
    return y


class RMSNorm(nn.Module):
    """RMSNorm over the last axis with a learnable weight (init ones)."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        if dim <= 0:
            raise ValueError(f"dim must be > 0, got {dim}")
        if eps <= 0:
            raise ValueError(f"eps must be > 0, got {eps}")
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.shape[-1] != self.dim:
            raise ValueError(f"expected last dimension {self.dim}, got {x.shape[-1]}")
        if _ops.use_kernels(x):
            return _ops.rms_norm(x, self.weight, self.eps)
        return rms_norm_reference(x, self.weight, self.eps)


class HeadwiseRMSNorm(nn.Module):
    """RMS-normalise ``[B,T,H,Dh]`` over ``Dh`` with a per-head affine."""

    def __init__(self, num_heads: int, head_dim: int, eps: float = 1e-6,
                 elementwise_affine: bool = True, per_head_affine: bool = True,
                 *, device=None, dtype=None):
        super().__init__()
        if num_heads <= 0 or head_dim <= 0:
            raise ValueError("num_heads and head_dim must be > 0")
        if eps <= 0:
            raise ValueError("eps must be > 0")
        self.num_heads, self.head_dim, self.eps = num_heads, head_dim, float(eps)
        self.elementwise_affine, self.per_head_affine = elementwise_affine, per_head_affine
        if elementwise_affine:
            shape = (num_heads, head_dim) if per_head_affine else (head_dim,)
            self.weight = nn.Parameter(torch.ones(shape, device=device, dtype=dtype))
        else:
            self.register_parameter("weight", None)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.ndim != 4 or x.shape[2:] != (self.num_heads, self.head_dim):
            raise ValueError(f"expected [B,T,{self.num_heads},{self.head_dim}], got {tuple(x.shape)}")
        if self.weight is not None and self.per_head_affine and _ops.use_kernels(x):
            b, t, h, dh = x.shape
            return _ops.rms_norm(x.reshape(b, t * h, dh), self.weight, self.eps,
                                 per_row_weight_period=h).reshape(b, t, h, dh)
        work = _low_to_fp32(x)
        y = (work * torch.rsqrt(work.square().mean(dim=-1, keepdim=True) + self.eps)).to(x.dtype)
        if self.weight is not None:
            w = self.weight.to(x.dtype)
            y = y * (w[None, None] if self.per_head_affine else w[None, None, None])
        return y


# --------------------------------------------------------------------------- conv
class CausalShortConv1D(nn.Module):
    """Depthwise causal conv over ``[B,T,C]``; ``weight[c, j]`` multiplies ``x[t-j, c]``."""

    def __init__(self, channels: int, kernel_size: int = 4, bias: bool = False, *, device=None, dtype=None):
        super().__init__()
        if channels <= 0 or kernel_size <= 0:
            raise ValueError("channels and kernel_size must be > 0")
        self.channels, self.kernel_size = channels, kernel_size
        self.weight = nn.Parameter(torch.empty(channels, kernel_size, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.empty(channels, device=device, dtype=dtype)) if bias else None
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.normal_(self.weight, mean=0.0, std=0.02)
        if self.bias is not None:
            nn.init.zeros_(self.bias)

    def _history(self, x: torch.Tensor, state: ShortConvState | None) -> torch.Tensor:
        hist = self.kernel_size - 1
        if state is None:
            return x.new_zeros(x.shape[0], hist, self.channels)
        expected = (x.shape[0], hist, self.channels)
        if tuple(state.buffer.shape) != expected:
            raise ValueError(f"state buffer must have shape {expected}")
        if state.buffer.device != x.device or state.buffer.dtype != x.dtype:
            raise ValueError("state buffer must match the input device and dtype")
        return state.buffer

    def forward(self, x: torch.Tensor, state: ShortConvState | None = None, return_state: bool = False):
        if x.ndim != 3 or x.shape[-1] != self.channels:
            raise ValueError(f"x must have shape [B,T,{self.channels}]")
        history = self._history(x, state)
        combined = torch.cat((history, x), dim=1)
        if x.shape[1] == 0:
            out = x.clone()
        else:
            out = F.conv1d(combined.transpose(1, 2), self.weight.flip(-1).unsqueeze(1),
                           self.bias, groups=self.channels).transpose(1, 2)
        if not return_state:
            return out
        hist = self.kernel_size - 1
        nxt = combined[:, :0] if hist == 0 else combined[:, -hist:]
        return out, ShortConvState(nxt.clone())


# --------------------------------------------------------------------------- SiTU-GLU
def softcap(x: torch.Tensor, beta: float) -> torch.Tensor:
    if beta <= 0:
        raise ValueError("beta must be > 0")
    return torch.tanh(x / beta) * beta


def situ_glu_activation(gate: torch.Tensor, up: torch.Tensor, beta_gate: float = 4.0,
                        beta_up: float = 25.0) -> torch.Tensor:
    """``softcap(g, bg) * sigmoid(g) * softcap(u, bu)``."""
    if gate.shape != up.shape:
        raise ValueError("gate and up must have identical shapes")
    if beta_gate <= 0 or beta_up <= 0:
        raise ValueError("beta_gate and beta_up must be > 0")
    if _ops.use_kernels(gate):
        return _ops.situ_glu(gate, up, beta_gate, beta_up)
    return softcap(gate, beta_gate) * torch.sigmoid(gate) * softcap(up, beta_up)


class SiTUGLU(nn.Module):
    """``down(softcap(gate(x),4) * sigmoid(gate(x)) * softcap(up(x),25))``."""

    def __init__(self, d_model: int, hidden_dim: int, beta_gate: float = 4.0, beta_up: float = 25.0,
                 bias: bool = False, output_bias: bool | None = None, init_std: float = 0.02,
                 *, device=None, dtype=None):
        super().__init__()
        if d_model <= 0 or hidden_dim <= 0 or beta_gate <= 0 or beta_up <= 0 or init_std <= 0:
            raise ValueError("invalid SiTU-GLU configuration")
        self.d_model, self.hidden_dim = d_model, hidden_dim
        self.beta_gate, self.beta_up = float(beta_gate), float(beta_up)
        output_bias = bias if output_bias is None else output_bias
        kw = {"device": device, "dtype": dtype}
        self.gate_proj = Linear(d_model, hidden_dim, bias=bias, **kw)
        self.up_proj = Linear(d_model, hidden_dim, bias=bias, **kw)
        self.down_proj = Linear(hidden_dim, d_model, bias=output_bias, **kw)
        self.init_std = float(init_std)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        for proj in (self.gate_proj, self.up_proj, self.down_proj):
            nn.init.normal_(proj.weight, mean=0.0, std=self.init_std)
            if proj.bias is not None:
                nn.init.zeros_(proj.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.ndim < 1 or x.shape[-1] != self.d_model:
            raise ValueError(f"x must have shape [...,{self.d_model}]")
        hidden = situ_glu_activation(self.gate_proj(x), self.up_proj(x), self.beta_gate, self.beta_up)
        return self.down_proj(hidden)


# --------------------------------------------------------------------------- gates
class FullRankOutputGate(nn.Module):
    """``output_proj(sigmoid(gate_proj(residual_input)) * attention_output)``."""

    def __init__(self, d_model: int, bias: bool = False, output_bias: bool = False, init_std: float = 0.02,
                 *, device=None, dtype=None, value_width: int | None = None):
        super().__init__()
        value_width = d_model if value_width is None else int(value_width)
        if d_model <= 0 or init_std <= 0 or value_width <= 0:
            raise ValueError("invalid output gate configuration")
        # value_width < d_model only for a tensor-parallel shard owning a subset of the heads
        self.d_model, self.value_width, self.init_std = d_model, value_width, float(init_std)
        kw = {"device": device, "dtype": dtype}
        self.gate_proj = Linear(d_model, value_width, bias=bias, **kw)
        self.output_proj = Linear(value_width, d_model, bias=output_bias, **kw)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        for proj in (self.gate_proj, self.output_proj):
            nn.init.normal_(proj.weight, mean=0.0, std=self.init_std)
            if proj.bias is not None:
                nn.init.zeros_(proj.bias)

    def gate_values(self, residual_input: torch.Tensor) -> torch.Tensor:
        if residual_input.ndim != 3 or residual_input.shape[-1] != self.d_model:
            raise ValueError(f"residual_input must have shape [B,T,{self.d_model}]")
        return torch.sigmoid(self.gate_proj(residual_input))

    def forward(self, attention_output: torch.Tensor, residual_input: torch.Tensor, *, return_gate: bool = False,
                gate_logits: torch.Tensor | None = None):
        """``gate_logits``: ``gate_proj(residual_input)`` already computed (by a fused projection group)."""
        if attention_output.ndim != 3 or attention_output.shape[-1] != self.value_width:
            raise ValueError(f"attention_output must have shape [B,T,{self.value_width}]")
        if attention_output.shape[:2] != residual_input.shape[:2] or residual_input.shape[-1] != self.d_model:
            raise ValueError("attention_output and residual_input must share [B,T] (residual width d_model)")
        logits = self.gate_proj(residual_input) if gate_logits is None else gate_logits
        if _ops.use_kernels(logits):
            gated = _ops.sigmoid_mul(logits, attention_output)
            gate = None
        else:
            gate = torch.sigmoid(logits)
            gated = gate * attention_output
        out = self.output_proj(gated)
        if return_gate:
            return out, (torch.sigmoid(logits) if gate is None else gate)
        return out


class PrimitiveAttentionPostprocess(nn.Module):
    """Head-wise norm, head combine, then the full-rank output gate."""

    def __init__(self, num_heads: int, head_dim: int, *, eps: float = 1e-6, norm_affine: bool = True,
                 per_head_affine: bool = True, gate_bias: bool = False, output_bias: bool = False):
        super().__init__()
        self.num_heads, self.head_dim, self.d_model = num_heads, head_dim, num_heads * head_dim
        self.norm = HeadwiseRMSNorm(num_heads, head_dim, eps=eps, elementwise_affine=norm_affine,
                                    per_head_affine=per_head_affine)
        self.output_gate = FullRankOutputGate(self.d_model, bias=gate_bias, output_bias=output_bias)

    def forward(self, head_outputs, residual_input, *, return_gate: bool = False):
        return self.output_gate(combine_heads(self.norm(head_outputs)), residual_input, return_gate=return_gate)


@dataclass
class KDAProjectionOutput:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    beta: torch.Tensor
    alpha: torch.Tensor


@dataclass
class AttentionModuleOutput:
    hidden_states: torch.Tensor
    state: object | None = None
    diagnostics: dict | None = None


__all__ = [
    "ShortConvState", "split_heads", "combine_heads", "rms_norm_reference", "RMSNorm",
    "HeadwiseRMSNorm", "CausalShortConv1D", "softcap", "situ_glu_activation", "SiTUGLU",
    "FullRankOutputGate", "PrimitiveAttentionPostprocess", "KDAProjectionOutput", "AttentionModuleOutput",
]
