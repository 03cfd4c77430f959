"""Kimi Delta Attention (KDA): per-channel gated delta rule with short convs.

Parity targets (reference paths):
  * ``src/kda/config.py:10-82``        KDAConfig
  * ``src/kda/projections.py:32-225``  q/k/v + ShortConv + SiLU + L2 norm, beta, low-rank decay
  * ``src/kda/decay.py:7-43``          g = g_min * sigmoid(exp(A_log) * z)
  * ``src/kda/recurrent.py:25-80``     exact token recurrence (decay, delta write, read)
  * ``src/kda/chunkwise.py:17-107``    chunked UT/WY form
  * ``src/kda/kda.py:38-206``          KimiDeltaAttention
  * ``src/kda/state.py:13-67``         KDAState

The chunk algebra implemented here (and in ``csrc/kda_chunk.cu``) is, per chunk
of C tokens with cumulative log-decay ``G = cumsum(g)``:

    A   = diag(beta) * strict_lower((k e^G)(k e^-G)^T)      (pairwise decay dots)
    M   = (I + A)^-1 diag(beta)
    W   = M (k e^G),  U = M v,  V' = U - W S
    O   = (q e^G) S + lower((q e^G)(k e^-G)^T) V'
    S  <- e^{G_C} S + (k e^{G_C - G})^T V'

Pairwise factors ``e^{G_i - G_j}`` are formed with a reference point between i
and j, so no factor exceeds one off the diagonal block (decay is bounded below
by ``g_min``, which bounds the diagonal-block factors).
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from typing import Literal

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops as _ops
from .linear import Linear
from ..runtime import host_checks
from .primitives import (CausalShortConv1D, FullRankOutputGate, HeadwiseRMSNorm, ShortConvState,
                         combine_heads)


# --------------------------------------------------------------------------- config
@dataclass(frozen=True)
class KDAConfig:
    d_model: int
    num_heads: int
    key_head_dim: int
    value_head_dim: int
    short_conv_kernel_size: int = 4
    decay_rank: int | None = None
    g_min: float = -5.0
    chunk_size: int = 64
    secondary_tile_size: int = 16
    eps: float = 1e-6
    projection_bias: bool = False
    short_conv_bias: bool = False
    beta_bias: bool = False
    output_gate_bias: bool = False
    output_bias: bool = False
    accumulate_state_in_fp32: bool = True
    decay_initializer: Literal["official_fla", "zeros"] = "official_fla"
    init_std: float = 0.02

    def __post_init__(self) -> None:
        for name in ("d_model", "num_heads", "key_head_dim", "value_head_dim",
                     "short_conv_kernel_size", "chunk_size", "secondary_tile_size"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be > 0, got {getattr(self, name)}")
        if self.d_model != self.num_heads * self.value_head_dim:
            raise ValueError("d_model must equal num_heads * value_head_dim")
        if self.decay_rank is not None and self.decay_rank <= 0:
            raise ValueError("decay_rank must be > 0 when provided")
        if self.g_min >= 0:
            raise ValueError("g_min must be negative")
        if self.secondary_tile_size > self.chunk_size:
            raise ValueError("secondary_tile_size must be <= chunk_size")
        if self.eps <= 0 or self.init_std <= 0:
            raise ValueError("eps and init_std must be > 0")
        if self.decay_initializer not in ("official_fla", "zeros"):
            raise ValueError("decay_initializer must be 'official_fla' or 'zeros'")

    @property
    def resolved_decay_rank(self) -> int:
        return self.value_head_dim if self.decay_rank is None else self.decay_rank

    @property
    def key_width(self) -> int:
        return self.num_heads * self.key_head_dim

    @property
    def value_width(self) -> int:
        return self.num_heads * self.value_head_dim

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "KDAConfig":
        return cls(**values)


# --------------------------------------------------------------------------- state
@dataclass
class KDAState:
    """Recurrent matrix ``[B,H,K,V]`` (fp32), three conv histories and offsets."""

    recurrent_state: torch.Tensor
    q_conv_state: ShortConvState
    k_conv_state: ShortConvState
    v_conv_state: ShortConvState
    sequence_offset: torch.Tensor
    # A serving cache owned by one decoder: decode kernels advance its tensors in place instead
    # of returning new ones (the previous step's state is not kept).
    inplace: bool = False

    def __post_init__(self) -> None:
        if self.recurrent_state.ndim != 4:
            raise ValueError("recurrent_state must have shape [B,H,K,V]")
        b = self.recurrent_state.shape[0]
        if tuple(self.sequence_offset.shape) != (b,):
            raise ValueError("sequence_offset must have shape [B]")
        if self.sequence_offset.dtype != torch.long:
            raise TypeError("sequence_offset must use torch.long")
        for s in (self.q_conv_state, self.k_conv_state, self.v_conv_state):
            if s.buffer.shape[0] != b:
                raise ValueError("all ShortConv states must match recurrent batch size")

    def clone(self) -> "KDAState":
        return KDAState(self.recurrent_state.clone(), self.q_conv_state.clone(), self.k_conv_state.clone(),
                        self.v_conv_state.clone(), self.sequence_offset.clone())

    def reorder(self, indices: torch.Tensor) -> "KDAState":
        if indices.ndim != 1 or indices.dtype != torch.long:
            raise ValueError("indices must be a rank-1 torch.long tensor")
        sel = lambda t: t.index_select(0, indices)  # noqa: E731
        return KDAState(sel(self.recurrent_state), ShortConvState(sel(self.q_conv_state.buffer)),
                        ShortConvState(sel(self.k_conv_state.buffer)), ShortConvState(sel(self.v_conv_state.buffer)),
                        sel(self.sequence_offset))


@dataclass
class KDAOperatorOutput:
    hidden_states: torch.Tensor
    final_state: torch.Tensor | None = None
    states_per_token: tuple | None = None


@dataclass
class KDAOutput:
    hidden_states: torch.Tensor
    state: KDAState | None = None
    diagnostics: dict | None = None


# --------------------------------------------------------------------------- validation helpers
def validate_attention_mask(mask, batch: int, tokens: int, *, require_nonempty: bool = True):
    if mask is None:
        return None
    if tuple(mask.shape) != (batch, tokens):
        raise ValueError(f"attention_mask must have shape {(batch, tokens)}")
    if mask.dtype != torch.bool:
        raise TypeError("attention_mask must be boolean (True means valid)")
    if not host_checks():  # value checks ran on the host copy of the batch
        return mask
    if tokens > 1 and torch.any((~mask[:, :-1]) & mask[:, 1:]):
        raise ValueError("attention_mask must be monotonic right-padding")
    if require_nonempty and torch.any(mask.sum(dim=1) == 0):
        raise ValueError("all-padding sequences are not supported")
    return mask


def _validate_core(q, k, v, g, beta, initial_state, mask):
    if q.ndim != 4:
        raise ValueError("q must have shape [B,T,H,K]")
    b, t, h, kd = q.shape
    if t == 0:
        raise ValueError("KDA does not support empty sequences")
    if k.shape != q.shape or g.shape != q.shape:
        raise ValueError("k and g must have the same shape as q")
    if v.ndim != 4 or v.shape[:3] != (b, t, h):
        raise ValueError("v must have shape [B,T,H,V] matching q")
    if tuple(beta.shape) != (b, t, h):
        raise ValueError("beta must have shape [B,T,H]")
    if initial_state is not None and tuple(initial_state.shape) != (b, h, kd, v.shape[-1]):
        raise ValueError("initial_state must have shape [B,H,K,V]")
    validate_attention_mask(mask, b, t)
    return b, t, h, kd, v.shape[-1]


def _work_dtype(dtype: torch.dtype, fp32: bool) -> torch.dtype:
    return torch.float32 if fp32 and dtype in (torch.float16, torch.bfloat16) else dtype


def apply_operator_mask(q, g, beta, mask):
    """Padded positions read nothing, decay nothing and write nothing."""
    if mask is None:
        return q, g, beta
    valid = mask[:, :, None]
    return (q * valid[..., None].to(q.dtype), torch.where(valid[..., None], g, torch.zeros_like(g)),
            torch.where(valid, beta, torch.zeros_like(beta)))


# --------------------------------------------------------------------------- reference cores (PyTorch)
def recurrent_kda(q, k, v, g, beta, initial_state=None, output_final_state=False, attention_mask=None, *,
                  accumulate_state_in_fp32=True, return_states_per_token=False) -> KDAOperatorOutput:
    """Exact per-token recurrence: decay, delta-rule write, then read."""
    b, t, h, kd, vd = _validate_core(q, k, v, g, beta, initial_state, attention_mask)
    act = v.dtype
    wd = _work_dtype(act, accumulate_state_in_fp32)
    qw, kw, vw, gw, bw = (x.to(wd) for x in (q, k, v, g, beta))
    qw, gw, bw = apply_operator_mask(qw, gw, bw, attention_mask)
    state = torch.zeros(b, h, kd, vd, dtype=wd, device=q.device)
    if initial_state is not None:
        state = state + initial_state.to(wd)
    outs, hist = [], ([] if return_states_per_token else None)
    for i in range(t):
        state = state * torch.exp(gw[:, i])[..., None]
        err = vw[:, i] - torch.einsum("bhkv,bhk->bhv", state, kw[:, i])
        state = state + torch.einsum("bhk,bhv->bhkv", bw[:, i, :, None] * kw[:, i], err)
        outs.append(torch.einsum("bhkv,bhk->bhv", state, qw[:, i]))
        if hist is not None:
            hist.append(state)
    return KDAOperatorOutput(torch.stack(outs, 1).to(act), state if output_final_state else None,
                             tuple(hist) if hist is not None else None)


def _pairwise_decay_dot(left, right, log_left, log_right, include_diagonal: bool):
    """``sum_k left_i[k] exp(Ll_i[k]-Lr_j[k]) right_j[k]`` for j<=i (or j<i).

    Inputs ``[..., C, K]``; the exponent is only evaluated on the causal triangle,
    so every factor is <= 1 in magnitude.
    """
    c = left.shape[-2]
    diff = log_left[..., :, None, :] - log_right[..., None, :, :]
    keep = torch.ones(c, c, dtype=torch.bool, device=left.device).tril(0 if include_diagonal else -1)
    diff = diff.masked_fill(~keep[..., None], float("-inf"))
    return torch.einsum("...ik,...ijk,...jk->...ij", left, torch.exp(diff), right)


def chunk_ut_transform(k, v, g, beta):
    """UT transform of ``[..., C, K]`` chunks; returns (M, U, W, G, k*e^G)."""
    G = torch.cumsum(g, dim=-2)
    strict = _pairwise_decay_dot(k, k, G, G, include_diagonal=False)
    c = k.shape[-2]
    eye = torch.eye(c, dtype=k.dtype, device=k.device)
    lower = eye + beta[..., None] * strict
    M = torch.linalg.solve_triangular(lower, torch.diag_embed(beta), upper=False, unitriangular=True)
    kg = torch.exp(G) * k
    return M, M @ v, M @ kg, G, kg


def chunkwise_kda(q, k, v, g, beta, initial_state=None, output_final_state=False, attention_mask=None, *,
                  chunk_size=64, secondary_tile_size=16, accumulate_state_in_fp32=True) -> KDAOperatorOutput:
    """Chunked UT/WY KDA; the per-chunk algebra is batched over all chunks and
    only the ``[K,V]`` state recurrence runs sequentially."""
    if chunk_size <= 0 or secondary_tile_size <= 0:
        raise ValueError("invalid chunk_size / secondary_tile_size")
    b, t, h, kd, vd = _validate_core(q, k, v, g, beta, initial_state, attention_mask)
    act = v.dtype
    wd = _work_dtype(act, accumulate_state_in_fp32)
    qw, kw, vw, gw, bw = (x.to(wd) for x in (q, k, v, g, beta))
    qw, gw, bw = apply_operator_mask(qw, gw, bw, attention_mask)
    c = min(chunk_size, t)
    n = (t + c - 1) // c
    pad = n * c - t
    if pad:
        # Zero-padded tail tokens neither decay (g=0) nor write (beta=0) nor read (q=0).
        qw, kw, vw, gw = (F.pad(x, (0, 0, 0, 0, 0, pad)) for x in (qw, kw, vw, gw))
        bw = F.pad(bw, (0, 0, 0, pad))

    def chunked(x):  # [B,T,H,D] -> [B,H,N,C,D]
        return x.reshape(b, n, c, h, -1).permute(0, 3, 1, 2, 4)

    qc, kc, vc, gc = chunked(qw), chunked(kw), chunked(vw), chunked(gw)
    bc = bw.reshape(b, n, c, h).permute(0, 3, 1, 2)
    M, U, W, G, kg = chunk_ut_transform(kc, vc, gc, bc)
    P = _pairwise_decay_dot(qc, kc, G, G, include_diagonal=True)
    qg = torch.exp(G) * qc
    g_end = G[..., -1:, :]  # [B,H,N,1,K]
    k_end = torch.exp(g_end - G) * kc
    state = torch.zeros(b, h, kd, vd, dtype=wd, device=q.device)
    if initial_state is not None:
        state = state + initial_state.to(wd)
    outs = []
    for i in range(n):
        vp = U[:, :, i] - W[:, :, i] @ state
        outs.append(qg[:, :, i] @ state + P[:, :, i] @ vp)
        state = state * torch.exp(g_end[:, :, i, 0])[..., None] + k_end[:, :, i].transpose(-1, -2) @ vp
    o = torch.stack(outs, dim=2).permute(0, 2, 3, 1, 4).reshape(b, n * c, h, vd)[:, :t]
    return KDAOperatorOutput(o.to(act), state if output_final_state else None)


def kda_core(q, k, v, g, beta, initial_state=None, output_final_state=False, attention_mask=None, *,
             chunk_size=64, secondary_tile_size=16, accumulate_state_in_fp32=True) -> KDAOperatorOutput:
    """Dispatch to the sm_100a chunk kernel on CUDA, else the PyTorch chunk form."""
    if _ops.use_kernels(q) and accumulate_state_in_fp32:
        _validate_core(q, k, v, g, beta, initial_state, attention_mask)
        qm, gm, bm = apply_operator_mask(q, g, beta, attention_mask)
        o, fs = _ops.kda_chunk(qm, k, v, gm, bm, initial_state, output_final_state, chunk_size)
        return KDAOperatorOutput(o, fs)
    return chunkwise_kda(q, k, v, g, beta, initial_state, output_final_state, attention_mask,
                         chunk_size=chunk_size, secondary_tile_size=secondary_tile_size,
                         accumulate_state_in_fp32=accumulate_state_in_fp32)


# --------------------------------------------------------------------------- UT transform (public)
@dataclass
class UTTransformOutput:
    M: torch.Tensor
    U: torch.Tensor
    W: torch.Tensor
    log_gamma: torch.Tensor
    k_gamma: torch.Tensor


def ut_transform(k, v, g, beta, secondary_tile_size: int = 16) -> UTTransformOutput:
    """UT transform of canonical ``[B,C,H,*]`` inputs; ``M`` is ``[B,H,C,C]``."""
    M, U, W, G, kg = chunk_ut_transform(k.permute(0, 2, 1, 3), v.permute(0, 2, 1, 3),
                                        g.permute(0, 2, 1, 3), beta.permute(0, 2, 1))
    p = lambda x: x.permute(0, 2, 1, 3)  # noqa: E731
    return UTTransformOutput(M, p(U), p(W), p(G), p(kg))


# --------------------------------------------------------------------------- modules
@dataclass
class KDAProjectionResult:
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    beta: torch.Tensor
    decay_logits: torch.Tensor
    q_conv_state: ShortConvState | None = None
    k_conv_state: ShortConvState | None = None
    v_conv_state: ShortConvState | None = None


class KDAProjections(nn.Module):
    """q/k/v linears -> short causal conv -> SiLU (q,k L2-normalised per head),
    ``beta = sigmoid(W_b x)`` and low-rank decay logits ``alpha_up(alpha_down x) + b_alpha``."""

    def __init__(self, config: KDAConfig):
        super().__init__()
        self.config = c = config
        self.q_proj = Linear(c.d_model, c.key_width, bias=c.projection_bias)
        self.k_proj = Linear(c.d_model, c.key_width, bias=c.projection_bias)
        self.v_proj = Linear(c.d_model, c.value_width, bias=c.projection_bias)
        self.q_conv = CausalShortConv1D(c.key_width, c.short_conv_kernel_size, bias=c.short_conv_bias)
        self.k_conv = CausalShortConv1D(c.key_width, c.short_conv_kernel_size, bias=c.short_conv_bias)
        self.v_conv = CausalShortConv1D(c.value_width, c.short_conv_kernel_size, bias=c.short_conv_bias)
        self.beta_proj = Linear(c.d_model, c.num_heads, bias=c.beta_bias)
        self.alpha_down = Linear(c.d_model, c.resolved_decay_rank, bias=False)
        self.alpha_up = Linear(c.resolved_decay_rank, c.key_width, bias=False)
        self.b_alpha = nn.Parameter(torch.empty(c.num_heads, c.key_head_dim))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        for proj in (self.q_proj, self.k_proj, self.v_proj, self.beta_proj, self.alpha_down, self.alpha_up):
            nn.init.normal_(proj.weight, mean=0.0, std=self.config.init_std)
            if proj.bias is not None:
                nn.init.zeros_(proj.bias)
        if self.config.decay_initializer == "official_fla":
            # log-uniform dt in [1e-3, 1e-1] mapped through the inverse softplus.
            dt = torch.exp(torch.rand_like(self.b_alpha) * (math.log(0.1) - math.log(0.001))
                           + math.log(0.001)).clamp_min(1e-4)
            with torch.no_grad():
                self.b_alpha.copy_(dt + torch.log(-torch.expm1(-dt)))
        else:
            nn.init.zeros_(self.b_alpha)

    def _run_conv(self, module, x, state, mask, return_state):
        if mask is None or bool(mask.all()):
            if return_state:
                return module(x, state, return_state=True)
            return module(x, state), None
        # Right-padded rows: run each valid prefix so padding never enters the history.
        lengths = mask.sum(dim=1).tolist()
        outs, bufs = [], []
        for i, length in enumerate(lengths):
            st = ShortConvState(state.buffer[i:i + 1]) if state is not None else None
            o, nxt = module(x[i:i + 1, :length], st, return_state=True)
            outs.append(F.pad(o, (0, 0, 0, x.shape[1] - length)))
            bufs.append(nxt.buffer)
        return torch.cat(outs, 0), (ShortConvState(torch.cat(bufs, 0)) if return_state else None)

    def forward(self, hidden_states, *, q_conv_state=None, k_conv_state=None, v_conv_state=None,
                attention_mask=None, output_final_state=False, inplace_state=False,
                projected=None) -> KDAProjectionResult:
        """``projected``: the (q, k, v, alpha_down, beta) linear outputs when the caller computed them
        in one fused group GEMM together with the output-gate logits."""
        c = self.config
        if hidden_states.ndim != 3 or hidden_states.shape[-1] != c.d_model:
            raise ValueError(f"hidden_states must have shape [B,T,{c.d_model}]")
        b, t, _ = hidden_states.shape
        if t == 0:
            raise ValueError("KDA projections do not support empty sequences")
        validate_attention_mask(attention_mask, b, t)
        fused = (_ops.use_kernels(hidden_states) and not output_final_state and q_conv_state is None
                 and attention_mask is None and not c.short_conv_bias)
        if projected is not None:
            ql, kl, vl, adown, blog = projected
        else:
            ql, kl, vl = self.q_proj(hidden_states), self.k_proj(hidden_states), self.v_proj(hidden_states)
            adown, blog = self.alpha_down(hidden_states), self.beta_proj(hidden_states)
        beta = torch.sigmoid(blog)
        be = torch.finfo(beta.dtype).eps
        beta = beta.clamp(be, 1.0 - be)
        decay_logits = self.alpha_up(adown).reshape(b, t, c.num_heads, c.key_head_dim)
        decay_logits = decay_logits + self.b_alpha[None, None]
        states = (q_conv_state, k_conv_state, v_conv_state)
        hl = c.key_head_dim // 8
        step = (_ops.use_kernels(hidden_states) and t == 1 and attention_mask is None
                and 1 <= c.short_conv_kernel_size <= 8 and c.key_head_dim % 8 == 0 and 0 < hl <= 32
                and hl & (hl - 1) == 0 and c.value_width % 8 == 0
                and all(st is not None and st.buffer.dtype == ql.dtype
                        and st.buffer.shape[1] == c.short_conv_kernel_size - 1 for st in states))
        if step:
            # One decode token: the three conv streams advance in one launch (history shifted in
            # place -- on copies unless the state belongs to a serving cache).
            hists = [st.buffer if inplace_state else st.buffer.clone() for st in states]
            convs = (self.q_conv, self.k_conv, self.v_conv)
            q, k, v = _ops.conv_silu_norm_step([ql, kl, vl], hists, [m.weight for m in convs], [m.bias for m in convs],
                                               [c.key_head_dim, c.key_head_dim, 0], c.eps)
            return KDAProjectionResult(q.view(b, t, c.num_heads, c.key_head_dim),
                                       k.view(b, t, c.num_heads, c.key_head_dim),
                                       v.view(b, t, c.num_heads, c.value_head_dim), beta, decay_logits,
                                       ShortConvState(hists[0]), ShortConvState(hists[1]), ShortConvState(hists[2]))
        if fused:
            # One kernel per stream: causal conv (zero history) + SiLU (+ per-head L2 norm).
            q = _ops.conv_silu_norm(ql, self.q_conv.weight, c.key_head_dim, c.eps, True)
            k = _ops.conv_silu_norm(kl, self.k_conv.weight, c.key_head_dim, c.eps, True)
            v = _ops.conv_silu_norm(vl, self.v_conv.weight, c.value_head_dim, c.eps, False)
            return KDAProjectionResult(q.view(b, t, c.num_heads, c.key_head_dim),
                                       k.view(b, t, c.num_heads, c.key_head_dim),
                                       v.view(b, t, c.num_heads, c.value_head_dim), beta, decay_logits)
        q, nq = self._run_conv(self.q_conv, ql, q_conv_state, attention_mask, output_final_state)
        k, nk = self._run_conv(self.k_conv, kl, k_conv_state, attention_mask, output_final_state)
        v, nv = self._run_conv(self.v_conv, vl, v_conv_state, attention_mask, output_final_state)
        q = F.normalize(F.silu(q).reshape(b, t, c.num_heads, c.key_head_dim), p=2, dim=-1, eps=c.eps)
        k = F.normalize(F.silu(k).reshape(b, t, c.num_heads, c.key_head_dim), p=2, dim=-1, eps=c.eps)
        v = F.silu(v).reshape(b, t, c.num_heads, c.value_head_dim)
        return KDAProjectionResult(q, k, v, beta, decay_logits, nq, nk, nv)


class LowerBoundedDecay(nn.Module):
    """``g = g_min * sigmoid(exp(A_log) * z)``; returns ``(g, exp g)``."""

    def __init__(self, num_heads: int, g_min: float = -5.0, *, device=None):
        super().__init__()
        if num_heads <= 0 or g_min >= 0:
            raise ValueError("num_heads must be > 0 and g_min negative")
        self.num_heads, self.g_min = num_heads, float(g_min)
        self.A_log = nn.Parameter(torch.zeros(num_heads, dtype=torch.float32, device=device))

    def forward(self, logits: torch.Tensor):
        if logits.ndim != 4 or logits.shape[2] != self.num_heads:
            raise ValueError(f"logits must have shape [B,T,{self.num_heads},K]")
        if _ops.use_kernels(logits):
            g = _ops.kda_decay(logits, self.A_log, self.g_min)
            return g, None
        scale = self.A_log.exp().to(dtype=logits.dtype)[None, None, :, None]
        p = torch.sigmoid(scale * logits)
        e = torch.finfo(p.dtype).eps
        g = self.g_min * p.clamp(e, 1.0 - e)
        return g, torch.exp(g)


class KimiDeltaAttention(nn.Module):
    """Kimi Delta Attention; ``mode`` selects recurrent / chunkwise / decode cores."""

    def __init__(self, config: KDAConfig):
        super().__init__()
        self.config = config
        self.projections = KDAProjections(config)
        self.decay = LowerBoundedDecay(config.num_heads, config.g_min)
        self.output_norm = HeadwiseRMSNorm(config.num_heads, config.value_head_dim, eps=config.eps)
        self.output_gate = FullRankOutputGate(config.d_model, bias=config.output_gate_bias,
                                              output_bias=config.output_bias, init_std=config.init_std, value_width=config.value_width)

    def projection_groups(self):
        """Weights that read the block input and run as one fused GEMM on CUDA: q, k, v, the output
        gate (widths multiples of 64), then the decay down-projection and beta (the ragged last)."""
        p = self.projections
        return [[p.q_proj.weight, p.k_proj.weight, p.v_proj.weight, self.output_gate.gate_proj.weight,
                 p.alpha_down.weight, p.beta_proj.weight]]

    def _validate_state(self, x, state):
        if state is None:
            return
        c, b = self.config, x.shape[0]
        if tuple(state.recurrent_state.shape) != (b, c.num_heads, c.key_head_dim, c.value_head_dim):
            raise ValueError("state recurrent tensor has the wrong shape")
        hist = c.short_conv_kernel_size - 1
        exp = ((b, hist, c.key_width), (b, hist, c.key_width), (b, hist, c.value_width))
        got = tuple(tuple(s.buffer.shape) for s in (state.q_conv_state, state.k_conv_state, state.v_conv_state))
        if got != exp:
            raise ValueError(f"state ShortConv buffers must have shapes {exp}")

    def forward(self, hidden_states, attention_mask=None, state: KDAState | None = None,
                mode: Literal["recurrent", "chunkwise", "decode"] = "chunkwise", output_final_state: bool = False,
                output_diagnostics: bool = False) -> KDAOutput:
        c = self.config
        if hidden_states.ndim != 3 or hidden_states.shape[-1] != c.d_model:
            raise ValueError(f"hidden_states must have shape [B,T,{c.d_model}]")
        b, t, _ = hidden_states.shape
        if t == 0:
            raise ValueError("KDA does not support empty sequences")
        if mode not in ("recurrent", "chunkwise", "decode"):
            raise ValueError(f"unsupported KDA mode {mode!r}")
        if mode == "decode" and t != 1:
            raise ValueError("decode mode requires exactly one token")
        validate_attention_mask(attention_mask, b, t)
        self._validate_state(hidden_states, state)
        return_state = output_final_state or mode == "decode"
        inplace = state is not None and state.inplace and mode == "decode"
        projected = gate_logits = None
        group = self.projection_groups()[0]
        if (_ops.use_kernels(hidden_states) and self.projections.q_proj.bias is None
                and self.projections.beta_proj.bias is None and self.output_gate.gate_proj.bias is None
                and _ops.linear_group_supported(hidden_states, group)):
            ql, kl, vl, gate_logits, adown, blog = _ops.linear_group(hidden_states, group)
            projected = (ql, kl, vl, adown, blog)
        proj = self.projections(hidden_states, q_conv_state=state.q_conv_state if state else None,
                                k_conv_state=state.k_conv_state if state else None,
                                v_conv_state=state.v_conv_state if state else None,
                                attention_mask=attention_mask, output_final_state=return_state,
                                inplace_state=inplace, projected=projected)
        g, alpha = self.decay(proj.decay_logits)
        init = state.recurrent_state if state is not None else None
        kw = dict(initial_state=init, output_final_state=return_state or output_diagnostics,
                  attention_mask=attention_mask, accumulate_state_in_fp32=c.accumulate_state_in_fp32)
        if mode in ("recurrent", "decode"):
            if (mode == "decode" and _ops.use_kernels(hidden_states) and init is not None and attention_mask is None
                    and c.key_head_dim == 64 and c.value_head_dim == 64):
                o, fs = _ops.kda_decode_step(proj.q, proj.k, proj.v, g, proj.beta, init,
                                             out_state=init if inplace else None)
                core = KDAOperatorOutput(o, fs)
            else:
                core = recurrent_kda(proj.q, proj.k, proj.v, g, proj.beta, **kw)
        else:
            core = kda_core(proj.q, proj.k, proj.v, g, proj.beta, chunk_size=c.chunk_size,
                            secondary_tile_size=c.secondary_tile_size, **kw)
        normalized = self.output_norm(core.hidden_states)
        out, gate = self.output_gate(combine_heads(normalized), hidden_states, return_gate=True,
                                     gate_logits=gate_logits)
        if attention_mask is not None:
            out = out * attention_mask[..., None].to(out.dtype)
        nxt = None
        if return_state:
            lengths = (torch.full((b,), t, dtype=torch.long, device=hidden_states.device) if attention_mask is None
                       else attention_mask.sum(dim=1).to(torch.long))
            offset = lengths if state is None else state.sequence_offset.to(hidden_states.device) + lengths
            if inplace:
                offset = state.sequence_offset.copy_(offset)
            nxt = KDAState(core.final_state, proj.q_conv_state, proj.k_conv_state, proj.v_conv_state, offset,
                           inplace=inplace)
        diagnostics = None
        if output_diagnostics:
            from .diagnostics import build_kda_diagnostics
            diagnostics = build_kda_diagnostics(proj.q, proj.k, proj.beta, g, torch.exp(g), core.final_state,
                                                core.hidden_states, out, gate, attention_mask, c.chunk_size,
                                                math.exp(c.g_min))
        return KDAOutput(out, nxt, diagnostics)


__all__ = [
    "KDAConfig", "KDAState", "KDAOutput", "KDAOperatorOutput", "KDAProjectionResult", "KDAProjections",
    "LowerBoundedDecay", "KimiDeltaAttention", "recurrent_kda", "chunkwise_kda", "kda_core", "ut_transform",
    "UTTransformOutput", "chunk_ut_transform", "validate_attention_mask", "apply_operator_mask",
]
