"""Gated Multi-head Latent Attention (NoPE) with a compressed latent KV cache.

Parity targets (reference paths):
  * ``src/mla/config.py:10-97``       GatedMLAConfig
  * ``src/mla/latent_kv.py:22-79``    compression / key_up / value_up
  * ``src/mla/projections.py:24-55``  MLAProjections
  * ``src/mla/attention.py:35-195``   masked causal attention (manual and SDPA forms)
  * ``src/mla/gated_mla.py:32-183``   GatedMLA (QK-Clip proxy, sigmoid gate, out-proj)
  * ``src/mla/cache.py:12-163``       MLACache (latent-only cache, right padding)

Differences by design:
  * full-sequence training on CUDA runs the sm_100a causal flash-attention kernel
    (per-row key lengths instead of a materialised ``[B,Tq,Tk]`` mask);
  * the reference re-expands K/V from the whole latent cache every decode step;
    :func:`absorbed_latent_decode` folds ``W_uk`` into the query and ``W_uv`` into
    the output so decode reads only the ``[T,L]`` latent cache.
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
from .primitives import FullRankOutputGate, combine_heads


@dataclass(frozen=True)
class GatedMLAConfig:
    d_model: int
    num_heads: int
    q_head_dim: int
    v_head_dim: int
    kv_latent_dim: int
    attention_dropout: float = 0.0
    output_dropout: float = 0.0
    projection_bias: bool = False
    output_gate_bias: bool = False
    output_bias: bool = False
    use_nope: bool = True
    keep_attention_output_fp32: bool = True
    use_sdpa: bool = True
    attention_backend: Literal["auto", "manual", "sdpa"] = "auto"
    init_std: float = 0.02

    def __post_init__(self) -> None:
        for name in ("d_model", "num_heads", "q_head_dim", "v_head_dim", "kv_latent_dim"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be > 0")
        if self.d_model != self.num_heads * self.v_head_dim:
            raise ValueError("d_model must equal num_heads * v_head_dim")
        if self.kv_latent_dim > self.full_kv_width:
            raise ValueError("kv_latent_dim must not exceed the uncompressed per-token KV width")
        for name in ("attention_dropout", "output_dropout"):
            if not 0.0 <= getattr(self, name) < 1.0:
                raise ValueError(f"{name} must satisfy 0 <= p < 1")
        if not self.use_nope:
            raise ValueError("Kimi K3 Gated MLA requires use_nope=True")
        if self.attention_backend not in ("auto", "manual", "sdpa"):
            raise ValueError("attention_backend must be 'auto', 'manual', or 'sdpa'")
        if self.attention_backend == "sdpa" and not self.use_sdpa:
            raise ValueError("attention_backend='sdpa' is incompatible with use_sdpa=False")
        if self.init_std <= 0:
            raise ValueError("init_std must be > 0")

    @property
    def query_width(self) -> int:
        return self.num_heads * self.q_head_dim

    @property
    def value_width(self) -> int:
        return self.num_heads * self.v_head_dim

    @property
    def full_kv_width(self) -> int:
        return self.num_heads * (self.q_head_dim + self.v_head_dim)

    @property
    def cache_compression_ratio(self) -> float:
        return self.full_kv_width / self.kv_latent_dim

    @property
    def resolved_backend(self) -> str:
        if self.attention_backend == "auto":
            return "sdpa" if self.use_sdpa else "manual"
        return self.attention_backend

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "GatedMLAConfig":
        return cls(**values)


# --------------------------------------------------------------------------- cache
@dataclass
class MLACache:
    """Latent-only KV cache ``[B,T,L]`` with a right-padding mask and offsets."""

    latent_kv: torch.Tensor
    attention_mask: torch.Tensor | None
    sequence_offset: torch.Tensor

    def __post_init__(self) -> None:
        if self.latent_kv.ndim != 3:
            raise ValueError("latent_kv must have shape [B,T,L]")
        b, t, _ = self.latent_kv.shape
        if self.attention_mask is not None:
            if tuple(self.attention_mask.shape) != (b, t) or self.attention_mask.dtype != torch.bool:
                raise ValueError("cache attention_mask must be boolean [B,T]")
        if tuple(self.sequence_offset.shape) != (b,) or self.sequence_offset.dtype != torch.long:
            raise ValueError("sequence_offset must be a torch.long [B] tensor")

    @classmethod
    def empty(cls, batch_size: int, latent_dim: int, *, device=None, dtype=None) -> "MLACache":
        if batch_size <= 0 or latent_dim <= 0:
            raise ValueError("batch_size and latent_dim must be > 0")
        return cls(torch.empty(batch_size, 0, latent_dim, device=device, dtype=dtype),
                   torch.empty(batch_size, 0, device=device, dtype=torch.bool),
                   torch.zeros(batch_size, device=device, dtype=torch.long))

    @property
    def cache_length(self) -> int:
        return self.latent_kv.shape[1]

    @property
    def cache_elements(self) -> int:
        return self.latent_kv.numel()

    def clone(self) -> "MLACache":
        return MLACache(self.latent_kv.clone(), None if self.attention_mask is None else self.attention_mask.clone(),
                        self.sequence_offset.clone())

    def reorder(self, indices: torch.Tensor) -> "MLACache":
        if indices.ndim != 1 or indices.dtype != torch.long:
            raise ValueError("indices must be a rank-1 torch.long tensor")
        return MLACache(self.latent_kv.index_select(0, indices),
                        None if self.attention_mask is None else self.attention_mask.index_select(0, indices),
                        self.sequence_offset.index_select(0, indices))

    def append(self, latent_kv: torch.Tensor, attention_mask: torch.Tensor | None = None) -> "MLACache":
        """Return a new cache with each row's valid new tokens packed after its valid old ones.

        Vectorised repack: destination slot of a valid token = (#valid tokens before it
        in its row), computed with a cumulative sum; no per-row Python loop.
        """
        if latent_kv.ndim != 3:
            raise ValueError("new latent_kv must have shape [B,T,L]")
        b, t, l = latent_kv.shape
        if b != self.latent_kv.shape[0] or l != self.latent_kv.shape[2]:
            raise ValueError("new latent_kv batch and latent dim must match cache")
        if latent_kv.dtype != self.latent_kv.dtype:
            raise TypeError("new latent_kv and cache must share dtype")
        dev = latent_kv.device
        if dev != self.latent_kv.device:
            raise ValueError("new latent_kv and cache must share device")
        new_mask = torch.ones(b, t, dtype=torch.bool, device=dev) if attention_mask is None else attention_mask
        if tuple(new_mask.shape) != (b, t) or new_mask.dtype != torch.bool:
            raise ValueError("new attention_mask must be boolean with shape [B,T]")
        old_mask = (torch.ones(b, self.cache_length, dtype=torch.bool, device=dev)
                    if self.attention_mask is None else self.attention_mask)
        values = torch.cat((self.latent_kv, latent_kv), dim=1)
        mask = torch.cat((old_mask, new_mask), dim=1)
        lengths = mask.sum(dim=1).to(torch.long)
        if mask.all():
            return MLACache(values, mask, lengths)
        max_len = int(lengths.max().item()) if b else 0
        slot = torch.cumsum(mask.to(torch.long), dim=1) - 1
        packed = values.new_zeros(b, max_len, l)
        rows = torch.arange(b, device=dev)[:, None].expand_as(slot)
        packed[rows[mask], slot[mask]] = values[mask]
        packed_mask = torch.arange(max_len, device=dev)[None, :] < lengths[:, None]
        return MLACache(packed, packed_mask, lengths)


class StaticMLACache(MLACache):
    """A serving cache: a preallocated latent buffer ``[B, Tmax, L]`` whose valid rows are the
    prefix ``[0, sequence_offset[b])``.  :meth:`append` writes one decode token per row in place
    (no reallocation, no host synchronisation), so a decode step can be captured in a CUDA graph
    and replayed; rows that reach ``Tmax`` keep overwriting their last slot.  Built from a
    prefill cache with :meth:`from_cache`."""

    def __init__(self, latent_kv: torch.Tensor, sequence_offset: torch.Tensor):
        super().__init__(latent_kv, None, sequence_offset)

    @classmethod
    def from_cache(cls, cache: MLACache, max_length: int) -> "StaticMLACache":
        b, t, l = cache.latent_kv.shape
        if max_length < t:
            raise ValueError(f"max_length {max_length} is shorter than the prefilled cache ({t})")
        buf = cache.latent_kv.new_zeros(b, max_length, l)
        buf[:, :t] = cache.latent_kv
        if cache.attention_mask is not None:
            buf[:, :t] *= cache.attention_mask[..., None].to(buf.dtype)
        return cls(buf, cache.sequence_offset.clone())

    @property
    def valid_lengths(self) -> torch.Tensor:
        return self.sequence_offset

    def valid_mask(self) -> torch.Tensor:
        return torch.arange(self.latent_kv.shape[1], device=self.latent_kv.device)[None, :] < self.sequence_offset[:, None]

    def clone(self) -> "StaticMLACache":
        return StaticMLACache(self.latent_kv.clone(), self.sequence_offset.clone())

    def reorder(self, indices: torch.Tensor) -> "StaticMLACache":
        return StaticMLACache(self.latent_kv.index_select(0, indices), self.sequence_offset.index_select(0, indices))

    def append(self, latent_kv: torch.Tensor, attention_mask: torch.Tensor | None = None) -> "StaticMLACache":
        b, t, l = latent_kv.shape
        if t != 1 or attention_mask is not None and attention_mask.shape != (b, 1):
            raise ValueError("a static MLA cache appends exactly one token per row")
        if latent_kv.dtype != self.latent_kv.dtype:
            latent_kv = latent_kv.to(self.latent_kv.dtype)
        slot = self.sequence_offset.clamp(max=self.latent_kv.shape[1] - 1)
        rows = torch.arange(b, device=latent_kv.device)
        self.latent_kv.index_put_((rows, slot), latent_kv[:, 0])
        step = 1 if attention_mask is None else attention_mask[:, 0].to(torch.long)
        self.sequence_offset.add_(step)
        return self


# --------------------------------------------------------------------------- projections
@dataclass
class LatentKVOutput:
    latent_kv: torch.Tensor
    key: torch.Tensor
    value: torch.Tensor


class LatentKVProjection(nn.Module):
    """Compress once to ``L`` and reconstruct K and V from the latent."""

    def __init__(self, config: GatedMLAConfig):
        super().__init__()
        self.config = c = config
        self.compression = Linear(c.d_model, c.kv_latent_dim, bias=c.projection_bias)
        self.key_up = Linear(c.kv_latent_dim, c.query_width, bias=c.projection_bias)
        self.value_up = Linear(c.kv_latent_dim, c.value_width, bias=c.projection_bias)
        for proj in (self.compression, self.key_up, self.value_up):
            nn.init.normal_(proj.weight, mean=0.0, std=c.init_std)
            if proj.bias is not None:
                nn.init.zeros_(proj.bias)

    def compress(self, hidden_states):
        return self.compression(hidden_states)

    def reconstruct(self, latent_kv):
        c = self.config
        if latent_kv.ndim != 3 or latent_kv.shape[-1] != c.kv_latent_dim:
            raise ValueError(f"latent_kv must have shape [B,T,{c.kv_latent_dim}]")
        b, t, _ = latent_kv.shape
        pair = [self.key_up.weight, self.value_up.weight]
        if (_ops.use_kernels(latent_kv) and self.key_up.bias is None and self.value_up.bias is None
                and _ops.linear_group_supported(latent_kv, pair)):
            key, value = _ops.linear_group(latent_kv, pair)  # K and V from one read of the latent
        else:
            key, value = self.key_up(latent_kv), self.value_up(latent_kv)
        return key.reshape(b, t, c.num_heads, c.q_head_dim), value.reshape(b, t, c.num_heads, c.v_head_dim)

    def forward(self, hidden_states) -> LatentKVOutput:
        latent = self.compress(hidden_states)
        return LatentKVOutput(latent, *self.reconstruct(latent))


@dataclass
class MLAProjectionOutput:
    query: torch.Tensor
    latent_kv: torch.Tensor
    key: torch.Tensor
    value: torch.Tensor


class MLAProjections(nn.Module):
    def __init__(self, config: GatedMLAConfig):
        super().__init__()
        self.config = config
        self.query = Linear(config.d_model, config.query_width, bias=config.projection_bias)
        self.latent_kv = LatentKVProjection(config)
        nn.init.normal_(self.query.weight, mean=0.0, std=config.init_std)
        if self.query.bias is not None:
            nn.init.zeros_(self.query.bias)

    def project_queries(self, hidden_states):
        b, t, _ = hidden_states.shape
        return self.query(hidden_states).reshape(b, t, self.config.num_heads, self.config.q_head_dim)

    def compress_kv(self, hidden_states):
        return self.latent_kv.compress(hidden_states)

    def reconstruct_kv(self, latent_kv):
        return self.latent_kv.reconstruct(latent_kv)

    def forward(self, hidden_states) -> MLAProjectionOutput:
        q = self.project_queries(hidden_states)
        lat = self.compress_kv(hidden_states)
        return MLAProjectionOutput(q, lat, *self.reconstruct_kv(lat))


# --------------------------------------------------------------------------- attention math
def _acc_dtype(dtype, fp32: bool):
    return torch.float32 if fp32 and dtype in (torch.float16, torch.bfloat16) else dtype


def _allowed_mask(q, key_tokens, attention_mask, query_mask, is_causal, query_positions):
    b, tq = q.shape[:2]
    key_valid = (torch.ones(b, key_tokens, dtype=torch.bool, device=q.device) if attention_mask is None
                 else attention_mask)
    query_valid = torch.ones(b, tq, dtype=torch.bool, device=q.device) if query_mask is None else query_mask
    allowed = key_valid[:, None, :].expand(b, tq, key_tokens)
    if is_causal:
        if query_positions is None:
            query_positions = (torch.arange(tq, device=q.device) + key_tokens - tq)[None, :].expand(b, -1)
        allowed = allowed & (torch.arange(key_tokens, device=q.device)[None, None, :] <= query_positions[:, :, None])
    return allowed & query_valid[:, :, None]


def manual_causal_attention(q, k, v, attention_mask=None, is_causal=True, dropout_p=0.0, keep_output_fp32=True, *,
                            query_mask=None, query_positions=None, training=False, return_attentions=False):
    """Reference-precision masked attention (softmax in fp32 when upcasting)."""
    allowed = _allowed_mask(q, k.shape[1], attention_mask, query_mask, is_causal, query_positions)
    cd = _acc_dtype(q.dtype, keep_output_fp32)
    qq, kk, vv = (x.transpose(1, 2).to(cd) for x in (q, k, v))
    scores = (qq @ kk.transpose(-2, -1)) / math.sqrt(q.shape[-1])
    ea = allowed[:, None]
    scores = scores.masked_fill(~ea, -torch.inf)
    valid_rows = ea.any(dim=-1, keepdim=True)
    probs = torch.softmax(torch.where(valid_rows, scores, torch.zeros_like(scores)), dim=-1)
    probs = torch.where(ea, probs, torch.zeros_like(probs))
    probs = F.dropout(probs, p=dropout_p, training=training)
    out = (probs @ vv).transpose(1, 2)
    if not keep_output_fp32 and out.dtype != q.dtype:
        out = out.to(q.dtype)
    return (out, probs) if return_attentions else out


def mla_attention(q, k, v, attention_mask=None, is_causal=True, dropout_p=0.0, keep_output_fp32=True, *,
                  backend="sdpa", query_mask=None, query_positions=None, training=False, return_attentions=False):
    """Masked causal attention over ``[B,T,H,D]`` tensors (reference semantics)."""
    if backend not in ("manual", "sdpa"):
        raise ValueError("backend must be 'manual' or 'sdpa'")
    if backend == "manual" or return_attentions:
        return manual_causal_attention(q, k, v, attention_mask, is_causal, dropout_p, keep_output_fp32,
                                       query_mask=query_mask, query_positions=query_positions, training=training,
                                       return_attentions=return_attentions)
    allowed = _allowed_mask(q, k.shape[1], attention_mask, query_mask, is_causal, query_positions)
    cd = _acc_dtype(q.dtype, keep_output_fp32)
    qq, kk, vv = (x.transpose(1, 2).to(cd) for x in (q, k, v))
    out = F.scaled_dot_product_attention(qq, kk, vv, attn_mask=allowed[:, None],
                                         dropout_p=dropout_p if training else 0.0, is_causal=False).transpose(1, 2)
    out = torch.where(allowed.any(dim=-1)[:, :, None, None], out, torch.zeros_like(out))
    if not keep_output_fp32 and out.dtype != q.dtype:
        out = out.to(q.dtype)
    return out


def absorbed_latent_decode(query, latent_cache, cache_mask, key_up_weight, value_up_weight, num_heads, *,
                           lengths=None):
    """One-token decode attending over the latent cache directly.

    ``score_t = q_h . (W_uk,h c_t) = (W_uk,h^T q_h) . c_t`` and
    ``o_h = W_uv,h (sum_t p_t c_t)``; K/V are never materialised.
    query ``[B,1,H,Dq]``, latent_cache ``[B,T,L]`` -> ``[B,1,H,Dv]`` (fp32).  ``lengths`` [B]
    (valid prefix per row) replaces ``cache_mask`` for a preallocated cache.
    """
    b, _, h, dq = query.shape
    l = latent_cache.shape[-1]
    if _ops.use_kernels(query):
        return _ops.mla_absorbed_decode(query, latent_cache, cache_mask, key_up_weight, value_up_weight,
                                        lengths=lengths)
    if lengths is not None:
        cache_mask = torch.arange(latent_cache.shape[1], device=query.device)[None, :] < lengths[:, None]
    wd = torch.promote_types(query.dtype, torch.float32)
    wuk = key_up_weight.to(wd).reshape(h, dq, l)
    wuv = value_up_weight.to(wd).reshape(h, -1, l)
    q_lat = torch.einsum("bhd,hdl->bhl", query[:, 0].to(wd), wuk) / math.sqrt(dq)
    scores = torch.einsum("bhl,btl->bht", q_lat, latent_cache.to(wd))
    if cache_mask is not None:
        scores = scores.masked_fill(~cache_mask[:, None, :], -torch.inf)
    p = torch.softmax(scores, dim=-1)
    ctx = torch.einsum("bht,btl->bhl", p, latent_cache.to(wd))
    return torch.einsum("bhl,hvl->bhv", ctx, wuv)[:, None]


# --------------------------------------------------------------------------- module
@dataclass
class GatedMLAOutput:
    hidden_states: torch.Tensor
    cache: MLACache | None = None
    attentions: torch.Tensor | None = None
    diagnostics: dict | None = None


def validate_right_padding_mask(mask, batch, tokens, *, require_nonempty=True):
    from .kda import validate_attention_mask
    return validate_attention_mask(mask, batch, tokens, require_nonempty=require_nonempty)


class GatedMLA(nn.Module):
    """Global NoPE attention over a latent KV with a full-rank sigmoid output gate."""

    def __init__(self, config: GatedMLAConfig):
        super().__init__()
        self.config = config
        self.projections = MLAProjections(config)
        self.output_gate = FullRankOutputGate(config.d_model, bias=config.output_gate_bias,
                                              output_bias=config.output_bias, init_std=config.init_std, value_width=config.value_width)
        self.output_dropout = nn.Dropout(config.output_dropout)
        self.absorbed_decode = True

    def projection_groups(self):
        """Weights that run as one fused GEMM each on CUDA: those reading the block input (query,
        latent compression, output gate) and those reading the latent (key and value
        reconstruction)."""
        p = self.projections
        return [[p.query.weight, p.latent_kv.compression.weight, self.output_gate.gate_proj.weight],
                [p.latent_kv.key_up.weight, p.latent_kv.value_up.weight]]

    def _postprocess(self, attention_output, hidden_states, gate_logits=None):
        combined = combine_heads(attention_output)
        logits = self.output_gate.gate_proj(hidden_states) if gate_logits is None else gate_logits
        gp = self.output_gate.output_proj
        if _ops.use_kernels(combined) and gp.bias is None:
            gated = _ops.sigmoid_mul(logits, combined.to(hidden_states.dtype))
            out = self.output_dropout(gp(gated))
            return out.to(hidden_states.dtype), None
        gate = torch.sigmoid(logits)
        cd = combined.dtype
        if not isinstance(gp, nn.Linear):  # a tensor-parallel projection that also reduces its output
            out = gp(combined * gate.to(cd))
        else:
            out = F.linear(combined * gate.to(cd), gp.weight.to(cd), None if gp.bias is None else gp.bias.to(cd))
        return self.output_dropout(out).to(hidden_states.dtype), gate

    def _record_qk_scale(self, query, key):
        with torch.no_grad():
            self._last_qk_scale = (query.detach().float().square().mean().sqrt()
                                   * key.detach().float().square().mean().sqrt() * math.sqrt(self.config.q_head_dim))

    def forward(self, hidden_states, attention_mask=None, cache: MLACache | None = None, use_cache=False,
                output_attentions=False, output_diagnostics=False, *, position_ids=None) -> GatedMLAOutput:
        c = self.config
        if position_ids is not None:
            raise ValueError("position_ids are unsupported: Kimi Gated MLA is NoPE")
        if hidden_states.ndim != 3 or hidden_states.shape[-1] != c.d_model or hidden_states.shape[1] == 0:
            raise ValueError(f"hidden_states must have shape [B,T,{c.d_model}] with T > 0")
        b, t = hidden_states.shape[:2]
        validate_right_padding_mask(attention_mask, b, t)
        dev = hidden_states.device
        gate_logits = None
        group = self.projection_groups()[0]
        if (_ops.use_kernels(hidden_states) and not c.projection_bias and self.output_gate.gate_proj.bias is None
                and _ops.linear_group_supported(hidden_states, group)):
            q_flat, latent, gate_logits = _ops.linear_group(hidden_states, group)
            query = q_flat.reshape(b, t, c.num_heads, c.q_head_dim)
        else:
            query = self.projections.project_queries(hidden_states)
            latent = self.projections.compress_kv(hidden_states)
        need_probs = output_attentions or output_diagnostics
        fast_full = (cache is None and not use_cache and not need_probs and attention_mask is None
                     and _ops.use_kernels(hidden_states) and c.attention_dropout == 0.0)
        fast_decode = (cache is not None and t == 1 and attention_mask is None and not need_probs
                       and self.absorbed_decode and c.projection_bias is False)
        if fast_full:
            key, value = self.projections.reconstruct_kv(latent)
            self._record_qk_scale(query, key)
            raw = _ops.flash_attention(query, key, value, causal=True)
            out, gate = self._postprocess(raw, hidden_states, gate_logits)
            return GatedMLAOutput(out, None, None, None)
        if cache is None and not use_cache and not need_probs and attention_mask is None and not output_diagnostics:
            # Full causal sequence without padding and without a cache to build: no mask at all.
            key, value = self.projections.reconstruct_kv(latent)
            self._record_qk_scale(query, key)
            raw = mla_attention(query, key, value, None, is_causal=True, dropout_p=c.attention_dropout,
                                keep_output_fp32=c.keep_attention_output_fp32, backend=c.resolved_backend,
                                training=self.training)
            out, gate = self._postprocess(raw, hidden_states, gate_logits)
            return GatedMLAOutput(out, None, None, None)
        current_mask = torch.ones(b, t, dtype=torch.bool, device=dev) if attention_mask is None else attention_mask
        prev = torch.zeros(b, dtype=torch.long, device=dev) if cache is None else cache.sequence_offset
        # The cache stores latents in the dtype the compression produces (bf16 under autocast).
        base = (MLACache.empty(b, c.kv_latent_dim, device=dev, dtype=latent.dtype) if cache is None else cache)
        if cache is not None:
            if cache.latent_kv.shape[-1] != c.kv_latent_dim:
                raise ValueError("cache latent dimension does not match config")
            if cache.latent_kv.dtype != latent.dtype:
                latent = latent.to(cache.latent_kv.dtype)
        updated = base.append(latent, current_mask)
        if fast_decode:
            # Weight-absorbed decode: attend over the latent cache; K/V never rebuilt.
            raw = absorbed_latent_decode(query, updated.latent_kv, updated.attention_mask,
                                         self.projections.latent_kv.key_up.weight,
                                         self.projections.latent_kv.value_up.weight, c.num_heads,
                                         lengths=getattr(updated, "valid_lengths", None))
            if not c.keep_attention_output_fp32:
                raw = raw.to(hidden_states.dtype)
            out, gate = self._postprocess(raw, hidden_states, gate_logits)
            return GatedMLAOutput(out, updated if use_cache else None, None, None)
        key, value = self.projections.reconstruct_kv(updated.latent_kv)
        self._record_qk_scale(query, key)
        qpos = prev[:, None] + torch.arange(t, device=dev)[None, :]
        cache_mask = updated.valid_mask() if isinstance(updated, StaticMLACache) else updated.attention_mask
        result = mla_attention(query, key, value, cache_mask, is_causal=True,
                               dropout_p=c.attention_dropout, keep_output_fp32=c.keep_attention_output_fp32,
                               backend=c.resolved_backend, query_mask=current_mask, query_positions=qpos,
                               training=self.training, return_attentions=need_probs)
        raw, probs = (result if need_probs else (result, None))
        out, gate = self._postprocess(raw, hidden_states, gate_logits)
        out = out * current_mask[..., None].to(out.dtype)
        diagnostics = None
        if output_diagnostics:
            from .diagnostics import build_mla_diagnostics
            if gate is None:
                gate = self.output_gate.gate_values(hidden_states)
            diagnostics = build_mla_diagnostics(query, key, value, updated.latent_kv, gate, probs,
                                                cache_mask, current_mask, updated.cache_elements,
                                                c.full_kv_width, raw, out, self._last_qk_scale)
        return GatedMLAOutput(out, updated if use_cache else None, probs if output_attentions else None, diagnostics)


__all__ = [
    "GatedMLAConfig", "MLACache", "StaticMLACache", "LatentKVProjection", "LatentKVOutput", "MLAProjections", "MLAProjectionOutput",
    "manual_causal_attention", "mla_attention", "absorbed_latent_decode", "GatedMLA", "GatedMLAOutput",
]
