"""Baseline causal Transformer (the reference's ablation / test-fixture control, not Kimi).

Parity: ``src/transformer_modules/{embedding,rope,rope_utils,mha,swiglu,baseline_block,
baseline_transformer}.py`` and ``src/causal_lm.py:26-158`` (reference): token embedding,
rotary position embedding (rotate-half convention, optional partial rotary dims, explicit or
automatic positions), causal multi-head self-attention with a KV cache for decoding, SwiGLU
MLP, pre-norm blocks with RMSNorm, tied LM head. Parameter names match the reference so its
state dicts load unchanged. On CUDA with 64-wide heads and no cache the attention runs on the
framework's flash-attention kernel.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import ops as _ops
from .primitives import RMSNorm


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    d = x.shape[-1]
    if d % 2:
        raise ValueError(f"rotate_half requires an even last dimension, got {d}")
    return torch.cat((-x[..., d // 2:], x[..., : d // 2]), dim=-1)


class RotaryEmbedding(nn.Module):
    """``x [B, T, H, D]`` -> rotated ``x`` (first ``rotary_dim`` channels)."""

    def __init__(self, dim: int, rotary_dim: Optional[int] = None, base: float = 10000.0):
        super().__init__()
        rotary_dim = dim if rotary_dim is None else rotary_dim
        if dim <= 0 or rotary_dim <= 0 or rotary_dim > dim or rotary_dim % 2 or base <= 0:
            raise ValueError("invalid rotary configuration")
        self.dim, self.rotary_dim, self.base = dim, rotary_dim, base
        inv = 1.0 / (base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim))
        self.register_buffer("inv_freq", inv, persistent=False)

    def positions(self, b: int, t: int, device, position_ids=None, start_pos: int = 0) -> torch.Tensor:
        if position_ids is None:
            return torch.arange(start_pos, start_pos + t, device=device, dtype=torch.float32)
        p = position_ids.to(device)
        if p.dim() == 1 and p.shape[0] == t:
            return p.float()
        if p.dim() == 2 and tuple(p.shape) == (b, t):
            return p.float()
        raise ValueError("position_ids must be None, shape [T], or shape [B, T]")

    def forward(self, x: torch.Tensor, position_ids=None, start_pos: int = 0) -> torch.Tensor:
        if x.ndim != 4 or x.shape[-1] != self.dim:
            raise ValueError(f"x must have shape [B,T,H,{self.dim}]")
        b, t = x.shape[:2]
        pos = self.positions(b, t, x.device, position_ids, start_pos)
        freqs = pos[..., None] * self.inv_freq.to(x.device)
        emb = torch.cat((freqs, freqs), dim=-1)
        if emb.dim() == 2:
            emb = emb[None]
        cos, sin = emb.cos()[:, :, None, :].to(x.dtype), emb.sin()[:, :, None, :].to(x.dtype)
        r = self.rotary_dim
        rot = x[..., :r] * cos + rotate_half(x[..., :r]) * sin
        return torch.cat((rot, x[..., r:]), dim=-1) if r < self.dim else rot


@dataclass
class CausalMHAConfig:
    d_model: int
    n_heads: int
    head_dim: Optional[int] = None
    attention_dropout: float = 0.0
    residual_dropout: float = 0.0
    use_bias: bool = False
    use_rope: bool = True
    rope_theta: float = 10000.0
    rotary_dim: Optional[int] = None
    max_seq_len: int = 1024
    init_std: float = 0.02

    def validate(self) -> None:
        if self.d_model <= 0 or self.n_heads <= 0:
            raise ValueError("d_model and n_heads must be positive")
        hd = self.resolved_head_dim
        if hd <= 0 or self.n_heads * hd != self.d_model:
            raise ValueError("For baseline CausalMHA, n_heads * head_dim must equal d_model")
        if not 0.0 <= self.attention_dropout < 1.0 or not 0.0 <= self.residual_dropout < 1.0:
            raise ValueError("dropouts must satisfy 0 <= p < 1")
        if self.max_seq_len <= 0 or self.init_std <= 0 or self.rope_theta <= 0:
            raise ValueError("max_seq_len, init_std and rope_theta must be positive")
        if self.rotary_dim is not None and (self.rotary_dim <= 0 or self.rotary_dim > hd or self.rotary_dim % 2):
            raise ValueError("rotary_dim must be even and <= head_dim")

    @property
    def resolved_head_dim(self) -> int:
        return self.head_dim if self.head_dim is not None else self.d_model // self.n_heads


@dataclass
class KVCache:
    key: torch.Tensor    # [B, T, H, D]
    value: torch.Tensor
    mask: torch.Tensor   # [B, T]

    @property
    def length(self) -> int:
        return int(self.key.shape[1])


class MultiHeadSelfAttention(nn.Module):
    def __init__(self, config: CausalMHAConfig):
        super().__init__()
        config.validate()
        self.config = c = config
        hd = c.resolved_head_dim
        self.q_proj = nn.Linear(c.d_model, c.d_model, bias=c.use_bias)
        self.k_proj = nn.Linear(c.d_model, c.d_model, bias=c.use_bias)
        self.v_proj = nn.Linear(c.d_model, c.d_model, bias=c.use_bias)
        self.out_proj = nn.Linear(c.d_model, c.d_model, bias=c.use_bias)
        for lin in (self.q_proj, self.k_proj, self.v_proj, self.out_proj):
            nn.init.normal_(lin.weight, std=c.init_std)
            if lin.bias is not None:
                nn.init.zeros_(lin.bias)
        self.rope = RotaryEmbedding(hd, c.rotary_dim, c.rope_theta) if c.use_rope else None
        self.dropout = nn.Dropout(c.residual_dropout)

    def forward(self, x, attention_mask=None, position_ids=None, cache: KVCache | None = None, use_cache=False):
        c = self.config
        b, t, _ = x.shape
        hd = c.resolved_head_dim
        q = self.q_proj(x).view(b, t, c.n_heads, hd)
        k = self.k_proj(x).view(b, t, c.n_heads, hd)
        v = self.v_proj(x).view(b, t, c.n_heads, hd)
        start = 0 if cache is None else cache.length
        if self.rope is not None:
            q = self.rope(q, position_ids, start)
            k = self.rope(k, position_ids, start)
        mask_new = torch.ones(b, t, dtype=torch.bool, device=x.device) if attention_mask is None else attention_mask
        if cache is not None:
            k = torch.cat((cache.key, k), 1)
            v = torch.cat((cache.value, v), 1)
            kmask = torch.cat((cache.mask, mask_new), 1)
        else:
            kmask = mask_new
        new_cache = KVCache(k, v, kmask) if use_cache else None
        if (cache is None and attention_mask is None and _ops.use_kernels(x) and hd == 64
                and c.attention_dropout == 0.0):
            o = _ops.flash_attention(q, k, v, causal=True)
        else:
            s = k.shape[1]
            qpos = torch.arange(start, start + t, device=x.device)
            allow = (torch.arange(s, device=x.device)[None, :] <= qpos[:, None])[None, None] & kmask[:, None, None, :]
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               attn_mask=allow, dropout_p=c.attention_dropout if self.training
                                               else 0.0).transpose(1, 2)
        out = self.dropout(self.out_proj(o.reshape(b, t, c.d_model)))
        return (out, new_cache) if use_cache else out


def round_up_to_multiple(value: int, multiple_of: int) -> int:
    return ((value + multiple_of - 1) // multiple_of) * multiple_of


class SwiGLUFeedForward(nn.Module):
    def __init__(self, d_model: int, hidden_dim: int, bias: bool = False, dropout: float = 0.0, init_std: float = 0.02):
        super().__init__()
        self.gate_proj = nn.Linear(d_model, hidden_dim, bias=bias)
        self.up_proj = nn.Linear(d_model, hidden_dim, bias=bias)
        self.down_proj = nn.Linear(hidden_dim, d_model, bias=bias)
        for lin in (self.gate_proj, self.up_proj, self.down_proj):
            nn.init.normal_(lin.weight, std=init_std)
            if lin.bias is not None:
                nn.init.zeros_(lin.bias)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x):
        return self.dropout(self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x)))


@dataclass
class TransformerBlockConfig:
    d_model: int
    rms_norm_eps: float = 1e-6
    n_heads: int = 4
    head_dim: Optional[int] = None
    attention_dropout: float = 0.0
    residual_dropout: float = 0.0
    use_attention_bias: bool = False
    use_rope: bool = True
    rope_theta: float = 10000.0
    rotary_dim: Optional[int] = None
    max_seq_len: int = 1024
    mlp_hidden_dim: Optional[int] = None
    mlp_expansion_factor: float = 4.0
    mlp_multiple_of: int = 1
    mlp_dropout: float = 0.0
    use_mlp_bias: bool = False
    init_std: float = 0.02

    @property
    def resolved_mlp_hidden_dim(self) -> int:
        if self.mlp_hidden_dim is not None:
            return self.mlp_hidden_dim
        return round_up_to_multiple(int(self.d_model * self.mlp_expansion_factor), self.mlp_multiple_of)

    def attention_config(self) -> CausalMHAConfig:
        return CausalMHAConfig(self.d_model, self.n_heads, self.head_dim, self.attention_dropout,
                               self.residual_dropout, self.use_attention_bias, self.use_rope, self.rope_theta,
                               self.rotary_dim, self.max_seq_len, self.init_std)


class BaselineTransformerBlock(nn.Module):
    def __init__(self, config: TransformerBlockConfig):
        super().__init__()
        self.norm1 = RMSNorm(config.d_model, eps=config.rms_norm_eps)
        self.attention = MultiHeadSelfAttention(config.attention_config())
        self.norm2 = RMSNorm(config.d_model, eps=config.rms_norm_eps)
        self.mlp = SwiGLUFeedForward(config.d_model, config.resolved_mlp_hidden_dim, config.use_mlp_bias,
                                     config.mlp_dropout, config.init_std)

    def forward(self, x, attention_mask=None, position_ids=None, cache=None, use_cache=False):
        a = self.attention(self.norm1(x), attention_mask, position_ids, cache, use_cache)
        a, nc = a if use_cache else (a, None)
        x = x + a
        x = x + self.mlp(self.norm2(x))
        return (x, nc) if use_cache else x


class BaselineTransformer(nn.Module):
    def __init__(self, config: TransformerBlockConfig, n_layers: int):
        super().__init__()
        self.layers = nn.ModuleList(BaselineTransformerBlock(config) for _ in range(n_layers))

    def forward(self, x, attention_mask=None, position_ids=None, cache=None, use_cache=False):
        caches = []
        for i, layer in enumerate(self.layers):
            r = layer(x, attention_mask, position_ids, None if cache is None else cache[i], use_cache)
            x, c = r if use_cache else (r, None)
            caches.append(c)
        return (x, tuple(caches)) if use_cache else x


@dataclass
class CausalLMOutput:
    logits: torch.Tensor
    loss: Optional[torch.Tensor] = None
    cache: Optional[tuple] = None


@dataclass
class BaselineCausalLMConfig:
    vocab_size: int
    d_model: int = 128
    n_layers: int = 2
    n_heads: int = 4
    mlp_hidden_dim: Optional[int] = None
    max_seq_len: int = 128
    pad_token_id: Optional[int] = None
    tie_embeddings: bool = True
    use_rope: bool = True
    rope_theta: float = 10_000.0
    dropout: float = 0.0
    rms_norm_eps: float = 1e-6
    init_std: float = 0.02

    def validate(self) -> None:
        if self.vocab_size <= 0 or self.d_model <= 0 or self.n_layers <= 0:
            raise ValueError("vocab_size, d_model, and n_layers must be positive")
        if self.n_heads <= 0 or self.d_model % self.n_heads:
            raise ValueError("n_heads must divide d_model")
        if self.max_seq_len <= 0:
            raise ValueError("max_seq_len must be positive")
        if not 0.0 <= self.dropout < 1.0:
            raise ValueError("dropout must satisfy 0 <= p < 1")

    def block_config(self) -> TransformerBlockConfig:
        return TransformerBlockConfig(self.d_model, self.rms_norm_eps, self.n_heads, None, self.dropout, self.dropout,
                                      False, self.use_rope, self.rope_theta, None, self.max_seq_len,
                                      self.mlp_hidden_dim, init_std=self.init_std)


class TokenEmbedding(nn.Module):
    def __init__(self, vocab_size: int, d_model: int, pad_token_id=None, init_std: float = 0.02):
        super().__init__()
        self.token_embedding = nn.Embedding(vocab_size, d_model, padding_idx=pad_token_id)
        nn.init.normal_(self.token_embedding.weight, std=init_std)
        if pad_token_id is not None:
            with torch.no_grad():
                self.token_embedding.weight[pad_token_id].zero_()

    @property
    def weight(self):
        return self.token_embedding.weight

    def forward(self, ids):
        return self.token_embedding(ids)


class BaselineCausalLM(nn.Module):
    """MHA + RoPE + standard residuals + dense SwiGLU control model."""

    def __init__(self, config: BaselineCausalLMConfig):
        super().__init__()
        config.validate()
        self.config = config
        self.embedding = TokenEmbedding(config.vocab_size, config.d_model, config.pad_token_id, config.init_std)
        self.backbone = BaselineTransformer(config.block_config(), config.n_layers)
        self.final_norm = RMSNorm(config.d_model, eps=config.rms_norm_eps)
        self.lm_head = nn.Linear(config.d_model, config.vocab_size, bias=False)
        nn.init.normal_(self.lm_head.weight, std=config.init_std)
        if config.tie_embeddings:
            self.lm_head.weight = self.embedding.weight

    def forward_embeddings(self, hidden, *, labels=None, attention_mask=None, position_ids=None, cache=None,
                           use_cache=False) -> CausalLMOutput:
        b, t, _ = hidden.shape
        if t > self.config.max_seq_len and cache is None:
            raise ValueError("sequence exceeds max_seq_len")
        r = self.backbone(hidden, attention_mask, position_ids, cache, use_cache)
        hidden, new_cache = r if use_cache else (r, None)
        logits = self.lm_head(self.final_norm(hidden))
        loss = None
        if labels is not None:
            loss = F.cross_entropy(logits.reshape(-1, self.config.vocab_size).float(), labels.reshape(-1),
                                   ignore_index=self.config.pad_token_id if self.config.pad_token_id is not None
                                   else -100)
        return CausalLMOutput(logits, loss, new_cache)

    def forward(self, input_ids, labels=None, attention_mask=None, position_ids=None, cache=None, use_cache=False):
        if input_ids.ndim != 2:
            raise ValueError("input_ids must have shape [B,T]")
        if attention_mask is None and self.config.pad_token_id is not None and cache is None:
            attention_mask = input_ids.ne(self.config.pad_token_id)
        return self.forward_embeddings(self.embedding(input_ids), labels=labels, attention_mask=attention_mask,
                                       position_ids=position_ids, cache=cache, use_cache=use_cache)

    def num_parameters(self, trainable_only: bool = False) -> int:
        return sum(p.numel() for p in self.parameters() if p.requires_grad or not trainable_only)


__all__ = ["rotate_half", "RotaryEmbedding", "CausalMHAConfig", "KVCache", "MultiHeadSelfAttention",
           "SwiGLUFeedForward", "TransformerBlockConfig", "BaselineTransformerBlock", "BaselineTransformer",
           "TokenEmbedding", "BaselineCausalLMConfig", "BaselineCausalLM", "CausalLMOutput", "round_up_to_multiple"]
