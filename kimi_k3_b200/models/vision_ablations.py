"""Hierarchical (strided depthwise pooling) and Swin (shifted windows) vision encoders.

Parity targets (reference paths):
  * ``src/vision/hierarchical_encoder.py:23-233`` HierarchicalTokenPool, HierarchicalVisionConfig,
    HierarchicalMoonViTEncoder
  * ``src/vision/swin_encoder.py:66-468`` WindowSelfAttention (relative position bias),
    SwinTransformerBlock (shifted windows with region masks), SwinPatchMerging, SwinMoonViTEncoder

These are ablation encoders; they share parameter names with the reference so
checkpoints transfer.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .vision import (DropPath, LearnedAbsolutePositionEmbedding, VisionEncoderOutput, VisionMLP,
                     VisionPatchEmbedding, VisionTransformerBlock, build_vision_norm, initialize_vision_module,
                     to_2tuple, validate_token_grid)


def _check_stages(cfg):
    image, patch = to_2tuple(cfg.image_size, "image_size"), to_2tuple(cfg.patch_size, "patch_size")
    if image[0] % patch[0] or image[1] % patch[1]:
        raise ValueError("configured image_size must be divisible by patch_size")
    n = len(cfg.embed_dims)
    if n == 0 or len(cfg.depths) != n or len(cfg.num_heads) != n:
        raise ValueError("embed_dims, depths, and num_heads must have equal nonzero length")
    if cfg.in_channels <= 0 or any(v <= 0 for v in tuple(cfg.embed_dims) + tuple(cfg.depths) + tuple(cfg.num_heads)):
        raise ValueError("all stage values must be > 0")
    if any(d % h for d, h in zip(cfg.embed_dims, cfg.num_heads)):
        raise ValueError("every embed_dim must be divisible by its num_heads")
    for name in ("dropout", "attention_dropout", "drop_path_rate"):
        if not 0 <= getattr(cfg, name) < 1:
            raise ValueError(f"{name} must be in [0, 1)")


# --------------------------------------------------------------------------- hierarchical
class HierarchicalTokenPool(nn.Module):
    """Stride-2 3x3 depthwise conv, 1x1 projection, norm; the mask is max-pooled."""

    def __init__(self, input_dim, output_dim, *, norm_type="rmsnorm", norm_eps=1e-6, bias=False):
        super().__init__()
        self.input_dim = input_dim
        self.depthwise = nn.Conv2d(input_dim, input_dim, 3, stride=2, padding=1, groups=input_dim, bias=bias)
        self.projection = nn.Conv2d(input_dim, output_dim, 1, bias=bias)
        self.norm = build_vision_norm(norm_type, output_dim, norm_eps)

    def forward(self, tokens, grid_size, padding_mask=None):
        b, h, w = validate_token_grid(tokens, grid_size, self.input_dim)
        f = self.projection(self.depthwise(tokens.reshape(b, h, w, self.input_dim).permute(0, 3, 1, 2)))
        grid = (f.shape[-2], f.shape[-1])
        out = self.norm(f.flatten(2).transpose(1, 2))
        nm = None
        if padding_mask is not None:
            nm = F.max_pool2d(padding_mask.reshape(b, 1, h, w).float(), 3, stride=2, padding=1).flatten(1).bool()
        return out, grid, nm


@dataclass(frozen=True)
class HierarchicalVisionConfig:
    image_size: int | tuple = 224
    patch_size: int | tuple = 14
    in_channels: int = 3
    embed_dims: tuple = (96, 192, 384)
    depths: tuple = (2, 2, 4)
    num_heads: tuple = (6, 12, 12)
    mlp_ratio: float = 4.0
    norm_type: str = "rmsnorm"
    norm_eps: float = 1e-6
    position_embedding_type: str = "learned_absolute"
    patch_bias: bool = False
    qkv_bias: bool = False
    proj_bias: bool = False
    mlp_bias: bool = False
    pool_bias: bool = False
    dropout: float = 0.0
    attention_dropout: float = 0.0
    drop_path_rate: float = 0.0
    initializer_std: float = 0.02

    def __post_init__(self):
        _check_stages(self)
        if self.mlp_ratio <= 0:
            raise ValueError("mlp_ratio must be > 0")
        if self.position_embedding_type not in ("none", "learned_absolute"):
            raise ValueError("unsupported position_embedding_type")


class HierarchicalMoonViTEncoder(nn.Module):
    def __init__(self, config: HierarchicalVisionConfig):
        super().__init__()
        self.config = c = config
        image, patch = to_2tuple(c.image_size, "image_size"), to_2tuple(c.patch_size, "patch_size")
        self.patch_embedding = VisionPatchEmbedding(c.in_channels, c.embed_dims[0], patch, bias=c.patch_bias)
        grids, cur = [], (image[0] // patch[0], image[1] // patch[1])
        for i in range(len(c.embed_dims)):
            grids.append(cur)
            if i < len(c.embed_dims) - 1:
                cur = ((cur[0] + 1) // 2, (cur[1] + 1) // 2)
        self.position_embeddings = (nn.ModuleList(LearnedAbsolutePositionEmbedding(g, d) for g, d in
                                                  zip(grids, c.embed_dims))
                                    if c.position_embedding_type == "learned_absolute" else nn.ModuleList())
        rates = torch.linspace(0, c.drop_path_rate, sum(c.depths)).tolist()
        cursor, self.stages = 0, nn.ModuleList()
        for d, depth, heads in zip(c.embed_dims, c.depths, c.num_heads):
            self.stages.append(nn.ModuleList(VisionTransformerBlock(
                d, heads, mlp_ratio=c.mlp_ratio, norm_type=c.norm_type, norm_eps=c.norm_eps, qkv_bias=c.qkv_bias,
                proj_bias=c.proj_bias, mlp_bias=c.mlp_bias, dropout=c.dropout, attention_dropout=c.attention_dropout,
                drop_path=rates[cursor + i]) for i in range(depth)))
            cursor += depth
        self.pools = nn.ModuleList(HierarchicalTokenPool(c.embed_dims[i], c.embed_dims[i + 1], norm_type=c.norm_type,
                                                         norm_eps=c.norm_eps, bias=c.pool_bias)
                                   for i in range(len(c.embed_dims) - 1))
        self.final_norm = build_vision_norm(c.norm_type, c.embed_dims[-1], c.norm_eps)
        self.apply(lambda m: initialize_vision_module(m, c.initializer_std))

    def forward(self, images, padding_mask=None, *, output_hidden_states=False, output_attentions=False):
        x, grid = self.patch_embedding(images)
        if padding_mask is not None and (padding_mask.shape != x.shape[:2] or padding_mask.dtype != torch.bool):
            raise ValueError("padding_mask must be boolean and match patch tokens")
        hs = [] if output_hidden_states else None
        at = [] if output_attentions else None
        for si, blocks in enumerate(self.stages):
            if len(self.position_embeddings):
                x = x + self.position_embeddings[si](grid, dtype=x.dtype, device=x.device)
            if hs is not None:
                hs.append(x)
            for blk in blocks:
                x, w = blk(x, padding_mask, output_attentions=output_attentions)
                if hs is not None:
                    hs.append(x)
                if at is not None:
                    at.append(w)
            if si < len(self.pools):
                x, grid, padding_mask = self.pools[si](x, grid, padding_mask)
        x = self.final_norm(x)
        if hs is not None:
            hs[-1] = x
        return VisionEncoderOutput(x, grid, tuple(hs) if hs is not None else None,
                                   tuple(at) if at is not None else None)


# --------------------------------------------------------------------------- swin
def window_partition(x, ws):
    """``[B,H,W,D]`` -> ``[B*nW, ws*ws, D]`` (zero-padded to multiples of ws)."""
    b, h, w, d = x.shape
    ph, pw = (-h) % ws, (-w) % ws
    x = F.pad(x, (0, 0, 0, pw, 0, ph))
    H, W = h + ph, w + pw
    win = x.reshape(b, H // ws, ws, W // ws, ws, d).permute(0, 1, 3, 2, 4, 5).reshape(-1, ws * ws, d)
    return win, (b, h, w, H, W)


def window_merge(win, ws, meta):
    b, h, w, H, W = meta
    d = win.shape[-1]
    x = win.reshape(b, H // ws, W // ws, ws, ws, d).permute(0, 1, 3, 2, 4, 5).reshape(b, H, W, d)
    return x[:, :h, :w]


class WindowSelfAttention(nn.Module):
    def __init__(self, dim, num_heads, window_size, *, qkv_bias=False, proj_bias=False, attention_dropout=0.0,
                 projection_dropout=0.0, use_relative_position_bias=True):
        super().__init__()
        if dim <= 0 or num_heads <= 0 or window_size <= 0 or dim % num_heads:
            raise ValueError("invalid window attention configuration")
        self.dim, self.num_heads, self.window_size = dim, num_heads, window_size
        self.head_dim = dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.qkv = nn.Linear(dim, 3 * dim, bias=qkv_bias)
        self.projection = nn.Linear(dim, dim, bias=proj_bias)
        self.attention_dropout = nn.Dropout(attention_dropout)
        self.projection_dropout = nn.Dropout(projection_dropout)
        if use_relative_position_bias:
            side = 2 * window_size - 1
            self.relative_position_bias = nn.Parameter(torch.zeros(side * side, num_heads))
            r = torch.arange(window_size)
            coords = torch.stack(torch.meshgrid(r, r, indexing="ij")).flatten(1)  # [2, ws*ws]
            rel = (coords[:, :, None] - coords[:, None, :]) + (window_size - 1)
            self.register_buffer("relative_position_index", rel[0] * side + rel[1], persistent=False)
            nn.init.trunc_normal_(self.relative_position_bias, std=0.02)
        else:
            self.relative_position_bias = None
            self.register_buffer("relative_position_index", None, persistent=False)

    def forward(self, windows, attention_mask=None, *, output_attentions=False):
        bw, n, _ = windows.shape
        if n != self.window_size ** 2:
            raise ValueError(f"each window must contain {self.window_size ** 2} tokens")
        q, k, v = self.qkv(windows).reshape(bw, n, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        scores = (q @ k.transpose(-2, -1)) * self.scale
        if self.relative_position_bias is not None:
            bias = self.relative_position_bias[self.relative_position_index.reshape(-1)]
            scores = scores + bias.reshape(n, n, self.num_heads).permute(2, 0, 1).unsqueeze(0)
        scores32 = scores.float()
        if attention_mask is not None:
            # the fill is float32's lowest value: a float64 lowest value would become -inf in the fp32
            # softmax, and a fully padded window row would turn into NaN (and NaN weight gradients)
            scores32 = scores32.masked_fill(~attention_mask[:, None], torch.finfo(torch.float32).min)
        p = F.softmax(scores32, dim=-1).to(scores.dtype)
        if attention_mask is not None:
            p = p * attention_mask[:, None].to(p.dtype)
            p = p / p.sum(-1, keepdim=True).clamp_min(torch.finfo(p.dtype).tiny)
        out = (self.attention_dropout(p) @ v).transpose(1, 2).reshape(bw, n, self.dim)
        return self.projection_dropout(self.projection(out)), (p if output_attentions else None)


class SwinTransformerBlock(nn.Module):
    def __init__(self, dim, num_heads, window_size, shift_size, *, mlp_ratio, norm_type, norm_eps, qkv_bias,
                 proj_bias, mlp_bias, dropout, attention_dropout, drop_path, use_relative_position_bias):
        super().__init__()
        if not 0 <= shift_size < window_size:
            raise ValueError("shift_size must be in [0, window_size)")
        self.dim, self.window_size, self.shift_size = dim, window_size, shift_size
        self.norm1 = build_vision_norm(norm_type, dim, norm_eps)
        self.attention = WindowSelfAttention(dim, num_heads, window_size, qkv_bias=qkv_bias, proj_bias=proj_bias,
                                             attention_dropout=attention_dropout, projection_dropout=dropout,
                                             use_relative_position_bias=use_relative_position_bias)
        self.drop_path1 = DropPath(drop_path)
        self.norm2 = build_vision_norm(norm_type, dim, norm_eps)
        self.mlp = VisionMLP(dim, int(dim * mlp_ratio), dropout=dropout, bias=mlp_bias)
        self.drop_path2 = DropPath(drop_path)

    def _attention_mask(self, b, h, w, device, padding_mask):
        valid = (torch.ones(b, h, w, dtype=torch.bool, device=device) if padding_mask is None
                 else padding_mask.reshape(b, h, w))
        region = torch.zeros(1, h, w, dtype=torch.long, device=device)
        if self.shift_size:
            # After rolling, tokens only attend to tokens from their own pre-shift window.
            rid = torch.arange(h, device=device) // self.window_size
            cid = torch.arange(w, device=device) // self.window_size
            region = (rid[:, None] * (w + 1) + cid[None, :]).unsqueeze(0)
            s = (-self.shift_size, -self.shift_size)
            valid, region = torch.roll(valid, s, (1, 2)), torch.roll(region, s, (1, 2))
        vw = window_partition(valid.unsqueeze(-1), self.window_size)[0].squeeze(-1)
        rw = window_partition(region.unsqueeze(-1), self.window_size)[0].squeeze(-1)
        if rw.shape[0] != vw.shape[0]:
            rw = rw.repeat(b, 1)
        return vw[:, :, None] & vw[:, None, :] & rw[:, :, None].eq(rw[:, None, :])

    def forward(self, tokens, grid_size, padding_mask=None, *, output_attentions=False):
        b, h, w = validate_token_grid(tokens, grid_size, self.dim)
        x = self.norm1(tokens).reshape(b, h, w, self.dim)
        mask = self._attention_mask(b, h, w, x.device, padding_mask)
        if self.shift_size:
            x = torch.roll(x, (-self.shift_size, -self.shift_size), (1, 2))
        win, meta = window_partition(x, self.window_size)
        win, weights = self.attention(win, mask, output_attentions=output_attentions)
        x = window_merge(win, self.window_size, meta)
        if self.shift_size:
            x = torch.roll(x, (self.shift_size, self.shift_size), (1, 2))
        x = tokens + self.drop_path1(x.reshape(b, -1, self.dim))
        return x + self.drop_path2(self.mlp(self.norm2(x))), weights


class SwinPatchMerging(nn.Module):
    def __init__(self, input_dim, output_dim, *, norm_type, norm_eps, bias):
        super().__init__()
        self.input_dim = input_dim
        self.norm = build_vision_norm(norm_type, 4 * input_dim, norm_eps)
        self.reduction = nn.Linear(4 * input_dim, output_dim, bias=bias)

    def forward(self, tokens, grid_size, padding_mask=None):
        b, h, w = validate_token_grid(tokens, grid_size, self.input_dim)
        ph, pw = h % 2, w % 2
        x = F.pad(tokens.reshape(b, h, w, self.input_dim), (0, 0, 0, pw, 0, ph))
        x = torch.cat((x[:, 0::2, 0::2], x[:, 0::2, 1::2], x[:, 1::2, 0::2], x[:, 1::2, 1::2]), -1)
        grid = (x.shape[1], x.shape[2])
        x = self.reduction(self.norm(x)).reshape(b, -1, self.reduction.out_features)
        nm = None
        if padding_mask is not None:
            m = F.pad(padding_mask.reshape(b, h, w), (0, pw, 0, ph), value=False)
            nm = (m[:, 0::2, 0::2] | m[:, 0::2, 1::2] | m[:, 1::2, 0::2] | m[:, 1::2, 1::2]).flatten(1)
        return x, grid, nm


@dataclass(frozen=True)
class SwinVisionConfig:
    image_size: int | tuple = 224
    patch_size: int | tuple = 14
    in_channels: int = 3
    embed_dims: tuple = (96, 192, 384)
    depths: tuple = (2, 2, 4)
    num_heads: tuple = (6, 12, 12)
    window_size: int = 4
    mlp_ratio: float = 4.0
    norm_type: str = "rmsnorm"
    norm_eps: float = 1e-6
    patch_bias: bool = False
    qkv_bias: bool = False
    proj_bias: bool = False
    mlp_bias: bool = False
    merge_bias: bool = False
    dropout: float = 0.0
    attention_dropout: float = 0.0
    drop_path_rate: float = 0.0
    use_relative_position_bias: bool = True
    initializer_std: float = 0.02

    def __post_init__(self):
        _check_stages(self)
        if self.window_size <= 0:
            raise ValueError("window_size must be > 0")


class SwinMoonViTEncoder(nn.Module):
    def __init__(self, config: SwinVisionConfig):
        super().__init__()
        self.config = c = config
        self.patch_embedding = VisionPatchEmbedding(c.in_channels, c.embed_dims[0], c.patch_size, bias=c.patch_bias)
        rates = torch.linspace(0, c.drop_path_rate, sum(c.depths)).tolist()
        cursor, self.stages = 0, nn.ModuleList()
        for d, depth, heads in zip(c.embed_dims, c.depths, c.num_heads):
            self.stages.append(nn.ModuleList(SwinTransformerBlock(
                d, heads, c.window_size, 0 if i % 2 == 0 else c.window_size // 2, mlp_ratio=c.mlp_ratio,
                norm_type=c.norm_type, norm_eps=c.norm_eps, qkv_bias=c.qkv_bias, proj_bias=c.proj_bias,
                mlp_bias=c.mlp_bias, dropout=c.dropout, attention_dropout=c.attention_dropout,
                drop_path=rates[cursor + i], use_relative_position_bias=c.use_relative_position_bias)
                for i in range(depth)))
            cursor += depth
        self.mergers = nn.ModuleList(SwinPatchMerging(c.embed_dims[i], c.embed_dims[i + 1], norm_type=c.norm_type,
                                                      norm_eps=c.norm_eps, bias=c.merge_bias)
                                     for i in range(len(c.embed_dims) - 1))
        self.final_norm = build_vision_norm(c.norm_type, c.embed_dims[-1], c.norm_eps)
        self.apply(lambda m: initialize_vision_module(m, c.initializer_std))

    def forward(self, images, padding_mask=None, *, output_hidden_states=False, output_attentions=False):
        x, grid = self.patch_embedding(images)
        if padding_mask is not None and (padding_mask.shape != x.shape[:2] or padding_mask.dtype != torch.bool):
            raise ValueError("padding_mask must be boolean and match patch tokens")
        hs = [x] if output_hidden_states else None
        at = [] if output_attentions else None
        for si, blocks in enumerate(self.stages):
            for blk in blocks:
                x, w = blk(x, grid, padding_mask, output_attentions=output_attentions)
                if hs is not None:
                    hs.append(x)
                if at is not None:
                    at.append(w)
            if si < len(self.mergers):
                x, grid, padding_mask = self.mergers[si](x, grid, padding_mask)
                if hs is not None:
                    hs.append(x)  # the merged tokens open the next stage
        x = self.final_norm(x)
        if hs is not None:
            hs[-1] = x
        return VisionEncoderOutput(x, grid, tuple(hs) if hs is not None else None,
                                   tuple(at) if at is not None else None)


__all__ = [
    "HierarchicalTokenPool", "HierarchicalVisionConfig", "HierarchicalMoonViTEncoder", "window_partition",
    "window_merge", "WindowSelfAttention", "SwinTransformerBlock", "SwinPatchMerging", "SwinVisionConfig",
    "SwinMoonViTEncoder",
]
