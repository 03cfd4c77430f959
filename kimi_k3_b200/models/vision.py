"""Vision path: MoonViT encoder, 2x2 token packing, projector, placeholder composer.

Parity targets (reference paths):
  * ``src/vision/vision_encoder.py:70-176``  MoonViTEncoder + VisionEncoderConfig
  * ``src/vision/{patch_embedding,positional_embedding,vision_block,vision_attention,vision_mlp,
    drop_path,pixel_shuffle,projector,utils}.py``
  * ``src/kimi_k3/vision_integration.py:26-221``  encode / pack / project / compose
  * ``src/kimi_k3/multimodal_composer.py:11-178`` placeholder replacement (length preserving)

The hierarchical (PiT pooling) and Swin ablation encoders live in
:mod:`kimi_k3_b200.models.vision_ablations`.
"""
from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..runtime import host_checks
from .primitives import RMSNorm


def to_2tuple(value, name: str) -> tuple[int, int]:
    if isinstance(value, int):
        pair = (value, value)
    elif isinstance(value, Sequence) and len(value) == 2:
        pair = (int(value[0]), int(value[1]))
    else:
        raise ValueError(f"{name} must be an int or a sequence of length 2")
    if pair[0] <= 0 or pair[1] <= 0:
        raise ValueError(f"{name} values must be > 0, got {pair}")
    return pair


def build_vision_norm(norm_type: str, dim: int, eps: float = 1e-6) -> nn.Module:
    if norm_type.lower() == "rmsnorm":
        return RMSNorm(dim, eps=eps)
    if norm_type.lower() == "layernorm":
        return nn.LayerNorm(dim, eps=eps)
    raise ValueError(f"norm_type must be 'rmsnorm' or 'layernorm', got {norm_type!r}")


def initialize_vision_module(module: nn.Module, std: float = 0.02) -> None:
    if isinstance(module, (nn.Linear, nn.Conv2d)):
        nn.init.trunc_normal_(module.weight, std=std)
        if module.bias is not None:
            nn.init.zeros_(module.bias)
    elif isinstance(module, nn.LayerNorm) and module.elementwise_affine:
        nn.init.ones_(module.weight)
        nn.init.zeros_(module.bias)


def validate_token_grid(tokens, grid_size, dim=None):
    if tokens.ndim != 3:
        raise ValueError("tokens must have shape [B, N, D]")
    b, n, w = tokens.shape
    h, gw = to_2tuple(grid_size, "grid_size")
    if n != h * gw:
        raise ValueError(f"token count N={n} does not match grid {grid_size}")
    if dim is not None and w != dim:
        raise ValueError(f"token width must be {dim}, got {w}")
    return b, h, gw


@dataclass
class VisionEncoderOutput:
    last_hidden_state: torch.Tensor
    grid_size: tuple
    hidden_states: tuple | None = None
    attentions: tuple | None = None


@dataclass
class PixelShuffleOutput:
    last_hidden_state: torch.Tensor
    grid_size: tuple


@dataclass(frozen=True)
class VisionEncoderConfig:
    image_size: int | tuple = 224
    patch_size: int | tuple = 14
    in_channels: int = 3
    embed_dim: int = 192
    depth: int = 6
    num_heads: int = 12
    mlp_ratio: float = 4.0
    norm_type: str = "rmsnorm"
    norm_eps: float = 1e-6
    position_embedding_type: str = "learned_absolute"
    use_cls_token: bool = False
    patch_bias: bool = False
    qkv_bias: bool = False
    proj_bias: bool = False
    mlp_bias: bool = False
    dropout: float = 0.0
    attention_dropout: float = 0.0
    drop_path_rate: float = 0.0
    initializer_std: float = 0.02

    def __post_init__(self):
        image, patch = to_2tuple(self.image_size, "image_size"), to_2tuple(self.patch_size, "patch_size")
        if image[0] % patch[0] or image[1] % patch[1]:
            raise ValueError("configured image_size must be divisible by patch_size")
        if self.in_channels <= 0 or self.embed_dim <= 0 or self.depth <= 0 or self.num_heads <= 0:
            raise ValueError("vision dimensions must be > 0")
        if self.embed_dim % self.num_heads:
            raise ValueError("embed_dim must be divisible by num_heads")
        if self.mlp_ratio <= 0:
            raise ValueError("mlp_ratio must be > 0")
        if self.position_embedding_type not in ("none", "learned_absolute"):
            raise ValueError("position_embedding_type must be 'none' or 'learned_absolute'")
        if not (0 <= self.dropout < 1 and 0 <= self.attention_dropout < 1 and 0 <= self.drop_path_rate < 1):
            raise ValueError("invalid dropout probability")
        if self.initializer_std <= 0:
            raise ValueError("initializer_std must be > 0")


class VisionPatchEmbedding(nn.Module):
    def __init__(self, in_channels, embed_dim, patch_size, *, bias=False, device=None, dtype=None):
        super().__init__()
        if in_channels <= 0 or embed_dim <= 0:
            raise ValueError("in_channels and embed_dim must be > 0")
        self.in_channels, self.embed_dim = in_channels, embed_dim
        self.patch_size = to_2tuple(patch_size, "patch_size")
        self.projection = nn.Conv2d(in_channels, embed_dim, kernel_size=self.patch_size, stride=self.patch_size,
                                    bias=bias, device=device, dtype=dtype)

    def forward(self, images):
        if images.ndim != 4 or images.shape[1] != self.in_channels:
            raise ValueError(f"images must have shape [B,{self.in_channels},H,W]")
        h, w = images.shape[-2:]
        if h % self.patch_size[0] or w % self.patch_size[1]:
            raise ValueError("image size must be divisible by patch size")
        feats = self.projection(images)
        return feats.flatten(2).transpose(1, 2), (feats.shape[-2], feats.shape[-1])


class LearnedAbsolutePositionEmbedding(nn.Module):
    """Learned grid positions, bicubic-resampled for other grid sizes."""

    def __init__(self, base_grid_size, dim, *, use_cls_token=False):
        super().__init__()
        self.base_grid_size = to_2tuple(base_grid_size, "base_grid_size")
        self.dim, self.use_cls_token = dim, use_cls_token
        self.patch_positions = nn.Parameter(torch.empty(1, self.base_grid_size[0] * self.base_grid_size[1], dim))
        self.cls_position = nn.Parameter(torch.empty(1, 1, dim)) if use_cls_token else None
        nn.init.trunc_normal_(self.patch_positions, std=0.02)
        if self.cls_position is not None:
            nn.init.trunc_normal_(self.cls_position, std=0.02)

    def forward(self, grid_size, *, dtype=None, device=None):
        h, w = to_2tuple(grid_size, "grid_size")
        bh, bw = self.base_grid_size
        pos = self.patch_positions
        if (h, w) != self.base_grid_size:
            pos = pos.reshape(1, bh, bw, self.dim).permute(0, 3, 1, 2)
            pos = F.interpolate(pos.float(), size=(h, w), mode="bicubic", align_corners=False)
            pos = pos.to(self.patch_positions.dtype).permute(0, 2, 3, 1).reshape(1, h * w, self.dim)
        if self.cls_position is not None:
            pos = torch.cat((self.cls_position, pos), dim=1)
        return pos.to(dtype=dtype, device=device)


class DropPath(nn.Module):
    def __init__(self, drop_prob: float = 0.0):
        super().__init__()
        if not 0.0 <= drop_prob < 1.0:
            raise ValueError("drop_prob must be in [0, 1)")
        self.drop_prob = float(drop_prob)

    def forward(self, x):
        if self.drop_prob == 0.0 or not self.training:
            return x
        keep = 1.0 - self.drop_prob
        mask = torch.rand((x.shape[0],) + (1,) * (x.ndim - 1), dtype=x.dtype, device=x.device) < keep
        return x * mask.to(x.dtype) / keep


class VisionSelfAttention(nn.Module):
    """Bidirectional attention with a key-padding mask."""

    def __init__(self, dim, num_heads, *, qkv_bias=False, proj_bias=False, attention_dropout=0.0,
                 projection_dropout=0.0):
        super().__init__()
        if dim <= 0 or num_heads <= 0 or dim % num_heads:
            raise ValueError("dim must be a positive multiple of num_heads")
        self.dim, self.num_heads, self.head_dim = dim, num_heads, dim // num_heads
        self.scale = self.head_dim ** -0.5
        self.qkv = nn.Linear(dim, 3 * dim, bias=qkv_bias)
        self.attention_dropout = nn.Dropout(attention_dropout)
        self.projection = nn.Linear(dim, dim, bias=proj_bias)
        self.projection_dropout = nn.Dropout(projection_dropout)

    def forward(self, x, padding_mask=None, *, output_attentions=False):
        if x.ndim != 3 or x.shape[-1] != self.dim:
            raise ValueError(f"x must have shape [B, N, {self.dim}]")
        b, n, _ = x.shape
        q, k, v = self.qkv(x).reshape(b, n, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4)
        if not output_attentions and x.is_cuda and self.attention_dropout.p == 0.0:
            from .. import ops as _ops
            if _ops.use_kernels(x):
                out = _ops.flash_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), causal=False,
                                           key_padding_mask=padding_mask)
                out = out.to(x.dtype).reshape(b, n, self.dim)
                return self.projection_dropout(self.projection(out)), None
        scores = (q @ k.transpose(-2, -1)) * self.scale
        if padding_mask is not None:
            vk = padding_mask[:, None, None, :]
            scores = scores.masked_fill(~vk, torch.finfo(scores.dtype).min)
        probs = F.softmax(scores.float(), dim=-1).to(scores.dtype)
        if padding_mask is not None:
            probs = probs * vk.to(probs.dtype)
            probs = probs / probs.sum(-1, keepdim=True).clamp_min(torch.finfo(probs.dtype).tiny)
        out = (self.attention_dropout(probs) @ v).transpose(1, 2).reshape(b, n, self.dim)
        return self.projection_dropout(self.projection(out)), (probs if output_attentions else None)


class VisionMLP(nn.Module):
    def __init__(self, dim, hidden_dim, *, dropout=0.0, bias=False):
        super().__init__()
        self.dim = dim
        self.fc1 = nn.Linear(dim, hidden_dim, bias=bias)
        self.activation = nn.GELU()
        self.dropout1 = nn.Dropout(dropout)
        self.fc2 = nn.Linear(hidden_dim, dim, bias=bias)
        self.dropout2 = nn.Dropout(dropout)

    def forward(self, x):
        return self.dropout2(self.fc2(self.dropout1(self.activation(self.fc1(x)))))


class VisionTransformerBlock(nn.Module):
    def __init__(self, dim, num_heads, *, mlp_ratio=4.0, norm_type="rmsnorm", norm_eps=1e-6, qkv_bias=False,
                 proj_bias=False, mlp_bias=False, dropout=0.0, attention_dropout=0.0, drop_path=0.0):
        super().__init__()
        self.norm1 = build_vision_norm(norm_type, dim, norm_eps)
        self.attention = VisionSelfAttention(dim, num_heads, qkv_bias=qkv_bias, proj_bias=proj_bias,
                                             attention_dropout=attention_dropout, projection_dropout=dropout)
        self.drop_path1 = DropPath(drop_path)
        self.norm2 = build_vision_norm(norm_type, dim, norm_eps)
        self.mlp = VisionMLP(dim, int(dim * mlp_ratio), dropout=dropout, bias=mlp_bias)
        self.drop_path2 = DropPath(drop_path)

    def forward(self, x, padding_mask=None, *, output_attentions=False):
        att, w = self.attention(self.norm1(x), padding_mask, output_attentions=output_attentions)
        x = x + self.drop_path1(att)
        return x + self.drop_path2(self.mlp(self.norm2(x))), w


class MoonViTEncoder(nn.Module):
    """Flat global-attention MoonViT encoder (no classifier head)."""

    def __init__(self, config: VisionEncoderConfig):
        super().__init__()
        self.config = c = config
        image, patch = to_2tuple(c.image_size, "image_size"), to_2tuple(c.patch_size, "patch_size")
        self.patch_embedding = VisionPatchEmbedding(c.in_channels, c.embed_dim, patch, bias=c.patch_bias)
        self.cls_token = nn.Parameter(torch.empty(1, 1, c.embed_dim)) if c.use_cls_token else None
        grid = (image[0] // patch[0], image[1] // patch[1])
        self.position_embedding = (LearnedAbsolutePositionEmbedding(grid, c.embed_dim, use_cls_token=c.use_cls_token)
                                   if c.position_embedding_type == "learned_absolute" else None)
        rates = torch.linspace(0, c.drop_path_rate, c.depth).tolist()
        self.blocks = nn.ModuleList(VisionTransformerBlock(
            c.embed_dim, c.num_heads, mlp_ratio=c.mlp_ratio, norm_type=c.norm_type, norm_eps=c.norm_eps,
            qkv_bias=c.qkv_bias, proj_bias=c.proj_bias, mlp_bias=c.mlp_bias, dropout=c.dropout,
            attention_dropout=c.attention_dropout, drop_path=rates[i]) for i in range(c.depth))
        self.final_norm = build_vision_norm(c.norm_type, c.embed_dim, c.norm_eps)
        self.apply(lambda m: initialize_vision_module(m, c.initializer_std))
        if self.cls_token is not None:
            nn.init.trunc_normal_(self.cls_token, std=c.initializer_std)

    def forward(self, images, padding_mask=None, *, output_hidden_states=False, output_attentions=False):
        x, grid = self.patch_embedding(images)
        b, n, _ = x.shape
        if padding_mask is not None and (tuple(padding_mask.shape) != (b, n) or padding_mask.dtype != torch.bool):
            raise ValueError(f"padding_mask must be boolean with shape {(b, n)}")
        if self.cls_token is not None:
            x = torch.cat((self.cls_token.expand(b, -1, -1), x), dim=1)
            if padding_mask is not None:
                padding_mask = torch.cat((torch.ones(b, 1, dtype=torch.bool, device=x.device), padding_mask), 1)
        if self.position_embedding is not None:
            x = x + self.position_embedding(grid, dtype=x.dtype, device=x.device)
        hs = [x] if output_hidden_states else None
        at = [] if output_attentions else None
        for blk in self.blocks:
            x, w = blk(x, padding_mask, output_attentions=output_attentions)
            if hs is not None:
                hs.append(x)
            if at is not None:
                at.append(w)
        x = self.final_norm(x)
        if hs is not None:
            hs[-1] = x  # the last entry is the encoder's (normalised) output itself
        return VisionEncoderOutput(x, grid, tuple(hs) if hs is not None else None,
                                   tuple(at) if at is not None else None)


class SpatialTokenPixelShuffle(nn.Module):
    """Pack each 2x2 token neighbourhood into one token of width 4D."""

    def forward(self, tokens, grid_size) -> PixelShuffleOutput:
        b, h, w = validate_token_grid(tokens, grid_size)
        if h % 2 or w % 2:
            raise ValueError(f"pixel packing requires an even grid, got {(h, w)}")
        d = tokens.shape[-1]
        s = tokens.reshape(b, h, w, d)
        packed = torch.cat((s[:, 0::2, 0::2], s[:, 0::2, 1::2], s[:, 1::2, 0::2], s[:, 1::2, 1::2]), dim=-1)
        return PixelShuffleOutput(packed.reshape(b, -1, 4 * d), (h // 2, w // 2))


class VisionProjector(nn.Module):
    def __init__(self, input_dim, hidden_dim, output_dim, *, activation="gelu", bias=False):
        super().__init__()
        acts = {"gelu": nn.GELU, "silu": nn.SiLU}
        if min(input_dim, hidden_dim, output_dim) <= 0 or activation not in acts:
            raise ValueError("invalid projector configuration")
        self.input_dim = input_dim
        self.fc1 = nn.Linear(input_dim, hidden_dim, bias=bias)
        self.activation = acts[activation]()
        self.fc2 = nn.Linear(hidden_dim, output_dim, bias=bias)

    def forward(self, tokens):
        if tokens.ndim != 3 or tokens.shape[-1] != self.input_dim:
            raise ValueError(f"tokens must have shape [B, N, {self.input_dim}]")
        return self.fc2(self.activation(self.fc1(tokens)))


# --------------------------------------------------------------------------- composition
@dataclass
class MultimodalMetadata:
    image_counts: torch.Tensor | None = None
    video_counts: torch.Tensor | None = None
    image_token_counts: torch.Tensor | None = None
    video_token_counts: torch.Tensor | None = None
    image_positions: torch.Tensor | None = None
    video_positions: torch.Tensor | None = None


@dataclass
class KimiK3VisionOutput:
    images: VisionEncoderOutput | None = None
    videos: VisionEncoderOutput | None = None


class VisualPlaceholderComposer(nn.Module):
    """Replace image/video placeholder embeddings with projected visual tokens in place."""

    def __init__(self, d_model, image_token_id, video_token_id):
        super().__init__()
        self.d_model, self.image_token_id, self.video_token_id = d_model, image_token_id, video_token_id

    @staticmethod
    def resolve_counts(name, counts, batch_size, item_count, device):
        if counts is None:
            if item_count != batch_size:
                raise ValueError(f"{name} is required for {item_count} visual items and text batch size {batch_size}")
            return torch.ones(batch_size, dtype=torch.long, device=device)
        if tuple(counts.shape) != (batch_size,) or counts.dtype not in (torch.int32, torch.int64):
            raise ValueError(f"{name} must be an integer tensor of shape {(batch_size,)}")
        if torch.device(counts.device) != torch.device(device):
            raise ValueError(f"{name} must be on the text device")
        if torch.any(counts < 0) or int(counts.sum().item()) != item_count:
            raise ValueError(f"{name} must be non-negative and sum to {item_count}")
        return counts

    def _replace(self, composed, input_ids, attention_mask, token_id, projected, pmask, counts, modality):
        placeholders = input_ids.eq(token_id)
        if torch.any(placeholders & ~attention_mask):
            raise ValueError(f"{modality} placeholder cannot occur in masked padding")
        if projected is None:
            if torch.any(placeholders):
                raise ValueError(f"{modality} placeholders require matching visual inputs")
            return None, None
        if projected.ndim != 3 or projected.shape[-1] != self.d_model:
            raise ValueError(f"{modality} projection must have shape [M,N,{self.d_model}]")
        if counts is None:
            raise ValueError(f"{modality}_counts must be resolved before composition")
        cursor, positions, per_sample = 0, [], []
        for bi, n_items in enumerate(counts.tolist()):
            items = [projected[cursor + j][pmask[cursor + j]] for j in range(n_items)]
            cursor += n_items
            vis = torch.cat(items, 0) if items else projected.new_empty(0, self.d_model)
            pos = torch.nonzero(placeholders[bi], as_tuple=False).flatten()
            if pos.numel() != vis.shape[0]:
                raise ValueError(f"sample {bi} has {pos.numel()} {modality} placeholders but {vis.shape[0]} "
                                 "projected valid visual tokens")
            if pos.numel():
                composed[bi, pos] = vis.to(composed.dtype)
                positions.append(torch.stack((torch.full_like(pos, bi), pos), -1))
            per_sample.append(vis.shape[0])
        allpos = torch.cat(positions) if positions else torch.empty(0, 2, dtype=torch.long, device=input_ids.device)
        return allpos, torch.tensor(per_sample, dtype=torch.long, device=input_ids.device)

    def forward(self, text_embeddings, input_ids, attention_mask, *, image_embeddings=None, image_mask=None,
                image_counts=None, video_embeddings=None, video_mask=None, video_counts=None):
        composed = text_embeddings.clone()
        ip, ic = self._replace(composed, input_ids, attention_mask, self.image_token_id, image_embeddings, image_mask,
                               image_counts, "image")
        vp = vc = None
        if self.video_token_id is not None:
            vp, vc = self._replace(composed, input_ids, attention_mask, self.video_token_id, video_embeddings,
                                   video_mask, video_counts, "video")
        elif video_embeddings is not None:
            raise ValueError("video_token_id is required for video inputs")
        return composed, MultimodalMetadata(image_counts, video_counts, ic, vc, ip, vp)


def pack_visual_mask(mask, grid):
    b, n = mask.shape
    h, w = grid
    if n != h * w or h % 2 or w % 2:
        raise ValueError("visual mask is incompatible with pixel shuffle")
    s = mask.reshape(b, h, w)
    return (s[:, 0::2, 0::2] & s[:, 0::2, 1::2] & s[:, 1::2, 0::2] & s[:, 1::2, 1::2]).flatten(1)


def make_vision_encoder(config) -> nn.Module:
    from .vision_ablations import (HierarchicalMoonViTEncoder, HierarchicalVisionConfig, SwinMoonViTEncoder,
                                   SwinVisionConfig)
    if isinstance(config, VisionEncoderConfig):
        return MoonViTEncoder(config)
    if isinstance(config, HierarchicalVisionConfig):
        return HierarchicalMoonViTEncoder(config)
    if isinstance(config, SwinVisionConfig):
        return SwinMoonViTEncoder(config)
    raise TypeError("unsupported vision configuration")


def encode_visual_items(*, values, vision_mask, is_video, vision_encoder, vision_token_packer, vision_projector,
                        output_hidden_states, output_attentions):
    if is_video:
        if values.ndim != 5:
            raise ValueError("video_values must have shape [M,F,C,H,W]")
        items, frames = values.shape[:2]
        ev, em = values.flatten(0, 1), (None if vision_mask is None else vision_mask.flatten(0, 1))
    else:
        if values.ndim != 4:
            raise ValueError("pixel_values must have shape [M,C,H,W]")
        items, frames, ev, em = values.shape[0], 1, values, vision_mask
    enc = vision_encoder(ev, em, output_hidden_states=output_hidden_states, output_attentions=output_attentions)
    tokens = enc.last_hidden_state
    vmask = torch.ones(tokens.shape[:2], dtype=torch.bool, device=tokens.device) if em is None else em
    if vision_token_packer is not None:
        vmask = pack_visual_mask(vmask, enc.grid_size)
        tokens = vision_token_packer(tokens, enc.grid_size).last_hidden_state
    proj = vision_projector(tokens)
    if is_video:
        proj = proj.reshape(items, frames * proj.shape[1], proj.shape[2])
        vmask = vmask.reshape(items, -1)
    return proj, vmask, enc, items


def prepare_multimodal_embeddings(*, config, input_ids, text_embeddings, attention_mask, pixel_values, video_values,
                                  vision_attention_mask, image_counts, video_counts, vision_encoder,
                                  vision_token_packer, vision_projector, composer, output_hidden_states,
                                  output_attentions):
    has_visual = pixel_values is not None or video_values is not None
    if not has_visual:
        ids = [i for i in (config.image_token_id, config.video_token_id) if i is not None]
        if not ids:
            return text_embeddings, None, None
        if not host_checks() or not bool(torch.isin(input_ids, torch.tensor(ids, device=input_ids.device)).any()):
            return text_embeddings, None, None
    if not config.enable_vision:
        raise ValueError("visual inputs cannot be used when vision is disabled")
    if pixel_values is not None and video_values is not None and vision_attention_mask is not None:
        raise ValueError("vision_attention_mask is ambiguous for mixed image/video input")
    ie = im = io = ve = vm = vo = None
    kw = dict(vision_encoder=vision_encoder, vision_token_packer=vision_token_packer,
              vision_projector=vision_projector, output_hidden_states=output_hidden_states,
              output_attentions=output_attentions)
    if pixel_values is not None:
        ie, im, io, n = encode_visual_items(values=pixel_values, vision_mask=vision_attention_mask, is_video=False, **kw)
        image_counts = composer.resolve_counts("image_counts", image_counts, input_ids.shape[0], n, input_ids.device)
    if video_values is not None:
        ve, vm, vo, n = encode_visual_items(values=video_values, vision_mask=vision_attention_mask, is_video=True, **kw)
        video_counts = composer.resolve_counts("video_counts", video_counts, input_ids.shape[0], n, input_ids.device)
    composed, meta = composer(text_embeddings, input_ids, attention_mask, image_embeddings=ie, image_mask=im,
                              image_counts=image_counts, video_embeddings=ve, video_mask=vm, video_counts=video_counts)
    return composed, KimiK3VisionOutput(io, vo), meta


__all__ = [
    "VisionEncoderConfig", "VisionEncoderOutput", "PixelShuffleOutput", "VisionPatchEmbedding",
    "LearnedAbsolutePositionEmbedding", "DropPath", "VisionSelfAttention", "VisionMLP", "VisionTransformerBlock",
    "MoonViTEncoder", "SpatialTokenPixelShuffle", "VisionProjector", "VisualPlaceholderComposer",
    "MultimodalMetadata", "KimiK3VisionOutput", "make_vision_encoder", "encode_visual_items",
    "prepare_multimodal_embeddings", "pack_visual_mask", "to_2tuple", "build_vision_norm",
    "initialize_vision_module", "validate_token_grid",
]
