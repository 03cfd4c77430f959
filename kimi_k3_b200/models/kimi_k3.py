"""KimiK3: embedding -> (vision) -> KimiBlock -> tied LM head -> (MTP) -> pretraining loss.

Parity targets (reference paths):
  * ``src/kimi_k3_mini.py:36-487``        KimiK3 (forward / prefill / decode_step, weight tying)
  * ``src/kimi_k3/config.py:49-345``      KimiK3Config, VisionProjectorConfig, tiny + canonical builders
  * ``src/kimi_k3/outputs.py``            KimiK3Output, ParameterReport
  * ``src/kimi_k3/validation.py:12-73``   mask validation and full / prefill / decode resolution

``forward(..., compute_logits=False)`` with labels computes the NTP and MTP losses
straight from the final hidden states (fused vocabulary projection + CE on CUDA);
``logits`` is then ``None``.  The default keeps the reference behaviour.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Literal

import torch
import torch.nn as nn

from ..runtime import host_checks
from .attnres import AttentionResidualConfig
from .backbone import HybridBackboneCache, KimiBlock, KimiBlockConfig
from .kda import KDAConfig
from .losses import KimiPretrainingLoss, KimiPretrainingLossOutput
from .mla import GatedMLAConfig
from .moe import StableLatentMoEConfig
from .mtp import KimiMTPConfig, KimiMTPHead
from .vision import (SpatialTokenPixelShuffle, VisionEncoderConfig, VisionProjector, VisualPlaceholderComposer,
                     make_vision_encoder, prepare_multimodal_embeddings)
from .vision_ablations import HierarchicalVisionConfig, SwinVisionConfig


@dataclass(frozen=True)
class VisionProjectorConfig:
    input_dim: int
    hidden_dim: int
    output_dim: int
    activation: Literal["gelu", "silu"] = "gelu"
    bias: bool = False

    def __post_init__(self) -> None:
        if min(self.input_dim, self.hidden_dim, self.output_dim) <= 0:
            raise ValueError("vision projector dimensions must be > 0")
        if self.activation not in ("gelu", "silu"):
            raise ValueError("unsupported vision projector activation")


def vision_output_dim(config) -> int:
    return config.embed_dim if isinstance(config, VisionEncoderConfig) else config.embed_dims[-1]


@dataclass(frozen=True)
class KimiK3Config:
    vocab_size: int
    d_model: int
    backbone: KimiBlockConfig
    pad_token_id: int | None = None
    bos_token_id: int | None = None
    eos_token_id: int | None = None
    image_token_id: int | None = None
    video_token_id: int | None = None
    tie_word_embeddings: bool = True
    use_bias_in_lm_head: bool = False
    vision: object | None = None
    vision_projector: VisionProjectorConfig | None = None
    mtp: KimiMTPConfig | None = None
    enable_vision: bool = True
    enable_mtp: bool = True
    vision_token_integration: str = "replace"
    vision_use_pixel_shuffle: bool = True
    freeze_vision_encoder: bool = False
    initializer_range: float = 0.02
    return_dict: bool = True
    output_hidden_states: bool = False
    output_attentions: bool = False
    output_router_diagnostics: bool = False
    output_attnres_diagnostics: bool = False

    def __post_init__(self) -> None:
        if self.vocab_size <= 0 or self.d_model <= 0 or self.initializer_range <= 0:
            raise ValueError("vocab_size, d_model and initializer_range must be > 0")
        if self.backbone.d_model != self.d_model:
            raise ValueError("backbone.d_model must match d_model")
        ids = [v for v in (self.pad_token_id, self.bos_token_id, self.eos_token_id, self.image_token_id,
                           self.video_token_id) if v is not None]
        if any(not 0 <= v < self.vocab_size for v in ids):
            raise ValueError("special token IDs must be inside the vocabulary")
        if len(set(ids)) != len(ids):
            raise ValueError("non-None special token IDs must be distinct")
        if self.vision_token_integration != "replace":
            raise ValueError("only replacement visual integration is supported")
        if self.enable_vision:
            if self.vision is None or self.vision_projector is None:
                raise ValueError("vision and vision_projector are required when vision is enabled")
            if self.image_token_id is None:
                raise ValueError("image_token_id is required when vision is enabled")
            width = vision_output_dim(self.vision)
            if self.vision_projector.input_dim != (4 * width if self.vision_use_pixel_shuffle else width):
                raise ValueError("vision_projector.input_dim does not match the visual path")
            if self.vision_projector.output_dim != self.d_model:
                raise ValueError("vision_projector.output_dim must equal d_model")
            if (self.vision_use_pixel_shuffle and isinstance(self.vision, VisionEncoderConfig)
                    and self.vision.use_cls_token):
                raise ValueError("pixel shuffle is incompatible with a CLS token")
        if self.enable_mtp:
            if self.mtp is None or not self.mtp.enabled:
                raise ValueError("an enabled MTP config is required")
            if self.mtp.d_model != self.d_model or self.mtp.vocab_size != self.vocab_size:
                raise ValueError("MTP dimensions must match the main model")

    def to_dict(self) -> dict:
        v = asdict(self)
        if isinstance(self.vision, VisionEncoderConfig):
            v["vision_type"] = "moonvit"
        elif isinstance(self.vision, HierarchicalVisionConfig):
            v["vision_type"] = "hierarchical"
        elif isinstance(self.vision, SwinVisionConfig):
            v["vision_type"] = "swin"
        return v

    @classmethod
    def from_dict(cls, values: dict) -> "KimiK3Config":
        v = dict(values)
        v["backbone"] = KimiBlockConfig.from_dict(v["backbone"])
        vt = v.pop("vision_type", None)
        if isinstance(v.get("vision"), dict):
            classes = {"moonvit": VisionEncoderConfig, "hierarchical": HierarchicalVisionConfig,
                       "swin": SwinVisionConfig}
            if vt not in classes:
                raise ValueError("serialized vision_type is missing or invalid")
            vv = dict(v["vision"])
            for key in ("embed_dims", "depths", "num_heads", "image_size", "patch_size"):
                if isinstance(vv.get(key), list):
                    vv[key] = tuple(vv[key])
            v["vision"] = classes[vt](**vv)
        if isinstance(v.get("vision_projector"), dict):
            v["vision_projector"] = VisionProjectorConfig(**v["vision_projector"])
        if isinstance(v.get("mtp"), dict):
            v["mtp"] = KimiMTPConfig.from_dict(v["mtp"])
        return cls(**v)


def _text_configs(d_model, *, num_heads, key_head_dim, q_head_dim, latent_dim, shared_hidden, routed_hidden,
                  num_routed, top_k, num_shared, groups, attnres_sublayers, target_depth_blocks=None):
    vdim = d_model // num_heads
    kda = KDAConfig(d_model=d_model, num_heads=num_heads, key_head_dim=key_head_dim, value_head_dim=vdim,
                    short_conv_kernel_size=4, chunk_size=64, secondary_tile_size=16)
    mla = GatedMLAConfig(d_model=d_model, num_heads=num_heads, q_head_dim=q_head_dim, v_head_dim=vdim,
                         kv_latent_dim=min(latent_dim, num_heads * (q_head_dim + vdim)))
    moe = StableLatentMoEConfig(d_model=d_model, latent_dim=latent_dim, num_shared_experts=num_shared,
                                num_routed_experts=num_routed, routed_experts_per_token=top_k,
                                shared_expert_hidden_dim=shared_hidden, routed_expert_hidden_dim=routed_hidden)
    block = KimiBlockConfig(d_model=d_model, num_pattern_repeats=groups, kda_config=kda, mla_config=mla,
                            stable_latent_moe_config=moe,
                            attention_residual_config=AttentionResidualConfig(
                                d_model, mode="block", sublayers_per_depth_block=attnres_sublayers,
                                target_num_depth_blocks=target_depth_blocks, backend="eager"))
    return block, kda, mla, moe


def kimi_k3_cpu_tiny_config(*, enable_vision: bool = True, enable_mtp: bool = True) -> KimiK3Config:
    """Small but structurally complete configuration for CPU tests."""
    d, vocab = 16, 128
    block, kda, mla, moe = _text_configs(d, num_heads=2, key_head_dim=4, q_head_dim=4, latent_dim=8, shared_hidden=20,
                                         routed_hidden=16, num_routed=4, top_k=2, num_shared=1, groups=1,
                                         attnres_sublayers=4)
    mtp = KimiMTPConfig(d_model=d, vocab_size=vocab, kda_config=kda, mla_config=mla, stable_latent_moe_config=moe,
                        attention_residual_config=AttentionResidualConfig(d, mode="block", sublayers_per_depth_block=4,
                                                                          backend="eager"))
    return KimiK3Config(vocab_size=vocab, d_model=d, backbone=block, pad_token_id=0, bos_token_id=1, eos_token_id=2,
                        image_token_id=3, video_token_id=4,
                        vision=VisionEncoderConfig(image_size=16, patch_size=4, embed_dim=16, depth=2, num_heads=4,
                                                   use_cls_token=False),
                        vision_projector=VisionProjectorConfig(64, 32, d), mtp=mtp, enable_vision=enable_vision,
                        enable_mtp=enable_mtp)


def kimi_k3_canonical_config() -> KimiK3Config:
    """Canonical Kimi K3 architecture metadata (no weights are allocated)."""
    d, vocab = 7168, 160000
    block, kda, mla, moe = _text_configs(d, num_heads=56, key_head_dim=128, q_head_dim=128, latent_dim=3584,
                                         shared_hidden=3072, routed_hidden=3072, num_routed=896, top_k=16,
                                         num_shared=2, groups=23, attnres_sublayers=24, target_depth_blocks=8)
    mtp = KimiMTPConfig(d_model=d, vocab_size=vocab, kda_config=kda, mla_config=mla, stable_latent_moe_config=moe,
                        attention_residual_config=AttentionResidualConfig(d, mode="block", sublayers_per_depth_block=8,
                                                                          target_num_depth_blocks=1,
                                                                          backend="two_phase"))
    return KimiK3Config(vocab_size=vocab, d_model=d, backbone=block, pad_token_id=0, bos_token_id=1, eos_token_id=2,
                        image_token_id=3, video_token_id=4,
                        vision=VisionEncoderConfig(image_size=224, patch_size=14, embed_dim=1152, depth=27,
                                                   num_heads=16, use_cls_token=False),
                        vision_projector=VisionProjectorConfig(4608, 7168, d), mtp=mtp)


@dataclass
class KimiK3Output:
    logits: torch.Tensor | None
    last_hidden_state: torch.Tensor
    cache: HybridBackboneCache | None = None
    mtp_logits: torch.Tensor | None = None
    hidden_states: tuple | None = None
    backbone_diagnostics: dict | None = None
    backbone_trace: object | None = None
    attnres_diagnostics: object | None = None
    mtp_diagnostics: object | None = None
    vision_outputs: object | None = None
    multimodal_metadata: object | None = None
    loss: torch.Tensor | None = None
    ntp_loss: object | None = None
    mtp_loss: object | None = None
    loss_output: KimiPretrainingLossOutput | None = None

    def to_tuple(self) -> tuple:
        return (self.logits, self.cache, self.hidden_states, self.mtp_logits)


@dataclass(frozen=True)
class ParameterReport:
    total: int
    trainable: int
    embeddings: int
    vision: int
    backbone: int
    lm_head_unique: int
    mtp: int


def build_parameter_report(model) -> ParameterReport:
    def uniq(*mods):
        out = {}
        for m in mods:
            if m is not None:
                for p in m.parameters():
                    out[id(p)] = p
        return out
    allp, emb = uniq(model), uniq(model.embed_tokens)
    lm = uniq(model.lm_head)
    return ParameterReport(sum(p.numel() for p in allp.values()),
                           sum(p.numel() for p in allp.values() if p.requires_grad),
                           sum(p.numel() for p in emb.values()),
                           sum(p.numel() for p in uniq(model.vision_encoder, model.vision_projector).values()),
                           sum(p.numel() for p in uniq(model.backbone).values()),
                           sum(lm[k].numel() for k in set(lm) - set(emb)),
                           sum(p.numel() for p in uniq(model.mtp).values()))


def validate_and_build_attention_mask(input_ids, inputs_embeds, attention_mask, *, d_model, pad_token_id):
    if (input_ids is None) == (inputs_embeds is None):
        raise ValueError("exactly one of input_ids or inputs_embeds must be provided")
    if input_ids is not None:
        if input_ids.ndim != 2:
            raise ValueError("input_ids must have shape [B,T]")
        if input_ids.dtype not in (torch.int32, torch.int64):
            raise TypeError("input_ids must use an integer dtype")
        b, t = input_ids.shape
        src = input_ids
    else:
        if inputs_embeds.ndim != 3 or inputs_embeds.shape[-1] != d_model:
            raise ValueError(f"inputs_embeds must have shape [B,T,{d_model}]")
        b, t = inputs_embeds.shape[:2]
        src = inputs_embeds
    if t == 0:
        raise ValueError("empty token sequences are not supported")
    if attention_mask is None:
        attention_mask = (input_ids.ne(pad_token_id) if input_ids is not None and pad_token_id is not None
                          else torch.ones(b, t, dtype=torch.bool, device=src.device))
    if tuple(attention_mask.shape) != (b, t) or attention_mask.dtype != torch.bool:
        raise ValueError(f"attention_mask must be boolean with shape {(b, t)}")
    if not host_checks():  # the caller validated the host copy of the mask
        return b, t, attention_mask
    if t > 1 and torch.any((~attention_mask[:, :-1]) & attention_mask[:, 1:]):
        raise ValueError("left padding is not supported by the current hybrid backbone")
    if torch.any(attention_mask.sum(dim=1) == 0):
        raise ValueError("all-padding sequences are not supported")
    return b, t, attention_mask


def resolve_execution_mode(cache, use_cache, tokens) -> str:
    if cache is not None and not use_cache:
        raise ValueError("a cache requires use_cache=True")
    if cache is not None and tokens != 1:
        raise ValueError("cached decode accepts exactly one new token")
    if cache is not None:
        return "decode"
    return "prefill" if use_cache else "full"


class KimiK3(nn.Module):
    """Complete Kimi K3 model; owns every trainable high-level path exactly once."""

    config_class = KimiK3Config

    def __init__(self, config: KimiK3Config):
        super().__init__()
        self.config = c = config
        self.embed_tokens = nn.Embedding(c.vocab_size, c.d_model, padding_idx=c.pad_token_id)
        self.backbone = KimiBlock(c.backbone)
        self.lm_head = nn.Linear(c.d_model, c.vocab_size, bias=c.use_bias_in_lm_head)
        if c.enable_vision:
            self.vision_encoder = make_vision_encoder(c.vision)
            self.vision_token_packer = SpatialTokenPixelShuffle() if c.vision_use_pixel_shuffle else None
            p = c.vision_projector
            self.vision_projector = VisionProjector(p.input_dim, p.hidden_dim, p.output_dim, activation=p.activation,
                                                    bias=p.bias)
            self.multimodal_composer = VisualPlaceholderComposer(c.d_model, c.image_token_id, c.video_token_id)
        else:
            self.vision_encoder = self.vision_token_packer = self.vision_projector = self.multimodal_composer = None
        nn.init.normal_(self.embed_tokens.weight, std=c.initializer_range)
        if c.pad_token_id is not None:
            with torch.no_grad():
                self.embed_tokens.weight[c.pad_token_id].zero_()
        nn.init.normal_(self.lm_head.weight, std=c.initializer_range)
        if self.lm_head.bias is not None:
            nn.init.zeros_(self.lm_head.bias)
        self.tie_weights()
        self.mtp = (KimiMTPHead(c.mtp, self.embed_tokens, self.lm_head, register_shared_modules=False)
                    if c.enable_mtp else None)
        self.pretraining_loss = KimiPretrainingLoss(
            lambda_mtp=c.mtp.loss_weight if c.enable_mtp and c.mtp is not None else 0.0,
            ignore_index=c.mtp.ignore_index if c.mtp is not None else -100)
        if c.freeze_vision_encoder and self.vision_encoder is not None:
            self.vision_encoder.requires_grad_(False)

    # ---- module access
    def get_input_embeddings(self):
        return self.embed_tokens

    def set_input_embeddings(self, value: nn.Embedding) -> None:
        if value.num_embeddings != self.config.vocab_size or value.embedding_dim != self.config.d_model:
            raise ValueError("replacement input embeddings have invalid shape")
        self.embed_tokens = value
        if self.mtp is not None:
            self.mtp.set_shared_modules(self.embed_tokens, self.lm_head)

    def get_output_embeddings(self):
        return self.lm_head

    def set_output_embeddings(self, value: nn.Linear) -> None:
        if value.in_features != self.config.d_model or value.out_features != self.config.vocab_size:
            raise ValueError("replacement LM head has invalid shape")
        self.lm_head = value
        if self.mtp is not None:
            self.mtp.set_shared_modules(self.embed_tokens, self.lm_head)

    def tie_weights(self) -> None:
        if self.config.tie_word_embeddings:
            self.lm_head.weight = self.embed_tokens.weight
        if getattr(self, "mtp", None) is not None:
            self.mtp.set_shared_modules(self.embed_tokens, self.lm_head)

    def get_vision_encoder(self):
        return self.vision_encoder

    def get_backbone(self):
        return self.backbone

    def get_mtp_head(self):
        return self.mtp

    def num_parameters(self, only_trainable: bool = False) -> int:
        uniq = {id(p): p for p in self.parameters()}.values()
        return sum(p.numel() for p in uniq if not only_trainable or p.requires_grad)

    def parameter_report(self) -> ParameterReport:
        return build_parameter_report(self)

    # ---- forward
    def forward(self, input_ids=None, attention_mask=None, position_ids=None, inputs_embeds=None, pixel_values=None,
                video_values=None, vision_attention_mask=None, image_counts=None, video_counts=None, cache=None,
                use_cache=False, cache_position=None, use_mtp=False, labels=None, training_phase=None, loss_mask=None,
                boundary_mask=None, token_weights=None, output_hidden_states=None, output_attentions=None,
                output_router_diagnostics=None, output_attnres_diagnostics=None, return_dict=None,
                compute_logits: bool = True, update_routing_bias: bool = False):
        c = self.config
        if position_ids is not None:
            raise ValueError("position_ids are unsupported because Kimi K3 uses NoPE")
        if cache_position is not None:
            raise ValueError("cache_position is owned by HybridBackboneCache")
        _, tokens, attention_mask = validate_and_build_attention_mask(input_ids, inputs_embeds, attention_mask,
                                                                      d_model=c.d_model, pad_token_id=c.pad_token_id)
        mode = resolve_execution_mode(cache, use_cache, tokens)
        if training_phase not in (None, "pretrain"):
            raise ValueError("KimiK3.forward only delegates pretraining loss; SFT/RL/MOPD use KimiTrainingObjective")
        if training_phase is not None and labels is None:
            raise ValueError("training_phase requires labels")
        if labels is not None and mode != "full":
            raise ValueError("training losses cannot run during prefill or decode")
        if labels is not None and labels.shape != attention_mask.shape:
            raise ValueError("labels must have shape [B,T]")
        if mode == "decode" and (pixel_values is not None or video_values is not None):
            raise ValueError("visual inputs are consumed during prefill, not decode")
        if inputs_embeds is not None and (pixel_values is not None or video_values is not None):
            raise ValueError("inputs_embeds cannot be combined with visual inputs")
        if use_mtp and self.mtp is None:
            raise ValueError("MTP was requested but is disabled")
        if use_mtp and mode != "full":
            raise ValueError("MTP is a full-sequence branch and cannot use cache")
        if use_mtp and input_ids is None:
            raise ValueError("MTP requires input_ids")
        if not compute_logits and labels is None:
            raise ValueError("compute_logits=False is only meaningful with labels")
        hidden_flag = c.output_hidden_states if output_hidden_states is None else output_hidden_states
        attn_flag = c.output_attentions if output_attentions is None else output_attentions
        router_flag = c.output_router_diagnostics if output_router_diagnostics is None else output_router_diagnostics
        attnres_flag = c.output_attnres_diagnostics if output_attnres_diagnostics is None else output_attnres_diagnostics

        emb = self.embed_tokens(input_ids) if input_ids is not None else inputs_embeds
        vis_out = meta = None
        # Decode steps carry generated tokens only: a generated id that equals a visual placeholder
        # is an ordinary token there (the visual inputs were consumed by the prefill).
        if input_ids is not None and mode != "decode":
            emb, vis_out, meta = prepare_multimodal_embeddings(
                config=c, input_ids=input_ids, text_embeddings=emb, attention_mask=attention_mask,
                pixel_values=pixel_values, video_values=video_values, vision_attention_mask=vision_attention_mask,
                image_counts=image_counts, video_counts=video_counts, vision_encoder=self.vision_encoder,
                vision_token_packer=self.vision_token_packer, vision_projector=self.vision_projector,
                composer=self.multimodal_composer, output_hidden_states=hidden_flag, output_attentions=attn_flag)
        if torch.is_autocast_enabled(emb.device.type) and emb.is_floating_point():
            # Keep the whole residual stream (AttnRes sources) in the autocast dtype.
            emb = emb.to(torch.get_autocast_dtype(emb.device.type))
        bo = self.backbone(emb, attention_mask=attention_mask, cache=cache, use_cache=use_cache, mode=mode,
                           output_hidden_states=hidden_flag, output_depth_weights=attnres_flag,
                           output_diagnostics=router_flag or attnres_flag, update_routing_bias=update_routing_bias)
        final = bo.last_hidden_state
        logits = self.lm_head(final) if compute_logits else None
        mtp_out = (self.mtp(final, input_ids, attention_mask=attention_mask, labels=labels, compute_loss=False,
                            return_logits=compute_logits, return_diagnostics=router_flag or attnres_flag,
                            update_routing_bias=update_routing_bias) if use_mtp else None)
        loss_out = None
        if labels is not None:
            if compute_logits:
                loss_out = self.pretraining_loss(
                    logits=logits, labels=labels, attention_mask=attention_mask, loss_mask=loss_mask,
                    boundary_mask=boundary_mask, token_weights=token_weights,
                    mtp_logits=None if mtp_out is None else mtp_out.logits,
                    mtp_labels=None if mtp_out is None else mtp_out.training_view.target_ids,
                    mtp_loss_mask=None if mtp_out is None else mtp_out.training_view.valid_mask,
                    future_offsets=None if mtp_out is None else (c.mtp.future_offset,))
            else:
                loss_out = self.pretraining_loss.forward_hidden(
                    hidden=final, head_weight=self.lm_head.weight, labels=labels, attention_mask=attention_mask,
                    loss_mask=loss_mask, boundary_mask=boundary_mask, token_weights=token_weights,
                    mtp_hidden=None if mtp_out is None else mtp_out.hidden_states,
                    mtp_labels=None if mtp_out is None else mtp_out.training_view.target_ids,
                    mtp_loss_mask=None if mtp_out is None else mtp_out.training_view.valid_mask,
                    future_offsets=None if mtp_out is None else (c.mtp.future_offset,))
        out = KimiK3Output(logits, final, bo.cache, None if mtp_out is None else mtp_out.logits, bo.hidden_states,
                           bo.diagnostics, bo.hidden_state_trace, bo.depth_outputs if attnres_flag else None,
                           None if mtp_out is None else mtp_out.diagnostics, vis_out, meta,
                           None if loss_out is None else loss_out.loss, None if loss_out is None else loss_out.ntp,
                           None if loss_out is None else loss_out.mtp, loss_out)
        use_dict = c.return_dict if return_dict is None else return_dict
        return out if use_dict else out.to_tuple()

    @torch.no_grad()
    def loss_normalizers(self, input_ids, labels=None, attention_mask=None, loss_mask=None, boundary_mask=None,
                         token_weights=None, use_mtp: bool = True) -> tuple:
        """``(ntp_normalizer, mtp_normalizer)`` the pretraining loss of this batch divides by.

        They depend only on ids, labels and masks, so a trainer computes them on the host copy
        of each micro-batch before the forward: accumulation windows can then backpropagate
        every micro-batch immediately with the window's global normalisers (token-exact, no
        retained graphs).
        """
        from .losses import align_token_inputs
        from .mtp import build_mtp_training_view
        labels = input_ids if labels is None else labels
        b, t = input_ids.shape
        if attention_mask is None:
            pad = self.config.pad_token_id
            attention_mask = input_ids.ne(pad) if pad is not None else torch.ones_like(input_ids, dtype=torch.bool)
        ntp = self.pretraining_loss.ntp_loss
        _, _, valid, w = align_token_inputs(labels, labels, alignment=ntp.label_alignment,
                                            attention_mask=attention_mask, loss_mask=loss_mask,
                                            boundary_mask=boundary_mask, token_weights=token_weights,
                                            ignore_index=ntp.ignore_index)
        ntp_n = float((w.float() * valid.float()).sum()) if token_weights is not None else float(valid.sum())
        mtp_n = 0.0
        if use_mtp and self.mtp is not None and self.config.enable_mtp and t > 2:
            view = build_mtp_training_view(input_ids.new_zeros(b, t, 1, dtype=torch.float32), input_ids,
                                           attention_mask, labels, ignore_index=self.pretraining_loss.mtp_loss.ignore_index)
            mtp_n = float((view.valid_mask & view.target_ids.ne(self.pretraining_loss.mtp_loss.ignore_index)).sum())
        return ntp_n, mtp_n

    @torch.no_grad()
    def prefill(self, input_ids, attention_mask=None, **kwargs):
        """Encode a prompt and build its cache with the same forward."""
        return self(input_ids=input_ids, attention_mask=attention_mask, use_cache=True, **kwargs)

    @torch.no_grad()
    def decode_step(self, input_ids, cache, attention_mask=None, **kwargs):
        """Advance one cached token (vision is not re-run)."""
        if cache is None:
            raise ValueError("decode_step requires a non-empty cache")
        return self(input_ids=input_ids, attention_mask=attention_mask, cache=cache, use_cache=True, **kwargs)


__all__ = [
    "VisionProjectorConfig", "vision_output_dim", "KimiK3Config", "kimi_k3_cpu_tiny_config",
    "kimi_k3_canonical_config", "KimiK3Output", "ParameterReport", "build_parameter_report", "KimiK3",
    "validate_and_build_attention_mask", "resolve_execution_mode",
]
