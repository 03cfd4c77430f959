"""Hybrid 3:1 KDA : Gated-MLA backbone with Stable LatentMoE and AttnRes.

Parity targets (reference paths):
  * ``src/hybrid_backbone/config.py:17-179``          HybridBackboneConfig
  * ``src/hybrid_backbone/attention_layer.py:27-344`` standard and AttnRes layer forwards
  * ``src/hybrid_backbone/backbone.py:35-663``        groups, final MLA, final norm, caches
  * ``src/hybrid_backbone/cache.py:33-126``           HybridLayerCache / HybridBackboneCache
  * ``src/hybrid_backbone/dense_ffn.py``              DenseKimiFFN ablation
  * ``src/kimi_block.py:24-176``                      KimiBlockConfig / KimiBlock

An all-valid attention mask is collapsed to ``None`` once per forward so every
layer takes its mask-free fused CUDA path (one host check instead of one per layer).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Literal

import torch
import torch.nn as nn

from ..debug import nvtx
from ..runtime import host_checks, mask_all_valid
from .attnres import (AttentionResidualBackboneOutput, AttentionResidualConfig, AttentionResidualSite,
                      BlockAttentionResidualController, DepthSiteMetadata, FullAttentionResidualController,
                      FullAttentionResidualState, padded_weight_matrix)
from .kda import KDAConfig, KDAState, KimiDeltaAttention
from .mla import GatedMLA, GatedMLAConfig, MLACache
from .moe import StableLatentMoE, StableLatentMoEConfig, StableLatentMoEOutput
from .primitives import RMSNorm, SiTUGLU

CANONICAL_ATTENTION_PATTERN = ("kda", "kda", "kda", "gated_mla")
VALID_MODES = ("full", "prefill", "decode")


@dataclass(frozen=True)
class HybridBackboneConfig:
    d_model: int
    num_hybrid_groups: int
    attention_pattern: tuple = CANONICAL_ATTENTION_PATTERN
    enforce_canonical_pattern: bool = True
    add_final_gated_mla: bool = True
    add_ffn_after_final_global: bool = True
    rms_norm_eps: float = 1e-6
    residual_dropout: float = 0.0
    ffn_dropout: float = 0.0
    mlp_hidden_dim: int | None = None
    kda_config: KDAConfig | None = None
    mla_config: GatedMLAConfig | None = None
    use_dense_ffn: bool = True
    channel_mixer_type: str = "dense"
    stable_latent_moe_config: StableLatentMoEConfig | None = None
    activation: str = "situ_glu"
    ffn_bias: bool = False
    init_std: float = 0.02
    attention_residual_config: AttentionResidualConfig | None = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "attention_pattern", tuple(self.attention_pattern))
        if self.d_model <= 0 or self.num_hybrid_groups <= 0 or not self.attention_pattern:
            raise ValueError("d_model, num_hybrid_groups and attention_pattern must be non-empty/positive")
        unknown = set(self.attention_pattern) - {"kda", "gated_mla"}
        if unknown:
            raise ValueError(f"unsupported attention types: {sorted(unknown)}")
        if self.enforce_canonical_pattern and self.attention_pattern != CANONICAL_ATTENTION_PATTERN:
            raise ValueError(f"the Kimi K3 profile requires the explicit 3:1 pattern {CANONICAL_ATTENTION_PATTERN}")
        if self.enforce_canonical_pattern and not self.add_final_gated_mla:
            raise ValueError("the Kimi K3 profile requires a final Gated MLA")
        if "kda" in self.attention_pattern and self.kda_config is None:
            raise ValueError("kda_config is required by attention_pattern")
        if ("gated_mla" in self.attention_pattern or self.add_final_gated_mla) and self.mla_config is None:
            raise ValueError("mla_config is required by attention_pattern")
        for name in ("kda_config", "mla_config"):
            sub = getattr(self, name)
            if sub is not None and sub.d_model != self.d_model:
                raise ValueError(f"{name}.d_model must equal backbone d_model")
        if self.rms_norm_eps <= 0:
            raise ValueError("rms_norm_eps must be > 0")
        for name in ("residual_dropout", "ffn_dropout"):
            if not 0.0 <= getattr(self, name) < 1.0:
                raise ValueError(f"{name} must satisfy 0 <= p < 1")
        if self.channel_mixer_type not in ("dense", "stable_latent_moe"):
            raise ValueError("unknown channel_mixer_type")
        if self.channel_mixer_type == "dense" and not self.use_dense_ffn:
            raise ValueError("dense channel mixing requires use_dense_ffn=True")
        if self.channel_mixer_type == "stable_latent_moe":
            if self.use_dense_ffn:
                raise ValueError("Stable LatentMoE and DenseKimiFFN cannot be active together")
            if self.stable_latent_moe_config is None or self.stable_latent_moe_config.d_model != self.d_model:
                raise ValueError("a matching stable_latent_moe_config is required for MoE mixing")
        elif self.stable_latent_moe_config is not None:
            raise ValueError("stable_latent_moe_config is only valid for MoE mixing")
        if self.activation != "situ_glu":
            raise ValueError("only activation='situ_glu' is supported")
        if self.attention_residual_config is not None:
            if self.attention_residual_config.d_model != self.d_model:
                raise ValueError("attention_residual_config.d_model must match backbone")
            self.attention_residual_config.validate_topology(self.num_attention_layers,
                                                             every_layer_has_ffn=self.add_ffn_after_final_global)

    @property
    def depth_mixing(self) -> str:
        return "standard" if self.attention_residual_config is None else self.attention_residual_config.mode

    @property
    def resolved_mlp_hidden_dim(self) -> int:
        return 4 * self.d_model if self.mlp_hidden_dim is None else self.mlp_hidden_dim

    @property
    def num_group_layers(self) -> int:
        return self.num_hybrid_groups * len(self.attention_pattern)

    @property
    def num_attention_layers(self) -> int:
        return self.num_group_layers + int(self.add_final_gated_mla)

    @property
    def num_kda_layers(self) -> int:
        return self.num_hybrid_groups * self.attention_pattern.count("kda")

    @property
    def num_mla_layers(self) -> int:
        return self.num_hybrid_groups * self.attention_pattern.count("gated_mla") + int(self.add_final_gated_mla)

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "HybridBackboneConfig":
        v = dict(values)
        for key, typ in (("kda_config", KDAConfig), ("mla_config", GatedMLAConfig),
                         ("attention_residual_config", AttentionResidualConfig),
                         ("stable_latent_moe_config", StableLatentMoEConfig)):
            if isinstance(v.get(key), dict):
                v[key] = typ.from_dict(v[key])
        return cls(**v)


# --------------------------------------------------------------------------- caches / outputs
@dataclass
class HybridLayerCache:
    attention_type: str
    state: KDAState | MLACache

    def __post_init__(self) -> None:
        expected = KDAState if self.attention_type == "kda" else MLACache
        if self.attention_type not in ("kda", "gated_mla") or not isinstance(self.state, expected):
            raise TypeError(f"{self.attention_type} cache requires {expected.__name__}")

    @property
    def sequence_offsets(self) -> torch.Tensor:
        return self.state.sequence_offset

    @property
    def num_elements(self) -> int:
        s = self.state
        if isinstance(s, MLACache):
            return s.latent_kv.numel()
        return sum(t.numel() for t in (s.recurrent_state, s.q_conv_state.buffer, s.k_conv_state.buffer,
                                       s.v_conv_state.buffer))

    def clone(self) -> "HybridLayerCache":
        return HybridLayerCache(self.attention_type, self.state.clone())

    def reorder(self, indices) -> "HybridLayerCache":
        return HybridLayerCache(self.attention_type, self.state.reorder(indices))


@dataclass
class HybridBackboneCache:
    layer_caches: tuple
    sequence_length: int

    def __post_init__(self) -> None:
        self.layer_caches = tuple(self.layer_caches)
        if not self.layer_caches:
            raise ValueError("layer_caches must not be empty")
        if self.sequence_length < 0:
            raise ValueError("sequence_length must be >= 0")

    @property
    def sequence_lengths(self) -> torch.Tensor:
        return self.layer_caches[0].sequence_offsets

    @property
    def kda_elements(self) -> int:
        return sum(c.num_elements for c in self.layer_caches if c.attention_type == "kda")

    @property
    def mla_elements(self) -> int:
        return sum(c.num_elements for c in self.layer_caches if c.attention_type == "gated_mla")

    @property
    def total_elements(self) -> int:
        return self.kda_elements + self.mla_elements

    def clone(self) -> "HybridBackboneCache":
        return HybridBackboneCache(tuple(c.clone() for c in self.layer_caches), self.sequence_length)

    def reorder(self, indices) -> "HybridBackboneCache":
        caches = tuple(c.reorder(indices) for c in self.layer_caches)
        lens = caches[0].sequence_offsets
        return HybridBackboneCache(caches, int(lens.max().item()) if lens.numel() else 0)


@dataclass
class HybridLayerOutput:
    hidden_states: torch.Tensor
    cache: HybridLayerCache | None = None
    diagnostics: dict | None = None
    pre_attention_state: torch.Tensor | None = None
    attention_output: torch.Tensor | None = None
    pre_ffn_state: torch.Tensor | None = None
    ffn_output: torch.Tensor | None = None


@dataclass
class HybridGroupOutput:
    hidden_states: torch.Tensor
    layer_caches: tuple | None = None
    hidden_states_by_layer: tuple | None = None
    diagnostics: tuple | None = None


@dataclass
class BackboneHiddenStateTrace:
    embedding: torch.Tensor
    pre_attention: tuple
    attention_outputs: tuple
    pre_ffn: tuple
    ffn_outputs: tuple
    final_mixed: torch.Tensor


@dataclass
class HybridBackboneOutput:
    last_hidden_state: torch.Tensor
    cache: HybridBackboneCache | None = None
    hidden_states: tuple | None = None
    hidden_state_trace: BackboneHiddenStateTrace | None = None
    depth_outputs: AttentionResidualBackboneOutput | None = None
    diagnostics: dict | None = None


def validate_backbone_inputs(hidden_states, attention_mask, d_model, mode):
    if hidden_states.ndim != 3 or hidden_states.shape[-1] != d_model:
        raise ValueError(f"hidden_states must have shape [B,T,{d_model}]")
    b, t, _ = hidden_states.shape
    if t == 0:
        raise ValueError("hybrid backbone does not support empty sequences")
    if mode not in VALID_MODES:
        raise ValueError(f"unsupported execution mode {mode!r}")
    if mode == "decode" and t != 1:
        raise ValueError("decode mode requires exactly one token")
    if attention_mask is None:
        return b, t, torch.ones(b, t, dtype=torch.bool, device=hidden_states.device)
    from .kda import validate_attention_mask
    validate_attention_mask(attention_mask, b, t)
    return b, t, attention_mask


def masked_norm_mean(hidden_states, mask):
    if mask is None:
        return hidden_states.float().norm(dim=-1).mean()
    return hidden_states.float().norm(dim=-1)[mask].mean()


def count_parameters(module) -> int:
    return sum(p.numel() for p in module.parameters())


# --------------------------------------------------------------------------- layers
class DenseKimiFFN(nn.Module):
    """Dense SiTU-GLU channel mixer (ablation)."""

    def __init__(self, d_model, hidden_dim, dropout=0.0, bias=False, init_std=0.02):
        super().__init__()
        if not 0.0 <= dropout < 1.0:
            raise ValueError("dropout must satisfy 0 <= p < 1")
        self.d_model, self.hidden_dim = d_model, hidden_dim
        self.transform = SiTUGLU(d_model, hidden_dim, bias=bias, output_bias=bias, init_std=init_std)
        self.dropout = nn.Dropout(dropout)

    def forward(self, hidden_states):
        if hidden_states.ndim != 3 or hidden_states.shape[-1] != self.d_model:
            raise ValueError(f"hidden_states must have shape [B,T,{self.d_model}]")
        return self.dropout(self.transform(hidden_states))


class HybridAttentionLayer(nn.Module):
    """Pre-norm attention residual + pre-norm FFN residual (or the AttnRes form)."""

    def __init__(self, attention_type, attention_module, ffn_module, d_model, norm_eps, residual_dropout=0.0, *,
                 layer_index, group_index, position_in_group, is_final_global=False, pre_attention_attnres=None,
                 pre_ffn_attnres=None):
        super().__init__()
        if attention_type not in ("kda", "gated_mla"):
            raise ValueError("unsupported attention_type")
        expected = KimiDeltaAttention if attention_type == "kda" else GatedMLA
        if not isinstance(attention_module, expected):
            raise TypeError(f"{attention_type} requires {expected.__name__}")
        if is_final_global and attention_type != "gated_mla":
            raise ValueError("final global layer must use Gated MLA")
        self.attention_type, self.d_model = attention_type, d_model
        self.layer_index, self.group_index, self.position_in_group = layer_index, group_index, position_in_group
        self.is_final_global = is_final_global
        self.attention_norm = RMSNorm(d_model, eps=norm_eps)
        self.attention = attention_module
        self.ffn_norm = RMSNorm(d_model, eps=norm_eps) if ffn_module is not None else None
        self.ffn = ffn_module
        self.residual_dropout = nn.Dropout(residual_dropout)
        self.pre_attention_attnres = pre_attention_attnres
        self.pre_ffn_attnres = pre_ffn_attnres

    @property
    def attention_label(self) -> str:
        return "gated_mla_final" if self.is_final_global else self.attention_type

    @property
    def channel_mixer(self):
        return self.ffn

    @property
    def pre_moe_attnres(self):
        return self.pre_ffn_attnres

    @property
    def moe(self):
        return self.ffn if isinstance(self.ffn, StableLatentMoE) else None

    def _attention_transform(self, x, mask, cache, *, use_cache, mode, output_diagnostics):
        if cache is not None and cache.attention_type != self.attention_type:
            raise ValueError("cache type does not match attention layer")
        state = None if cache is None else cache.state
        normed = self.attention_norm(x)
        if self.attention_type == "kda":
            r = self.attention(normed, attention_mask=mask, state=state,
                               mode="decode" if mode == "decode" else "chunkwise",
                               output_final_state=use_cache, output_diagnostics=output_diagnostics)
            return r.hidden_states, r.state, r.diagnostics
        r = self.attention(normed, attention_mask=mask, cache=state, use_cache=use_cache,
                           output_diagnostics=output_diagnostics)
        return r.hidden_states, r.cache, r.diagnostics

    def _channel_mixer_transform(self, x, *, update_routing_bias, output_diagnostics):
        if isinstance(self.ffn, StableLatentMoE):
            r = self.ffn(x, update_routing_bias=update_routing_bias, return_router_diagnostics=output_diagnostics)
            if isinstance(r, StableLatentMoEOutput):
                return r.hidden_states, r.diagnostics
            return r, None
        return self.ffn(x), None

    def forward(self, hidden_states, attention_mask, cache=None, *, use_cache=False, mode="full",
                output_diagnostics=False, update_routing_bias=False) -> HybridLayerOutput:
        attn_out, nstate, mdiag = self._attention_transform(hidden_states, attention_mask, cache, use_cache=use_cache,
                                                            mode=mode, output_diagnostics=output_diagnostics)
        post = hidden_states + self.residual_dropout(attn_out)
        ffn_out, cdiag = torch.zeros_like(post), None
        if self.ffn is not None:
            ffn_out, cdiag = self._channel_mixer_transform(self.ffn_norm(post), update_routing_bias=update_routing_bias,
                                                           output_diagnostics=output_diagnostics)
        out = post + self.residual_dropout(ffn_out)
        diag = None
        if output_diagnostics:
            diag = {"layer_index": self.layer_index, "group_index": self.group_index,
                    "position_in_group": self.position_in_group, "attention_type": self.attention_label,
                    "input_norm": masked_norm_mean(hidden_states, attention_mask),
                    "attention_output_norm": masked_norm_mean(attn_out, attention_mask),
                    "post_attention_residual_norm": masked_norm_mean(post, attention_mask),
                    "ffn_output_norm": masked_norm_mean(ffn_out, attention_mask),
                    "post_ffn_residual_norm": masked_norm_mean(out, attention_mask),
                    "mechanism": mdiag, "channel_mixer": cdiag}
        return HybridLayerOutput(out, HybridLayerCache(self.attention_type, nstate) if use_cache else None, diag)

    def forward_attnres(self, depth_controller, depth_state, attention_mask, cache=None, *, depth_block_sites=None,
                        use_cache=False, mode="full", output_depth_weights=False, output_depth_stats=False,
                        output_diagnostics=False, update_routing_bias=False):
        if self.pre_attention_attnres is None or self.pre_ffn_attnres is None:
            raise RuntimeError("AttnRes sites are not configured on this layer")

        def prepare(site):
            if isinstance(depth_controller, BlockAttentionResidualController):
                depth_controller.prepare_depth_block(depth_state, depth_block_sites[site.metadata.depth_block_index])

        prepare(self.pre_attention_attnres)
        amix = depth_controller.mix_for_site(self.pre_attention_attnres, depth_state,
                                             return_weights=output_depth_weights, return_stats=output_depth_stats)
        attn_out, nstate, mdiag = self._attention_transform(amix.mixed_state, attention_mask, cache,
                                                            use_cache=use_cache, mode=mode,
                                                            output_diagnostics=output_diagnostics)
        attn_out = self.residual_dropout(attn_out)
        depth_controller.append_output(depth_state, attn_out)
        prepare(self.pre_ffn_attnres)
        fmix = depth_controller.mix_for_site(self.pre_ffn_attnres, depth_state,
                                             return_weights=output_depth_weights, return_stats=output_depth_stats)
        if self.ffn is None or self.ffn_norm is None:
            raise RuntimeError("canonical AttnRes requires an FFN at every transformer layer")
        raw, cdiag = self._channel_mixer_transform(self.ffn_norm(fmix.mixed_state),
                                                   update_routing_bias=update_routing_bias,
                                                   output_diagnostics=output_diagnostics)
        ffn_out = self.residual_dropout(raw)
        depth_controller.append_output(depth_state, ffn_out)
        diag = None
        if output_diagnostics:
            diag = {"layer_index": self.layer_index, "group_index": self.group_index,
                    "position_in_group": self.position_in_group, "attention_type": self.attention_label,
                    "pre_attention_depth_norm": masked_norm_mean(amix.mixed_state, attention_mask),
                    "attention_output_norm": masked_norm_mean(attn_out, attention_mask),
                    "pre_ffn_depth_norm": masked_norm_mean(fmix.mixed_state, attention_mask),
                    "ffn_output_norm": masked_norm_mean(ffn_out, attention_mask),
                    "mechanism": mdiag, "channel_mixer": cdiag}
        return (HybridLayerOutput(ffn_out, HybridLayerCache(self.attention_type, nstate) if use_cache else None, diag,
                                  amix.mixed_state, attn_out, fmix.mixed_state, ffn_out), (amix, fmix))


class HybridAttentionGroup(nn.Module):
    def __init__(self, layers, *, group_index: int):
        super().__init__()
        if not layers:
            raise ValueError("hybrid group must contain at least one layer")
        self.group_index = group_index
        self.layers = nn.ModuleList(layers)

    @property
    def attention_types(self):
        return tuple(layer.attention_type for layer in self.layers)

    def forward(self, hidden_states, attention_mask, cache=None, *, use_cache=False, mode="full",
                output_hidden_states=False, output_diagnostics=False, update_routing_bias=False):
        caches, states, diags = [], [], []
        out = hidden_states
        for i, layer in enumerate(self.layers):
            with nvtx(f"layer {i} {layer.attention_type}"):
                lo = layer(out, attention_mask, None if cache is None else cache[i], use_cache=use_cache, mode=mode,
                           output_diagnostics=output_diagnostics, update_routing_bias=update_routing_bias)
            out = lo.hidden_states
            if use_cache:
                caches.append(lo.cache)
            if output_hidden_states:
                states.append(out)
            if output_diagnostics:
                diags.append(lo.diagnostics)
        return HybridGroupOutput(out, tuple(caches) if use_cache else None,
                                 tuple(states) if output_hidden_states else None,
                                 tuple(diags) if output_diagnostics else None)


class HybridAttentionBackbone(nn.Module):
    """Groups of (KDA, KDA, KDA, MLA) + final global MLA + final RMSNorm."""

    def __init__(self, config: HybridBackboneConfig):
        super().__init__()
        self.config = config
        self.attnres_config = config.attention_residual_config
        groups, li = [], 0
        for gi in range(config.num_hybrid_groups):
            layers = []
            for pos, kind in enumerate(config.attention_pattern):
                layers.append(self._make_layer(kind, li, gi, pos, include_ffn=True))
                li += 1
            groups.append(HybridAttentionGroup(layers, group_index=gi))
        self.groups = nn.ModuleList(groups)
        self.final_global_layer = (self._make_layer("gated_mla", li, None, None,
                                                    include_ffn=config.add_ffn_after_final_global,
                                                    is_final_global=True)
                                   if config.add_final_gated_mla else None)
        self.final_norm = RMSNorm(config.d_model, eps=config.rms_norm_eps)
        if config.depth_mixing == "full":
            self.depth_controller = FullAttentionResidualController()
        elif config.depth_mixing == "block":
            self.depth_controller = BlockAttentionResidualController(
                self.attnres_config.resolved_sublayers_per_depth_block, backend=self.attnres_config.backend)
        else:
            self.depth_controller = None
        ar = self.attnres_config
        self.final_output_attnres = (
            AttentionResidualSite(config.d_model, eps=ar.rms_norm_eps, logits_in_fp32=ar.logits_in_fp32,
                                  weighted_sum_in_fp32=ar.weighted_sum_in_fp32,
                                  metadata=self._site_metadata(config.num_attention_layers, "final_output"))
            if ar is not None and ar.mode != "standard" else None)

    def _make_ffn(self):
        c = self.config
        if c.channel_mixer_type == "stable_latent_moe":
            return StableLatentMoE(c.stable_latent_moe_config)
        return DenseKimiFFN(c.d_model, c.resolved_mlp_hidden_dim, dropout=c.ffn_dropout, bias=c.ffn_bias,
                            init_std=c.init_std)

    def _make_layer(self, kind, li, gi, pos, *, include_ffn, is_final_global=False):
        c, ar = self.config, self.attnres_config
        attn = KimiDeltaAttention(c.kda_config) if kind == "kda" else GatedMLA(c.mla_config)
        pre_a = pre_f = None
        if ar is not None and ar.mode != "standard":
            kw = dict(d_model=c.d_model, eps=ar.rms_norm_eps, logits_in_fp32=ar.logits_in_fp32,
                      weighted_sum_in_fp32=ar.weighted_sum_in_fp32)
            pre_a = AttentionResidualSite(**kw, metadata=self._site_metadata(li, "pre_attention", kind, gi, pos))
            pre_f = AttentionResidualSite(**kw, metadata=self._site_metadata(li, "pre_ffn", kind, gi, pos))
        return HybridAttentionLayer(kind, attn, self._make_ffn() if include_ffn else None, c.d_model, c.rms_norm_eps,
                                    c.residual_dropout, layer_index=li, group_index=gi, position_in_group=pos,
                                    is_final_global=is_final_global, pre_attention_attnres=pre_a,
                                    pre_ffn_attnres=pre_f)

    def _site_metadata(self, layer_index, site_kind, attention_type=None, group_index=None, position_in_group=None):
        if site_kind == "final_output":
            return DepthSiteMetadata(2 * self.config.num_attention_layers, None, "final_output", None, None, None,
                                     None, None)
        site_index = 2 * layer_index + (0 if site_kind == "pre_attention" else 1)
        block = pos_in_block = None
        if self.attnres_config is not None and self.attnres_config.mode == "block":
            bs = self.attnres_config.resolved_sublayers_per_depth_block
            block, pos_in_block = site_index // bs, site_index % bs
        return DepthSiteMetadata(site_index, layer_index, site_kind, attention_type, group_index, position_in_group,
                                 block, pos_in_block)

    @property
    def layers(self) -> tuple:
        layers = tuple(layer for g in self.groups for layer in g.layers)
        if self.final_global_layer is not None:
            layers += (self.final_global_layer,)
        return layers

    @property
    def attention_types(self):
        return tuple(layer.attention_label for layer in self.layers)

    @property
    def depth_site_metadata(self):
        if self.final_output_attnres is None:
            return ()
        md = [s.metadata for layer in self.layers for s in (layer.pre_attention_attnres, layer.pre_ffn_attnres)]
        return tuple(md + [self.final_output_attnres.metadata])

    @property
    def _depth_block_sites(self) -> dict:
        grouped: dict = {}
        for layer in self.layers:
            for site in (layer.pre_attention_attnres, layer.pre_ffn_attnres):
                if site is not None:
                    grouped.setdefault(site.metadata.depth_block_index, []).append(site)
        return {k: tuple(v) for k, v in grouped.items()}

    def _validate_cache(self, cache, batch, mode):
        if mode == "full" and cache is not None:
            raise ValueError("full mode does not accept an external cache")
        if mode == "decode" and cache is None:
            raise ValueError("decode mode requires a non-empty cache")
        if cache is None:
            return
        if len(cache.layer_caches) != len(self.layers):
            raise ValueError("cache layer count must match backbone layer count")
        for layer, lc in zip(self.layers, cache.layer_caches):
            if lc.attention_type != layer.attention_type:
                raise ValueError("cache order/type does not match backbone")
            if tuple(lc.sequence_offsets.shape) != (batch,):
                raise ValueError("cache batch size must match hidden_states")

    def forward(self, hidden_states, attention_mask=None, cache=None, use_cache=False, mode="full",
                output_hidden_states=False, output_depth_weights=False, output_diagnostics=False,
                update_routing_bias=False) -> HybridBackboneOutput:
        b, _, mask = validate_backbone_inputs(hidden_states, attention_mask, self.config.d_model, mode)
        self._validate_cache(cache, b, mode)
        # Layers see ``None`` for an all-valid mask: mask-free fused kernels apply.
        all_valid = mask_all_valid() if not host_checks() else bool(mask.all())
        layer_mask = None if (not output_diagnostics and all_valid) else mask
        if self.config.depth_mixing == "standard":
            return self._forward_standard(hidden_states, layer_mask, mask, cache, use_cache, mode,
                                          output_hidden_states, output_diagnostics, update_routing_bias)
        return self._forward_attnres(hidden_states, layer_mask, mask, cache, use_cache, mode, output_hidden_states,
                                     output_depth_weights, output_diagnostics, update_routing_bias)

    def _make_cache(self, caches, prev=None, tokens: int = 0):
        if not host_checks():
            # sync-free (decode-graph capture): every row advanced by `tokens` valid tokens
            return HybridBackboneCache(tuple(caches), (prev.sequence_length if prev is not None else 0) + tokens)
        offsets = caches[0].sequence_offsets
        return HybridBackboneCache(tuple(caches), int(offsets.max().item()))

    def _forward_standard(self, x, layer_mask, mask, cache, use_cache, mode, output_hidden_states,
                          output_diagnostics, update_routing_bias):
        cursor, caches, states, diags = 0, [], ([x] if output_hidden_states else []), []
        out = x
        for g in self.groups:
            n = len(g.layers)
            go = g(out, layer_mask, None if cache is None else cache.layer_caches[cursor:cursor + n],
                   use_cache=use_cache, mode=mode, output_hidden_states=output_hidden_states,
                   output_diagnostics=output_diagnostics, update_routing_bias=update_routing_bias)
            out = go.hidden_states
            cursor += n
            if use_cache:
                caches.extend(go.layer_caches)
            if output_hidden_states:
                states.extend(go.hidden_states_by_layer)
            if output_diagnostics:
                diags.extend(go.diagnostics)
        if self.final_global_layer is not None:
            fo = self.final_global_layer(out, layer_mask, None if cache is None else cache.layer_caches[cursor],
                                         use_cache=use_cache, mode=mode, output_diagnostics=output_diagnostics,
                                         update_routing_bias=update_routing_bias)
            out = fo.hidden_states
            if use_cache:
                caches.append(fo.cache)
            if output_hidden_states:
                states.append(out)
            if output_diagnostics:
                diags.append(fo.diagnostics)
        out = self.final_norm(out)
        if output_hidden_states:
            states.append(out)
        bc = self._make_cache(caches, cache, x.shape[1]) if use_cache else None
        diagnostics = None
        if output_diagnostics:
            from .diagnostics import build_backbone_diagnostics
            diagnostics = build_backbone_diagnostics(tuple(diags), self, bc, x.device)
        return HybridBackboneOutput(out, bc, tuple(states) if output_hidden_states else None, diagnostics=diagnostics)

    def _forward_attnres(self, x, layer_mask, mask, cache, use_cache, mode, output_hidden_states,
                         output_depth_weights, output_diagnostics, update_routing_bias):
        ctrl = self.depth_controller
        state = ctrl.initialize(x)
        block_sites = self._depth_block_sites if isinstance(ctrl, BlockAttentionResidualController) else None
        rw = output_depth_weights or self.attnres_config.return_depth_weights
        rs = rw or output_diagnostics or self.attnres_config.return_depth_stats
        caches, diags, site_stats = [], [], []
        legacy = [x] if output_hidden_states else []
        pre_a, a_out, pre_f, f_out = [], [], [], []
        for i, layer in enumerate(self.layers):
            with nvtx(f"layer {i} {layer.attention_label}"):
                lo, mixes = layer.forward_attnres(ctrl, state, layer_mask,
                                                  None if cache is None else cache.layer_caches[i],
                                                  depth_block_sites=block_sites, use_cache=use_cache, mode=mode,
                                                  output_depth_weights=rw, output_depth_stats=rs,
                                                  output_diagnostics=output_diagnostics,
                                                  update_routing_bias=update_routing_bias)
            if use_cache:
                caches.append(lo.cache)
            if output_diagnostics:
                diags.append(lo.diagnostics)
            if rs:
                site_stats.extend((mixes[0].stats, mixes[1].stats))
            if output_hidden_states:
                pre_a.append(lo.pre_attention_state)
                a_out.append(lo.attention_output)
                pre_f.append(lo.pre_ffn_state)
                f_out.append(lo.ffn_output)
                legacy.extend((lo.attention_output, lo.ffn_output))
        fmix = ctrl.finalize(state, self.final_output_attnres, return_weights=rw, return_stats=rs)
        out = self.final_norm(fmix.mixed_state)
        if output_hidden_states:
            legacy.extend((fmix.mixed_state, out))
        bc = self._make_cache(caches, cache, x.shape[1]) if use_cache else None
        depth = None
        if rs:
            depth = self._depth_outputs(tuple(site_stats), fmix.stats, state, rw)
        diagnostics = None
        if output_diagnostics:
            from .diagnostics import build_backbone_diagnostics
            diagnostics = build_backbone_diagnostics(tuple(diags), self, bc, x.device)
            all_stats = tuple(site_stats) + (fmix.stats,)
            diagnostics["depth_mixing"] = self.config.depth_mixing
            diagnostics["mean_embedding_weight"] = torch.stack([s.embedding_weight for s in all_stats]).mean()
            diagnostics["mean_depth_entropy"] = torch.stack([s.weight_entropy for s in all_stats]).mean()
            diagnostics["mean_retrieval_distance"] = torch.stack([s.mean_retrieval_distance for s in all_stats]).mean()
            diagnostics["fraction_dominated_by_embedding"] = torch.stack(
                [(s.dominant_source_index == 0).float() for s in all_stats]).mean()
            diagnostics["fraction_dominated_by_most_recent"] = torch.stack(
                [(s.dominant_source_index == s.source_count - 1).float() for s in all_stats]).mean()
            diagnostics["num_depth_blocks"] = depth.num_depth_blocks
            diagnostics["partial_final_block_size"] = depth.partial_final_block_size
        trace = (BackboneHiddenStateTrace(x, tuple(pre_a), tuple(a_out), tuple(pre_f), tuple(f_out), fmix.mixed_state)
                 if output_hidden_states else None)
        return HybridBackboneOutput(out, bc, tuple(legacy) if output_hidden_states else None, trace, depth,
                                    diagnostics)

    def _depth_outputs(self, site_stats, final_stats, state, rw):
        all_stats = site_stats + (final_stats,)
        matrix = smask = labels = None
        if rw:
            matrix, smask = padded_weight_matrix(all_stats)
            rows = []
            for item in all_stats:
                if self.config.depth_mixing == "full":
                    rows.append(("embedding",) + tuple(f"sublayer_{s}" for s in range(1, item.source_count)))
                else:
                    done = item.number_of_completed_blocks or 0
                    row = ["embedding"] + [f"depth_block_{k}" for k in range(done)]
                    if item.source_count > 1 + done:
                        row.append("current_partial")
                    rows.append(tuple(row))
            labels = tuple(rows)
        if isinstance(state, FullAttentionResidualState):
            n, elems, peak, nblocks, partial, scans = len(state.sources), state.source_elements, len(state.sources), 0, 0, 0
        else:
            n = 1 + len(state.completed_blocks)
            elems, peak, nblocks = state.source_elements, n, len(state.completed_blocks)
            last = state.block_sizes[-1] if state.block_sizes else 0
            partial = last if last < state.sublayers_per_depth_block else 0
            scans = state.inter_block_scan_count
        return AttentionResidualBackboneOutput(self.config.depth_mixing, site_stats, final_stats, matrix, smask,
                                               labels, n, elems, peak, nblocks, partial, scans)


# --------------------------------------------------------------------------- KimiBlock
@dataclass(frozen=True)
class KimiBlockConfig:
    d_model: int
    num_pattern_repeats: int
    kda_config: KDAConfig
    mla_config: GatedMLAConfig
    stable_latent_moe_config: StableLatentMoEConfig
    attention_residual_config: AttentionResidualConfig
    attention_pattern: tuple = CANONICAL_ATTENTION_PATTERN
    add_final_gated_mla: bool = True
    rms_norm_eps: float = 1e-6
    residual_dropout: float = 0.0
    init_std: float = 0.02

    def __post_init__(self) -> None:
        object.__setattr__(self, "attention_pattern", tuple(self.attention_pattern))
        if self.d_model <= 0 or self.num_pattern_repeats <= 0 or not self.attention_pattern:
            raise ValueError("invalid KimiBlockConfig dimensions")
        if not self.add_final_gated_mla:
            raise ValueError("KimiBlock requires the final global Gated MLA")
        unknown = set(self.attention_pattern) - {"kda", "gated_mla"}
        if unknown:
            raise ValueError(f"unsupported attention types: {sorted(unknown)}")
        for name in ("kda_config", "mla_config", "stable_latent_moe_config", "attention_residual_config"):
            if getattr(self, name).d_model != self.d_model:
                raise ValueError(f"{name}.d_model must match d_model")
        if self.attention_residual_config.mode == "standard":
            raise ValueError("canonical KimiBlock requires Full or Block AttnRes")

    @property
    def num_pattern_layers(self) -> int:
        return self.num_pattern_repeats * len(self.attention_pattern)

    @property
    def num_transformer_layers(self) -> int:
        return self.num_pattern_layers + int(self.add_final_gated_mla)

    @property
    def num_kda_layers(self) -> int:
        return self.num_pattern_repeats * self.attention_pattern.count("kda")

    @property
    def num_mla_layers(self) -> int:
        return self.num_pattern_repeats * self.attention_pattern.count("gated_mla") + int(self.add_final_gated_mla)

    @property
    def num_moe_layers(self) -> int:
        return self.num_transformer_layers

    def to_backbone_config(self) -> HybridBackboneConfig:
        return HybridBackboneConfig(
            d_model=self.d_model, num_hybrid_groups=self.num_pattern_repeats, attention_pattern=self.attention_pattern,
            enforce_canonical_pattern=False, add_final_gated_mla=self.add_final_gated_mla,
            add_ffn_after_final_global=True, rms_norm_eps=self.rms_norm_eps, residual_dropout=self.residual_dropout,
            ffn_dropout=0.0, kda_config=self.kda_config, mla_config=self.mla_config, use_dense_ffn=False,
            channel_mixer_type="stable_latent_moe", stable_latent_moe_config=self.stable_latent_moe_config,
            init_std=self.init_std, attention_residual_config=self.attention_residual_config)

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "KimiBlockConfig":
        v = dict(values)
        v["kda_config"] = KDAConfig.from_dict(v["kda_config"])
        v["mla_config"] = GatedMLAConfig.from_dict(v["mla_config"])
        v["stable_latent_moe_config"] = StableLatentMoEConfig.from_dict(v["stable_latent_moe_config"])
        v["attention_residual_config"] = AttentionResidualConfig.from_dict(v["attention_residual_config"])
        v["attention_pattern"] = tuple(v["attention_pattern"])
        return cls(**v)


class KimiBlock(nn.Module):
    """Text backbone block (no embeddings, head or loss)."""

    def __init__(self, config: KimiBlockConfig):
        super().__init__()
        self.config = config
        self.backbone = HybridAttentionBackbone(config.to_backbone_config())

    @property
    def layers(self):
        return self.backbone.layers

    @property
    def attention_types(self):
        return self.backbone.attention_types

    @property
    def moe_layers(self):
        return tuple(layer.ffn for layer in self.layers)

    def forward(self, hidden_states, attention_mask=None, cache=None, use_cache=False, mode="full",
                output_hidden_states=False, output_depth_weights=False, output_diagnostics=False,
                update_routing_bias=False) -> HybridBackboneOutput:
        return self.backbone(hidden_states, attention_mask=attention_mask, cache=cache, use_cache=use_cache,
                             mode=mode, output_hidden_states=output_hidden_states,
                             output_depth_weights=output_depth_weights, output_diagnostics=output_diagnostics,
                             update_routing_bias=update_routing_bias)


__all__ = [
    "CANONICAL_ATTENTION_PATTERN", "HybridBackboneConfig", "HybridLayerCache", "HybridBackboneCache",
    "HybridLayerOutput", "HybridGroupOutput", "HybridBackboneOutput", "BackboneHiddenStateTrace", "DenseKimiFFN",
    "HybridAttentionLayer", "HybridAttentionGroup", "HybridAttentionBackbone", "KimiBlockConfig", "KimiBlock",
    "validate_backbone_inputs", "masked_norm_mean", "count_parameters",
]
