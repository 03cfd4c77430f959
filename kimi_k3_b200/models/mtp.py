"""Multi-token prediction head: ``h[t] (+) E[x_{t+1}] -> x_{t+2}`` through one 3KDA+1MLA block.

Parity targets (reference paths):
  * ``src/mtp/config.py``           KimiMTPConfig (exactly one MTP layer, future offset 2)
  * ``src/mtp/fusion.py:11-47``      RMSNorm(h) || RMSNorm(E) -> d x 2d projection
  * ``src/mtp/block.py:22-84``       local hybrid block with AttnRes and MoE
  * ``src/mtp/alignment.py:43-116``  training view and structural feature mask
  * ``src/mtp/head.py:28-339``       compaction of valid rows, shared LM head, draft step

Rows whose feature mask has holes are packed left with a cumulative-sum scatter
(vectorised; the reference loops over rows). Fully valid batches skip packing.
"""
from __future__ import annotations

import weakref
from dataclasses import asdict, dataclass

import torch
import torch.nn as nn

from ..runtime import host_checks, mask_all_valid
from .attnres import AttentionResidualConfig
from .backbone import (CANONICAL_ATTENTION_PATTERN, HybridAttentionBackbone, HybridBackboneConfig,
                       HybridBackboneOutput)
from .kda import KDAConfig
from .linear import Linear
from .losses import MultiTokenPredictionLoss
from .mla import GatedMLAConfig
from .moe import StableLatentMoEConfig
from .primitives import RMSNorm


@dataclass(frozen=True)
class KimiMTPConfig:
    d_model: int
    vocab_size: int
    kda_config: KDAConfig | None = None
    mla_config: GatedMLAConfig | None = None
    stable_latent_moe_config: StableLatentMoEConfig | None = None
    attention_residual_config: AttentionResidualConfig | None = None
    enabled: bool = True
    num_mtp_layers: int = 1
    future_offset: int = 2
    loss_weight: float = 0.1
    fusion_kind: str = "concat_project"
    normalize_hidden: bool = True
    normalize_future_embedding: bool = True
    fusion_bias: bool = False
    share_main_lm_head: bool = True
    detach_backbone_hidden: bool = False
    ignore_index: int = -100
    rms_norm_eps: float = 1e-6
    residual_dropout: float = 0.0
    init_std: float = 0.02
    return_logits_by_default: bool = True

    def __post_init__(self) -> None:
        if self.d_model <= 0 or self.vocab_size <= 0:
            raise ValueError("d_model and vocab_size must be > 0")
        if self.num_mtp_layers != 1:
            raise ValueError("Kimi K3 reports exactly one MTP layer")
        if self.future_offset != 2:
            raise ValueError("canonical Kimi MTP predicts exactly x[t+2]")
        if self.loss_weight < 0:
            raise ValueError("loss_weight must be >= 0")
        if self.fusion_kind != "concat_project":
            raise ValueError("only fusion_kind='concat_project' is supported")
        if not self.normalize_hidden or not self.normalize_future_embedding:
            raise ValueError("canonical MTP requires both fusion inputs normalized")
        if self.fusion_bias:
            raise ValueError("canonical MTP fusion is bias-free")
        if not self.share_main_lm_head:
            raise ValueError("canonical MTP shares the main LM head")
        if self.rms_norm_eps <= 0 or self.init_std <= 0 or not 0.0 <= self.residual_dropout < 1.0:
            raise ValueError("invalid MTP numerics")
        if not self.enabled:
            return
        for name in ("kda_config", "mla_config", "stable_latent_moe_config", "attention_residual_config"):
            cfg = getattr(self, name)
            if cfg is None:
                raise ValueError(f"{name} is required when MTP is enabled")
            if cfg.d_model != self.d_model:
                raise ValueError(f"{name}.d_model must match d_model")
        if self.attention_residual_config.mode == "standard":
            raise ValueError("Kimi MTP requires Full or Block AttnRes")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "KimiMTPConfig":
        v = dict(values)
        for name, typ in (("kda_config", KDAConfig), ("mla_config", GatedMLAConfig),
                          ("stable_latent_moe_config", StableLatentMoEConfig),
                          ("attention_residual_config", AttentionResidualConfig)):
            if isinstance(v.get(name), dict):
                v[name] = typ.from_dict(v[name])
        return cls(**v)


@dataclass(frozen=True)
class MTPTrainingView:
    source_hidden: torch.Tensor
    future_input_ids: torch.Tensor
    target_ids: torch.Tensor
    valid_mask: torch.Tensor


@dataclass
class MTPDiagnostics:
    valid_token_count: torch.Tensor
    token_accuracy: torch.Tensor
    mean_logit_entropy: torch.Tensor
    mean_hidden_norm: torch.Tensor
    hidden_rms: torch.Tensor
    fusion_output_rms: torch.Tensor
    block: dict | None = None


@dataclass
class KimiMTPOutput:
    logits: torch.Tensor | None
    loss: torch.Tensor | None
    hidden_states: torch.Tensor | None
    training_view: MTPTrainingView
    diagnostics: MTPDiagnostics | None = None


@dataclass
class MTPDraftOutput:
    logits: torch.Tensor
    cache: object
    hidden_states: torch.Tensor


_INT = (torch.int8, torch.int16, torch.int32, torch.int64, torch.uint8)


def build_mtp_training_view(last_hidden_state, input_ids, attention_mask=None, labels=None, segment_ids=None, *,
                            ignore_index=-100) -> MTPTrainingView:
    """h[t] with x[t+1] predicts targets[t+2]."""
    if last_hidden_state.ndim != 3:
        raise ValueError("last_hidden_state must have shape [B,T,D]")
    b, t, _ = last_hidden_state.shape
    if tuple(input_ids.shape) != (b, t) or input_ids.dtype not in _INT:
        raise ValueError(f"input_ids must be an integer tensor of shape {(b, t)}")
    mask = (torch.ones(b, t, dtype=torch.bool, device=last_hidden_state.device) if attention_mask is None
            else attention_mask)
    targets = input_ids if labels is None else labels
    if labels is not None and (tuple(labels.shape) != (b, t) or labels.dtype not in _INT):
        raise ValueError(f"labels must be an integer tensor of shape {(b, t)}")
    tgt = targets[:, 2:]
    valid = mask[:, :-2] & mask[:, 1:-1] & mask[:, 2:] & tgt.ne(ignore_index)
    if segment_ids is not None:
        valid = valid & segment_ids[:, :-2].eq(segment_ids[:, 1:-1]) & segment_ids[:, 1:-1].eq(segment_ids[:, 2:])
    return MTPTrainingView(last_hidden_state[:, :-2], input_ids[:, 1:-1], tgt, valid)


def build_mtp_feature_mask(attention_mask, input_ids):
    mask = torch.ones_like(input_ids, dtype=torch.bool) if attention_mask is None else attention_mask
    return mask[:, :-2] & mask[:, 1:-1] & mask[:, 2:]


class KimiMTPFusion(nn.Module):
    def __init__(self, d_model: int, eps: float = 1e-6, init_std: float = 0.02):
        super().__init__()
        self.d_model = d_model
        self.hidden_norm = RMSNorm(d_model, eps=eps)
        self.future_embedding_norm = RMSNorm(d_model, eps=eps)
        self.projection = Linear(2 * d_model, d_model, bias=False)
        nn.init.normal_(self.projection.weight, mean=0.0, std=init_std)

    def forward(self, source_hidden, future_embeddings):
        if source_hidden.ndim != 3 or source_hidden.shape[-1] != self.d_model:
            raise ValueError(f"source_hidden must have shape [B,T,{self.d_model}]")
        if future_embeddings.shape != source_hidden.shape:
            raise ValueError("future_embeddings must have the same shape as source_hidden")
        if source_hidden.dtype != future_embeddings.dtype:
            raise TypeError("fusion inputs must share dtype")
        return self.projection(torch.cat((self.hidden_norm(source_hidden),
                                          self.future_embedding_norm(future_embeddings)), dim=-1))


class KimiMTPBlock(nn.Module):
    """One (KDA, KDA, KDA, MLA) group with its own AttnRes and MoE layers."""

    def __init__(self, config: KimiMTPConfig):
        super().__init__()
        if not config.enabled:
            raise ValueError("cannot instantiate KimiMTPBlock when MTP is disabled")
        self.config = config
        self.backbone = HybridAttentionBackbone(HybridBackboneConfig(
            d_model=config.d_model, num_hybrid_groups=1, attention_pattern=CANONICAL_ATTENTION_PATTERN,
            enforce_canonical_pattern=False, add_final_gated_mla=False, add_ffn_after_final_global=True,
            rms_norm_eps=config.rms_norm_eps, residual_dropout=config.residual_dropout, ffn_dropout=0.0,
            kda_config=config.kda_config, mla_config=config.mla_config, use_dense_ffn=False,
            channel_mixer_type="stable_latent_moe", stable_latent_moe_config=config.stable_latent_moe_config,
            init_std=config.init_std, attention_residual_config=config.attention_residual_config))

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
        return self.backbone(hidden_states, attention_mask=attention_mask, cache=cache, use_cache=use_cache, mode=mode,
                             output_hidden_states=output_hidden_states, output_depth_weights=output_depth_weights,
                             output_diagnostics=output_diagnostics, update_routing_bias=update_routing_bias)


class KimiMTPHead(nn.Module):
    """Teacher-forced x[t+2] head sharing the model's embedding and LM head."""

    def __init__(self, config: KimiMTPConfig, input_embeddings: nn.Embedding, lm_head: nn.Linear, *,
                 register_shared_modules: bool = True):
        super().__init__()
        self.config = config
        if input_embeddings.embedding_dim != config.d_model or input_embeddings.num_embeddings != config.vocab_size:
            raise ValueError("input_embeddings dimensions do not match config")
        if lm_head.in_features != config.d_model or lm_head.out_features != config.vocab_size:
            raise ValueError("lm_head dimensions do not match config")
        self._register_shared_modules = register_shared_modules
        self.set_shared_modules(input_embeddings, lm_head)
        self.fusion = KimiMTPFusion(config.d_model, eps=config.rms_norm_eps, init_std=config.init_std) \
            if config.enabled else None
        self.block = KimiMTPBlock(config) if config.enabled else None
        self.loss_fn = MultiTokenPredictionLoss(ignore_index=config.ignore_index, zero_valid_policy="connected_zero")

    def set_shared_modules(self, input_embeddings, lm_head) -> None:
        if self._register_shared_modules:
            self._registered_input_embeddings = input_embeddings
            self._registered_lm_head = lm_head
        else:
            object.__setattr__(self, "_input_embeddings_ref", weakref.ref(input_embeddings))
            object.__setattr__(self, "_lm_head_ref", weakref.ref(lm_head))

    @property
    def input_embeddings(self) -> nn.Embedding:
        if self._register_shared_modules:
            return self._registered_input_embeddings
        m = self._input_embeddings_ref()
        if m is None:
            raise RuntimeError("shared input embeddings are no longer alive")
        return m

    @property
    def lm_head(self) -> nn.Linear:
        if self._register_shared_modules:
            return self._registered_lm_head
        m = self._lm_head_ref()
        if m is None:
            raise RuntimeError("shared LM head is no longer alive")
        return m

    def get_input_embeddings(self):
        return self.input_embeddings

    def get_output_embeddings(self):
        return self.lm_head

    def _run_compacted(self, fused, feature_mask, *, output_hidden_states, output_diagnostics, update_routing_bias):
        b, t, d = fused.shape
        if mask_all_valid() if not host_checks() else bool(feature_mask.all()):
            out = self.block(fused, attention_mask=None, output_hidden_states=output_hidden_states,
                             output_diagnostics=output_diagnostics, update_routing_bias=update_routing_bias)
            return out.last_hidden_state, out.diagnostics
        lengths = feature_mask.sum(1)
        active = torch.nonzero(lengths > 0, as_tuple=False).flatten()
        result = fused.new_zeros(b, t, d)
        if active.numel() == 0:
            return result, None
        fm = feature_mask[active]
        width = int(lengths[active].max().item())
        slot = torch.cumsum(fm.long(), 1) - 1
        rows = torch.arange(active.numel(), device=fused.device)[:, None].expand_as(slot)
        compact = fused.new_zeros(active.numel(), width, d)
        compact[rows[fm], slot[fm]] = fused[active][fm]
        cmask = torch.arange(width, device=fused.device)[None, :] < lengths[active][:, None]
        out = self.block(compact, attention_mask=cmask, output_hidden_states=output_hidden_states,
                         output_diagnostics=output_diagnostics, update_routing_bias=update_routing_bias)
        scattered = fused.new_zeros(active.numel(), t, d)
        scattered[fm] = out.last_hidden_state[rows[fm], slot[fm]]
        result = result.index_copy(0, active, scattered)
        return result, out.diagnostics

    def forward(self, last_hidden_state, input_ids, attention_mask=None, labels=None, compute_loss=True,
                segment_ids=None, return_logits=None, return_hidden_states=False, return_diagnostics=False,
                update_routing_bias=False) -> KimiMTPOutput:
        view = build_mtp_training_view(last_hidden_state, input_ids, attention_mask, labels, segment_ids,
                                       ignore_index=self.config.ignore_index)
        if not self.config.enabled:
            return KimiMTPOutput(None, None, None, view, None)
        if segment_ids is not None:
            m = torch.ones_like(segment_ids, dtype=torch.bool) if attention_mask is None else attention_mask
            for row_s, row_m in zip(segment_ids, m):
                if torch.unique(row_s[row_m]).numel() > 1:
                    raise ValueError("packed segment execution is not supported by the KDA/MLA cache")
        src = view.source_hidden.detach() if self.config.detach_backbone_hidden else view.source_hidden
        future = self.input_embeddings(view.future_input_ids)
        if future.dtype != src.dtype:
            future = future.to(src.dtype)  # bf16 residual stream under autocast
        fused = self.fusion(src, future)
        hidden, bdiag = self._run_compacted(fused, build_mtp_feature_mask(attention_mask, input_ids),
                                            output_hidden_states=return_hidden_states,
                                            output_diagnostics=return_diagnostics,
                                            update_routing_bias=update_routing_bias)
        keep = self.config.return_logits_by_default if return_logits is None else return_logits
        logits = self.lm_head(hidden) if (keep or (labels is not None and compute_loss) or return_diagnostics) else None
        loss = (self.loss_fn(logits, view.target_ids, mtp_loss_mask=view.valid_mask,
                             future_offsets=(self.config.future_offset,)).loss
                if labels is not None and compute_loss else None)
        diag = self._diagnostics(logits, hidden, fused, view, bdiag) if return_diagnostics else None
        return KimiMTPOutput(logits if keep else None, loss, hidden, view, diag)

    @staticmethod
    def _diagnostics(logits, hidden, fused, view, block):
        valid = view.valid_mask
        if torch.any(valid):
            sel = logits[valid].float()
            p = sel.softmax(-1)
            ent = -(p * p.clamp_min(torch.finfo(torch.float32).tiny).log()).sum(-1).mean()
            acc = (sel.argmax(-1) == view.target_ids[valid]).float().mean()
            hn = hidden.float().norm(dim=-1)[valid].mean()
            hr = hidden.float()[valid].square().mean().sqrt()
            fr = fused.float()[valid].square().mean().sqrt()
        else:
            ent = acc = hn = hr = fr = logits.detach().new_zeros((), dtype=torch.float32)
        return MTPDiagnostics(valid.sum().detach(), acc.detach(), ent.detach(), hn.detach(), hr.detach(), fr.detach(),
                              block)

    def draft_one_step(self, source_hidden_t, intermediate_token_id, cache=None) -> MTPDraftOutput:
        """Eval-only speculative draft of x[t+2] from h[t] and x[t+1]."""
        if not self.config.enabled:
            raise RuntimeError("MTP is disabled")
        if self.training:
            raise RuntimeError("draft_one_step is an eval-only API")
        if intermediate_token_id.ndim != 2 or intermediate_token_id.shape[1] != 1 or \
                intermediate_token_id.dtype not in _INT:
            raise ValueError("intermediate_token_id must be an integer tensor of shape [B,1]")
        if tuple(source_hidden_t.shape) != (intermediate_token_id.shape[0], 1, self.config.d_model):
            raise ValueError("source_hidden_t must have shape [B,1,D]")
        future = self.input_embeddings(intermediate_token_id)
        fused = self.fusion(source_hidden_t, future.to(source_hidden_t.dtype))
        out = self.block(fused, cache=cache, use_cache=True, mode="prefill" if cache is None else "decode")
        h = out.last_hidden_state
        return MTPDraftOutput(self.lm_head(h), out.cache, h)



def _unique_numel(*modules) -> int:
    seen, total = set(), 0
    for m in modules:
        if m is None:
            continue
        for prm in m.parameters():
            if id(prm) not in seen:
                seen.add(id(prm))
                total += prm.numel()
    return total


def mtp_parameter_counts(head: KimiMTPHead) -> dict:
    """Parameter counts of an MTP head with shared (aliased) tensors counted once.

    ``unique_mtp_total`` is what the head adds to the model (fusion + block); the
    embedding and LM head are shared with the main model. Parity:
    ``src/mtp/parameter_count.py:20-46`` (reference).
    """
    fusion = _unique_numel(head.fusion)
    block = _unique_numel(head.block)
    emb = _unique_numel(head.input_embeddings)
    lm = _unique_numel(head.lm_head)
    return {"fusion": fusion, "block": block, "unique_mtp_output": 0, "unique_mtp_total": fusion + block,
            "shared_input_embeddings": emb, "shared_lm_head": lm,
            "shared_embedding_lm_overlap": emb + lm - _unique_numel(head.input_embeddings, head.lm_head),
            "all_referenced_unique": _unique_numel(head.fusion, head.block, head.input_embeddings, head.lm_head)}

__all__ = [
    "KimiMTPConfig", "MTPTrainingView", "MTPDiagnostics", "KimiMTPOutput", "MTPDraftOutput",
    "build_mtp_training_view", "build_mtp_feature_mask", "KimiMTPFusion", "KimiMTPBlock", "KimiMTPHead",
    "mtp_parameter_counts",
]
