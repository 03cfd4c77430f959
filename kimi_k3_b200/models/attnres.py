"""Attention Residuals (AttnRes): softmax mixing over depth sources.

Parity targets (reference paths):
  * ``src/attention_residuals/config.py:11-122``        AttentionResidualConfig
  * ``src/attention_residuals/site.py:16-106``          pseudo-query site, RMSNorm keys, depth softmax
  * ``src/attention_residuals/block_attnres.py:22-159`` block controller lifecycle
  * ``src/attention_residuals/block_state.py:14-114``   embedding + completed blocks + partial sum
  * ``src/attention_residuals/full_attnres.py``, ``full_state.py``
  * ``src/attention_residuals/two_phase.py:13-85``, ``online_softmax.py:10-86``
  * ``src/attention_residuals/diagnostics.py``          per-site depth statistics

On CUDA a site is one fused kernel (:func:`kimi_k3_b200.ops.attnres_mix`) that
reads each source tensor once through a pointer list -- no ``torch.stack`` of the
sources -- computing the key RMS, the logit, an online softmax over depth and the
fp32 weighted sum in a single pass.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field
from typing import Literal

import torch
import torch.nn as nn

from .. import ops as _ops
from .primitives import RMSNorm


@dataclass(frozen=True)
class AttentionResidualConfig:
    d_model: int
    mode: Literal["standard", "full", "block"] = "block"
    rms_norm_eps: float = 1e-6
    query_init: Literal["zeros"] = "zeros"
    logits_in_fp32: bool = True
    weighted_sum_in_fp32: bool = True
    transformer_layers_per_depth_block: int | None = None
    sublayers_per_depth_block: int | None = 24
    target_num_depth_blocks: int | None = None
    add_final_output_mixer: bool = True
    include_embedding_source: bool = True
    backend: Literal["eager", "two_phase"] = "eager"
    return_depth_weights: bool = False
    return_depth_stats: bool = False

    def __post_init__(self) -> None:
        if self.d_model <= 0:
            raise ValueError("d_model must be > 0")
        if self.mode not in ("standard", "full", "block"):
            raise ValueError("mode must be 'standard', 'full', or 'block'")
        if self.rms_norm_eps <= 0:
            raise ValueError("rms_norm_eps must be > 0")
        if self.query_init != "zeros":
            raise ValueError("canonical Kimi AttnRes requires query_init='zeros'")
        if not self.include_embedding_source:
            raise ValueError("canonical Kimi AttnRes requires the embedding source")
        if not self.add_final_output_mixer:
            raise ValueError("canonical Kimi AttnRes requires a final output mixer")
        for name in ("transformer_layers_per_depth_block", "sublayers_per_depth_block", "target_num_depth_blocks"):
            v = getattr(self, name)
            if v is not None and v <= 0:
                raise ValueError(f"{name} must be > 0 when provided")
        if self.mode == "block":
            if self.transformer_layers_per_depth_block is None and self.sublayers_per_depth_block is None:
                raise ValueError("block mode requires a depth block size")
            if (self.transformer_layers_per_depth_block is not None and self.sublayers_per_depth_block is not None
                    and 2 * self.transformer_layers_per_depth_block != self.sublayers_per_depth_block):
                raise ValueError("transformer-layer and sublayer block sizes contradict")
        elif (self.transformer_layers_per_depth_block is not None or self.sublayers_per_depth_block is not None
              or self.target_num_depth_blocks is not None):
            raise ValueError("depth block sizes are only valid when mode='block'")
        if self.backend not in ("eager", "two_phase"):
            raise ValueError("backend must be 'eager' or 'two_phase'")
        if self.backend == "two_phase" and self.mode != "block":
            raise ValueError("two_phase backend is only defined for block mode")

    @property
    def resolved_sublayers_per_depth_block(self) -> int:
        if self.mode != "block":
            raise ValueError("only block mode has a depth block size")
        if self.sublayers_per_depth_block is not None:
            return self.sublayers_per_depth_block
        return 2 * self.transformer_layers_per_depth_block

    def num_depth_blocks(self, num_transformer_layers: int) -> int:
        if num_transformer_layers <= 0:
            raise ValueError("num_transformer_layers must be > 0")
        if self.mode != "block":
            return 0
        return math.ceil(2 * num_transformer_layers / self.resolved_sublayers_per_depth_block)

    def validate_topology(self, num_transformer_layers: int, *, every_layer_has_ffn: bool) -> None:
        if self.mode == "standard":
            return
        if not every_layer_has_ffn:
            raise ValueError("canonical AttnRes requires Attention and FFN in every transformer layer")
        if self.target_num_depth_blocks is not None:
            observed = self.num_depth_blocks(num_transformer_layers)
            if observed != self.target_num_depth_blocks:
                raise ValueError(f"target_num_depth_blocks does not match topology: expected "
                                 f"{self.target_num_depth_blocks}, observed {observed}")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "AttentionResidualConfig":
        return cls(**values)


@dataclass(frozen=True)
class DepthSiteMetadata:
    site_index: int
    transformer_layer_index: int | None
    site_kind: str
    attention_type: str | None
    hybrid_group_index: int | None
    position_in_hybrid_group: int | None
    depth_block_index: int | None
    position_in_depth_block: int | None


@dataclass
class DepthSoftmaxStats:
    max_logit: torch.Tensor
    exp_sum: torch.Tensor
    weighted_sum: torch.Tensor
    logits: torch.Tensor | None = None


@dataclass
class DepthAttentionStats:
    metadata: DepthSiteMetadata
    source_count: int
    weight_entropy: torch.Tensor
    normalized_entropy: torch.Tensor
    max_weight: torch.Tensor
    min_weight: torch.Tensor
    embedding_weight: torch.Tensor
    most_recent_source_weight: torch.Tensor
    dominant_source_index: torch.Tensor
    dominant_source_weight: torch.Tensor
    mean_weighted_source_index: torch.Tensor
    mean_retrieval_distance: torch.Tensor
    completed_block_weight_total: torch.Tensor | None = None
    current_partial_weight: torch.Tensor | None = None
    current_depth_block_index: int | None = None
    number_of_completed_blocks: int | None = None
    mean_weights: torch.Tensor | None = None


@dataclass
class AttentionResidualMixOutput:
    mixed_state: torch.Tensor
    weights: torch.Tensor | None = None
    logits: torch.Tensor | None = None
    stats: DepthAttentionStats | None = None


@dataclass
class AttentionResidualBackboneOutput:
    mode: str
    site_stats: tuple
    final_output_stats: DepthAttentionStats | None
    averaged_weight_matrix: torch.Tensor | None = None
    source_mask: torch.Tensor | None = None
    source_labels: tuple | None = None
    source_tensor_count: int = 0
    source_elements: int = 0
    peak_source_count: int = 0
    num_depth_blocks: int = 0
    partial_final_block_size: int = 0
    inter_block_scan_count: int = 0


def _acc(dtype, enabled):
    return torch.float32 if enabled and dtype in (torch.float16, torch.bfloat16) else dtype


def stack_sources(sources: list) -> torch.Tensor:
    if not sources:
        raise ValueError("source list must not be empty")
    shape = sources[0].shape
    if any(s.shape != shape for s in sources):
        raise ValueError("all depth sources must have identical [B,T,D] shapes")
    if any(s.dtype != sources[0].dtype for s in sources):
        raise TypeError("all depth sources must share dtype")
    return torch.stack(sources, dim=2)


def build_depth_attention_stats(weights, metadata, *, mode, number_of_completed_blocks=0, has_current_partial=False,
                                retain_mean_weights=False) -> DepthAttentionStats:
    p = weights.float()
    s = p.shape[-1]
    entropy = -(p * p.clamp_min(torch.finfo(torch.float32).tiny).log()).sum(-1).mean()
    normalized = entropy / math.log(s) if s > 1 else entropy.new_zeros(())
    mw = p.mean(dim=(0, 1))
    dom = mw.argmax()
    widx = (mw * torch.arange(s, dtype=torch.float32, device=p.device)).sum()
    dest = torch.tensor(float(metadata.site_index), device=p.device)
    completed = partial = None
    if mode == "block":
        completed = mw[1:1 + number_of_completed_blocks].sum()
        partial = mw[-1] if has_current_partial else mw.new_zeros(())
    return DepthAttentionStats(metadata, s, entropy, normalized, mw.max(), mw.min(), mw[0], mw[-1], dom, mw[dom], widx,
                               (dest - widx).abs(), completed, partial, metadata.depth_block_index,
                               number_of_completed_blocks if mode == "block" else None,
                               mw if retain_mean_weights else None)


def padded_weight_matrix(stats):
    rows = [s.mean_weights for s in stats]
    if not rows or any(r is None for r in rows):
        raise ValueError("mean weights were not retained")
    width = max(r.numel() for r in rows)
    mat = rows[0].new_zeros(len(rows), width)
    mask = torch.zeros(len(rows), width, dtype=torch.bool, device=mat.device)
    for i, r in enumerate(rows):
        mat[i, : r.numel()] = r
        mask[i, : r.numel()] = True
    return mat, mask


def depth_softmax_mix_reference(sources, pseudo_query, key_norm, *, logits_in_fp32=True, weighted_sum_in_fp32=True):
    """``softmax_s(q . RMSNorm(src_s)) weighted sum`` over ``[B,T,S,D]`` sources."""
    keys = key_norm(sources)
    ld = _acc(sources.dtype, logits_in_fp32)
    logits = torch.einsum("d,btsd->bts", pseudo_query.to(ld), keys.to(ld))
    weights = torch.softmax(logits, dim=-1)
    sd = _acc(sources.dtype, weighted_sum_in_fp32)
    mixed = torch.einsum("bts,btsd->btd", weights.to(sd), sources.to(sd)).to(sources.dtype)
    return mixed, weights, logits


class AttentionResidualSite(nn.Module):
    """One pseudo-query (init zeros) attending over preceding depth outputs."""

    def __init__(self, d_model: int, eps: float = 1e-6, logits_in_fp32: bool = True,
                 weighted_sum_in_fp32: bool = True, *, metadata: DepthSiteMetadata | None = None):
        super().__init__()
        if d_model <= 0:
            raise ValueError("d_model must be > 0")
        self.d_model = d_model
        self.logits_in_fp32, self.weighted_sum_in_fp32 = logits_in_fp32, weighted_sum_in_fp32
        self.metadata = metadata
        self.pseudo_query = nn.Parameter(torch.zeros(d_model))
        self.key_norm = RMSNorm(d_model, eps=eps)

    def mix_list(self, sources: list, *, return_weights=False, return_logits=False, return_stats=False,
                 mode="full", number_of_completed_blocks=0, has_current_partial=False) -> AttentionResidualMixOutput:
        """Mix a list of ``[B,T,D]`` sources (fused kernel on CUDA)."""
        need_w = return_weights or return_logits or return_stats
        if (not need_w and _ops.use_kernels(sources[0]) and self.logits_in_fp32 and self.weighted_sum_in_fp32):
            mixed = _ops.attnres_mix(sources, self.pseudo_query, self.key_norm.weight, self.key_norm.eps)
            return AttentionResidualMixOutput(mixed)
        return self(stack_sources(sources), return_weights=return_weights, return_logits=return_logits,
                    return_stats=return_stats, mode=mode, number_of_completed_blocks=number_of_completed_blocks,
                    has_current_partial=has_current_partial)

    def forward(self, sources, *, return_weights=False, return_logits=False, return_stats=False, mode="full",
                number_of_completed_blocks=0, has_current_partial=False) -> AttentionResidualMixOutput:
        if sources.ndim != 4 or sources.shape[-1] != self.d_model or sources.shape[2] == 0:
            raise ValueError(f"sources must have shape [B,T,S,{self.d_model}] with S > 0")
        mixed, weights, logits = depth_softmax_mix_reference(sources, self.pseudo_query, self.key_norm,
                                                             logits_in_fp32=self.logits_in_fp32,
                                                             weighted_sum_in_fp32=self.weighted_sum_in_fp32)
        stats = None
        if return_stats:
            if self.metadata is None:
                raise ValueError("metadata is required to build site diagnostics")
            stats = build_depth_attention_stats(weights, self.metadata, mode=mode,
                                                number_of_completed_blocks=number_of_completed_blocks,
                                                has_current_partial=has_current_partial,
                                                retain_mean_weights=return_weights)
        return AttentionResidualMixOutput(mixed, weights if return_weights else None,
                                          logits if return_logits else None, stats)


# --------------------------------------------------------------------------- online softmax helpers
def depth_softmax_stats(logits, values, *, weighted_sum_dtype=None) -> DepthSoftmaxStats:
    mx = logits.max(dim=-1).values
    ex = torch.exp(logits - mx[..., None])
    sd = weighted_sum_dtype or ex.dtype
    return DepthSoftmaxStats(mx, ex.sum(-1), torch.einsum("bts,btsd->btd", ex.to(sd), values.to(sd)), logits)


def single_source_stats(logit, value, *, weighted_sum_dtype=None) -> DepthSoftmaxStats:
    return DepthSoftmaxStats(logit, torch.ones_like(logit), value.to(weighted_sum_dtype or logit.dtype), logit[..., None])


def merge_depth_softmax_stats(a: DepthSoftmaxStats, b: DepthSoftmaxStats) -> DepthSoftmaxStats:
    mx = torch.maximum(a.max_logit, b.max_logit)
    sa, sb = torch.exp(a.max_logit - mx), torch.exp(b.max_logit - mx)
    logits = None if a.logits is None or b.logits is None else torch.cat((a.logits, b.logits), -1)
    return DepthSoftmaxStats(mx, sa * a.exp_sum + sb * b.exp_sum,
                             sa[..., None] * a.weighted_sum + sb[..., None] * b.weighted_sum, logits)


def normalize_depth_softmax_stats(stats: DepthSoftmaxStats, dtype) -> torch.Tensor:
    return (stats.weighted_sum / stats.exp_sum[..., None]).to(dtype)


def weights_from_stats(stats: DepthSoftmaxStats) -> torch.Tensor:
    return torch.exp(stats.logits - stats.max_logit[..., None]) / stats.exp_sum[..., None]


def precompute_inter_block_stats(sources, sites) -> dict:
    """Scan the completed blocks once for every site of a depth block."""
    eps = sites[0].key_norm.eps
    ld = _acc(sources.dtype, sites[0].logits_in_fp32)
    sd = _acc(sources.dtype, sites[0].weighted_sum_in_fp32)
    nd = torch.float32 if sources.dtype in (torch.float16, torch.bfloat16) else sources.dtype
    x = sources.to(nd)
    base = (x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps)).to(sources.dtype)
    queries = torch.stack([s.pseudo_query.to(ld) for s in sites])
    weights = torch.stack([s.key_norm.weight.to(sources.dtype) for s in sites])
    keys = (base.unsqueeze(0) * weights[:, None, None, None, :]).to(ld)
    logits = torch.einsum("pd,pbtsd->pbts", queries, keys)
    return {s.metadata.site_index: depth_softmax_stats(logits[i], sources, weighted_sum_dtype=sd)
            for i, s in enumerate(sites)}


def score_single_partial(partial, site) -> torch.Tensor:
    keys = site.key_norm(partial)
    cd = _acc(partial.dtype, site.logits_in_fp32)
    return torch.einsum("d,btd->bt", site.pseudo_query.to(cd), keys.to(cd))


# --------------------------------------------------------------------------- states + controllers
@dataclass
class BlockAttentionResidualState:
    embedding: torch.Tensor
    sublayers_per_depth_block: int
    completed_blocks: list = field(default_factory=list)
    partial_block: torch.Tensor | None = None
    outputs_in_current_block: int = 0
    total_sublayer_outputs: int = 0
    current_depth_block_index: int = 0
    block_sizes: list = field(default_factory=list)
    phase_stats: dict = field(default_factory=dict)
    prepared_depth_block_index: int | None = None
    inter_block_scan_count: int = 0

    def __post_init__(self) -> None:
        if self.embedding.ndim != 3:
            raise ValueError("embedding must have shape [B,T,D]")
        if self.sublayers_per_depth_block <= 0:
            raise ValueError("sublayers_per_depth_block must be > 0")
        if (self.partial_block is None) != (self.outputs_in_current_block == 0):
            raise ValueError("partial block/count invariant violated")

    @property
    def source_elements(self) -> int:
        ts = [self.embedding] + self.completed_blocks + ([self.partial_block] if self.partial_block is not None else [])
        return sum(t.numel() for t in ts)

    def prepare_for_site(self) -> None:
        if self.outputs_in_current_block == self.sublayers_per_depth_block:
            self.close_current_block()

    def source_list(self) -> list:
        self.prepare_for_site()
        out = [self.embedding] + self.completed_blocks
        if self.partial_block is not None:
            out.append(self.partial_block)
        return out

    def available_sources(self) -> torch.Tensor:
        return stack_sources(self.source_list())

    def completed_sources(self) -> torch.Tensor:
        self.prepare_for_site()
        return stack_sources([self.embedding] + self.completed_blocks)

    def append_output(self, output) -> None:
        if output.shape != self.embedding.shape:
            raise ValueError("all depth sources must have identical [B,T,D] shapes")
        if self.outputs_in_current_block == self.sublayers_per_depth_block:
            raise RuntimeError("close full block before appending another output")
        self.partial_block = output if self.partial_block is None else self.partial_block + output
        self.outputs_in_current_block += 1
        self.total_sublayer_outputs += 1

    def close_current_block(self) -> None:
        if self.partial_block is None:
            return
        self.completed_blocks.append(self.partial_block)
        self.block_sizes.append(self.outputs_in_current_block)
        self.partial_block = None
        self.outputs_in_current_block = 0
        self.current_depth_block_index += 1
        self.phase_stats.clear()
        self.prepared_depth_block_index = None

    def finalize(self) -> None:
        self.close_current_block()

    def clone(self, detach: bool = False) -> "BlockAttentionResidualState":
        cp = (lambda t: t.detach().clone()) if detach else (lambda t: t.clone())
        return BlockAttentionResidualState(cp(self.embedding), self.sublayers_per_depth_block,
                                           [cp(b) for b in self.completed_blocks],
                                           None if self.partial_block is None else cp(self.partial_block),
                                           self.outputs_in_current_block, self.total_sublayer_outputs,
                                           self.current_depth_block_index, list(self.block_sizes),
                                           inter_block_scan_count=self.inter_block_scan_count)


@dataclass
class FullAttentionResidualState:
    sources: list
    num_sublayer_outputs: int = 0

    def __post_init__(self) -> None:
        if not self.sources:
            raise ValueError("Full AttnRes state requires the embedding source")
        if len(self.sources) != 1 + self.num_sublayer_outputs:
            raise ValueError("Full AttnRes source count invariant violated")

    @property
    def embedding(self):
        return self.sources[0]

    @property
    def source_elements(self) -> int:
        return sum(s.numel() for s in self.sources)

    def source_list(self) -> list:
        return list(self.sources)

    def available_sources(self):
        return stack_sources(self.sources)

    def append_output(self, output) -> None:
        if output.shape != self.embedding.shape:
            raise ValueError("all depth sources must have identical [B,T,D] shapes")
        self.sources.append(output)
        self.num_sublayer_outputs += 1

    def clone(self, detach: bool = False) -> "FullAttentionResidualState":
        return FullAttentionResidualState([s.detach().clone() if detach else s.clone() for s in self.sources],
                                          self.num_sublayer_outputs)


class BlockAttentionResidualController(nn.Module):
    """initialize -> prepare -> mix -> append -> finalize over an explicit block state."""

    def __init__(self, sublayers_per_depth_block: int, backend: str = "eager"):
        super().__init__()
        if sublayers_per_depth_block <= 0 or backend not in ("eager", "two_phase"):
            raise ValueError("invalid block controller configuration")
        self.sublayers_per_depth_block, self.backend = sublayers_per_depth_block, backend

    def initialize(self, embedding) -> BlockAttentionResidualState:
        return BlockAttentionResidualState(embedding, self.sublayers_per_depth_block)

    def prepare_depth_block(self, state, sites) -> None:
        state.prepare_for_site()
        if self.backend != "two_phase" or _ops.use_kernels(state.embedding):
            return
        if state.prepared_depth_block_index == state.current_depth_block_index:
            return
        state.phase_stats = precompute_inter_block_stats(state.completed_sources(), sites)
        state.prepared_depth_block_index = state.current_depth_block_index
        state.inter_block_scan_count += 1

    def mix_for_site(self, site, state, *, return_weights=False, return_logits=False, return_stats=False):
        state.prepare_for_site()
        completed = len(state.completed_blocks)
        has_partial = state.partial_block is not None
        if self.backend == "eager" or _ops.use_kernels(state.embedding):
            return site.mix_list(state.source_list(), return_weights=return_weights, return_logits=return_logits,
                                 return_stats=return_stats, mode="block", number_of_completed_blocks=completed,
                                 has_current_partial=has_partial)
        idx = site.metadata.site_index
        if idx not in state.phase_stats:
            raise RuntimeError("two-phase depth block must be prepared before mixing")
        merged = state.phase_stats[idx]
        if has_partial:
            plogit = score_single_partial(state.partial_block, site)
            merged = merge_depth_softmax_stats(merged, single_source_stats(
                plogit, state.partial_block,
                weighted_sum_dtype=_acc(state.partial_block.dtype, site.weighted_sum_in_fp32)))
        mixed = normalize_depth_softmax_stats(merged, state.embedding.dtype)
        weights = weights_from_stats(merged) if (return_weights or return_stats) else None
        stats = None
        if return_stats:
            stats = build_depth_attention_stats(weights, site.metadata, mode="block",
                                                number_of_completed_blocks=completed, has_current_partial=has_partial,
                                                retain_mean_weights=return_weights)
        return AttentionResidualMixOutput(mixed, weights if return_weights else None,
                                          merged.logits if return_logits else None, stats)

    def append_output(self, state, output) -> None:
        state.append_output(output)

    def finalize(self, state, final_site, *, return_weights=False, return_logits=False, return_stats=False):
        state.finalize()
        return final_site.mix_list(state.source_list(), return_weights=return_weights, return_logits=return_logits,
                                   return_stats=return_stats, mode="block",
                                   number_of_completed_blocks=len(state.completed_blocks), has_current_partial=False)


class FullAttentionResidualController(nn.Module):
    def initialize(self, embedding) -> FullAttentionResidualState:
        if embedding.ndim != 3:
            raise ValueError("embedding must have shape [B,T,D]")
        return FullAttentionResidualState([embedding], 0)

    def prepare_depth_block(self, state, sites) -> None:
        return None

    def mix_for_site(self, site, state, *, return_weights=False, return_logits=False, return_stats=False):
        return site.mix_list(state.source_list(), return_weights=return_weights, return_logits=return_logits,
                             return_stats=return_stats, mode="full")

    def append_output(self, state, output) -> None:
        state.append_output(output)

    def finalize(self, state, final_site, *, return_weights=False, return_logits=False, return_stats=False):
        return self.mix_for_site(final_site, state, return_weights=return_weights, return_logits=return_logits,
                                 return_stats=return_stats)


__all__ = [
    "AttentionResidualConfig", "DepthSiteMetadata", "DepthSoftmaxStats", "DepthAttentionStats",
    "AttentionResidualMixOutput", "AttentionResidualBackboneOutput", "AttentionResidualSite",
    "depth_softmax_mix_reference", "build_depth_attention_stats", "padded_weight_matrix", "depth_softmax_stats",
    "single_source_stats", "merge_depth_softmax_stats", "normalize_depth_softmax_stats", "weights_from_stats",
    "precompute_inter_block_stats", "score_single_partial", "BlockAttentionResidualState",
    "FullAttentionResidualState", "BlockAttentionResidualController", "FullAttentionResidualController",
    "stack_sources",
]
