"""Stable LatentMoE: shared full-width experts + routed latent-width experts.

Parity targets (reference paths):
  * ``src/stable_latent_moe/config.py:10-104``   StableLatentMoEConfig
  * ``src/stable_latent_moe/router.py:13-109``   sigmoid router, biased top-k, unbiased weights
  * ``src/stable_latent_moe/dispatch.py:37-107`` reference / vectorised sparse dispatch
  * ``src/stable_latent_moe/module.py:106-279``  forward + Quantile Balancing lifecycle
  * ``src/stable_latent_moe/quantile_balancing.py:10-57``, ``histogram.py:11-138``

B200 layout: routed experts are stored stacked (``gate_proj``/``up_proj``
``[E,H,L]``, ``down_proj`` ``[E,L,H]``) so one grouped GEMM serves every expert;
state-dict hooks translate to and from the reference's per-expert key names
``routed_experts.{e}.transform.{gate,up,down}_proj.weight``.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Literal

import torch
import torch.nn as nn

from .. import ops as _ops
from .linear import Linear
from ..runtime import host_checks
from .primitives import RMSNorm, SiTUGLU, situ_glu_activation


@dataclass(frozen=True)
class StableLatentMoEConfig:
    d_model: int
    latent_dim: int
    num_shared_experts: int = 2
    num_routed_experts: int = 896
    routed_experts_per_token: int = 16
    shared_expert_hidden_dim: int = 3072
    routed_expert_hidden_dim: int = 3072
    beta_gate: float = 4.0
    beta_up: float = 25.0
    norm_eps: float = 1e-6
    router_eps: float = 1e-9
    router_bias: bool = False
    expert_bias: bool = False
    projection_bias: bool = False
    routing_backend: Literal["reference", "vectorized"] = "vectorized"
    quantile_backend: Literal["exact", "histogram"] = "exact"
    enable_quantile_balancing: bool = True
    router_logits_dtype: Literal["input", "float32"] = "float32"
    routing_weights_dtype: Literal["input", "float32"] = "float32"
    routed_accumulation_dtype: Literal["input", "float32"] = "float32"
    histogram_num_bins: int = 256
    histogram_min_margin: float = -2.0
    histogram_max_margin: float = 2.0
    return_router_diagnostics: bool = False
    init_std: float = 0.02

    def __post_init__(self) -> None:
        for name in ("d_model", "latent_dim", "num_routed_experts", "routed_experts_per_token",
                     "shared_expert_hidden_dim", "routed_expert_hidden_dim"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be > 0")
        if self.num_shared_experts < 1:
            raise ValueError("Kimi Stable LatentMoE requires shared experts")
        if self.routed_experts_per_token > self.num_routed_experts:
            raise ValueError("routed_experts_per_token must not exceed num_routed_experts")
        if self.enable_quantile_balancing and self.routed_experts_per_token >= self.num_routed_experts:
            raise ValueError("Quantile Balancing requires top_k < num_experts")
        for name in ("beta_gate", "beta_up", "norm_eps", "router_eps", "init_std"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be > 0")
        if self.routing_backend not in ("reference", "vectorized"):
            raise ValueError("unknown routing_backend")
        if self.quantile_backend not in ("exact", "histogram"):
            raise ValueError("unknown quantile_backend")
        for name in ("router_logits_dtype", "routing_weights_dtype", "routed_accumulation_dtype"):
            if getattr(self, name) not in ("input", "float32"):
                raise ValueError(f"unknown dtype policy for {name}")
        if self.histogram_num_bins < 2:
            raise ValueError("histogram_num_bins must be >= 2")
        if self.histogram_max_margin <= self.histogram_min_margin:
            raise ValueError("histogram_max_margin must exceed histogram_min_margin")

    @property
    def top_k(self) -> int:
        return self.routed_experts_per_token

    @classmethod
    def kimi_k3(cls) -> "StableLatentMoEConfig":
        return cls(d_model=7168, latent_dim=3584, num_shared_experts=2, num_routed_experts=896,
                   routed_experts_per_token=16, shared_expert_hidden_dim=3072, routed_expert_hidden_dim=3072)

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "StableLatentMoEConfig":
        return cls(**values)


def policy_dtype(input_dtype: torch.dtype, policy: str) -> torch.dtype:
    return torch.float32 if policy == "float32" and input_dtype in (torch.float16, torch.bfloat16) else input_dtype


# --------------------------------------------------------------------------- outputs
@dataclass
class RouterOutput:
    selected_experts: torch.Tensor
    selected_raw_scores: torch.Tensor
    selected_weights: torch.Tensor
    expert_load: torch.Tensor
    cutoff_k_plus_one: torch.Tensor | None = None
    routing_bias_before: torch.Tensor | None = None
    raw_logits: torch.Tensor | None = None
    raw_scores: torch.Tensor | None = None
    biased_scores: torch.Tensor | None = None
    routing_bias_after: torch.Tensor | None = None


@dataclass
class QuantileBalanceUpdate:
    next_bias: torch.Tensor
    target_quantile: float
    quantiles: torch.Tensor
    margin_min: torch.Tensor
    margin_max: torch.Tensor
    num_tokens: int


@dataclass
class StableLatentMoEOutput:
    hidden_states: torch.Tensor
    shared_output: torch.Tensor | None = None
    routed_output: torch.Tensor | None = None
    router_output: RouterOutput | None = None
    diagnostics: dict | None = None


# --------------------------------------------------------------------------- router
class TopKRouter(nn.Module):
    """Sigmoid router over the full-width input; biased dispatch, unbiased weights."""

    tie_policy = "lowest index wins among equal biased scores"

    def __init__(self, config: StableLatentMoEConfig):
        super().__init__()
        self.config = config
        self.projection = Linear(config.d_model, config.num_routed_experts, bias=config.router_bias)
        self.register_buffer("routing_bias", torch.zeros(config.num_routed_experts))
        nn.init.normal_(self.projection.weight, mean=0.0, std=config.init_std)
        if self.projection.bias is not None:
            nn.init.zeros_(self.projection.bias)

    @torch.no_grad()
    def commit_next_bias(self, next_bias: torch.Tensor) -> None:
        if next_bias.shape != self.routing_bias.shape:
            raise ValueError("next routing bias has an invalid shape")
        if host_checks() and not torch.isfinite(next_bias).all():
            raise ValueError("next routing bias must be finite")
        self.routing_bias.copy_(next_bias.to(device=self.routing_bias.device, dtype=self.routing_bias.dtype))

    def forward(self, inputs, *, need_qb_cutoff=False, return_full_scores=False, logits=None) -> RouterOutput:
        """``logits``: ``projection(inputs)`` already computed (by a fused projection group)."""
        c = self.config
        if inputs.ndim != 2 or inputs.shape[-1] != c.d_model:
            raise ValueError(f"router inputs must have shape [M,{c.d_model}]")
        if need_qb_cutoff and c.top_k >= c.num_routed_experts:
            raise ValueError("Top-(k+1) cutoff requires k < num_experts")
        if logits is None:
            logits = self.projection(inputs)
        cd = policy_dtype(inputs.dtype, c.router_logits_dtype)
        wd = policy_dtype(inputs.dtype, c.routing_weights_dtype)
        if _ops.use_kernels(logits) and cd == torch.float32 and wd == torch.float32:
            # One fused kernel: sigmoid, +bias, top-(k[+1]), renormalise, expert histogram.
            sel, raw_sel, weights, cutoff, load, raw = _ops.router_topk(
                logits, self.routing_bias, c.top_k, need_qb_cutoff, c.router_eps, return_full_scores)
            return RouterOutput(sel, raw_sel, weights, load, cutoff if need_qb_cutoff else None,
                                self.routing_bias.detach().clone(),
                                logits if return_full_scores else None, raw,
                                (raw + self.routing_bias) if return_full_scores else None)
        raw = torch.sigmoid(logits.to(cd))
        biased = raw + self.routing_bias.to(cd)
        top_values, top_indices = torch.topk(biased, k=c.top_k + int(need_qb_cutoff), dim=-1)
        sel = top_indices[:, : c.top_k]
        raw_sel = raw.gather(-1, sel)
        rw = raw_sel.to(wd)
        weights = rw / rw.sum(dim=-1, keepdim=True).clamp_min(c.router_eps)
        load = torch.bincount(sel.reshape(-1), minlength=c.num_routed_experts)
        return RouterOutput(sel, raw_sel, weights, load, top_values[:, c.top_k] if need_qb_cutoff else None,
                            self.routing_bias.detach().clone(), logits if return_full_scores else None,
                            raw if return_full_scores else None, biased if return_full_scores else None)


# --------------------------------------------------------------------------- experts
class SharedExpert(nn.Module):
    """Always-active full-width SiTU-GLU expert (``transform`` holds the weights)."""

    def __init__(self, width, hidden_dim, beta_gate, beta_up, bias, init_std):
        super().__init__()
        self.width, self.hidden_dim = width, hidden_dim
        self.transform = SiTUGLU(width, hidden_dim, beta_gate=beta_gate, beta_up=beta_up, bias=bias,
                                 output_bias=bias, init_std=init_std)

    def forward(self, inputs):
        if inputs.shape[-1] != self.width:
            raise ValueError(f"expert input must have shape [...,{self.width}]")
        return self.transform(inputs)


RoutedExpert = SharedExpert


# Decode batches route at most this many (token, slot) rows: every expert is then applied to
# every token with batched GEMMs and the unselected results get weight zero.  Reading all the
# expert weights once is what the sparse path costs too at this size (almost every expert is
# hit), and it needs no routing tables, no padding of expert segments and no host sync.
_DENSE_DECODE_ROWS = 128


def dense_small_batch_experts(latent, experts, selected, weights, accumulation_dtype):
    """``sum_slot w[t, slot] * expert_{e[t, slot]}(x_t)`` for a small token batch (inference)."""
    m = latent.shape[0]
    e = experts.gate_proj.shape[0]
    dense_w = torch.zeros(m, e, device=latent.device, dtype=accumulation_dtype)
    dense_w.scatter_add_(1, selected.long(), weights.to(accumulation_dtype))
    x = latent.unsqueeze(0).expand(e, m, latent.shape[1])
    g = torch.bmm(x, experts.gate_proj.transpose(1, 2))
    u = torch.bmm(x, experts.up_proj.transpose(1, 2))
    h = situ_glu_activation(g, u, experts.beta_gate, experts.beta_up)
    y = torch.bmm(h, experts.down_proj.transpose(1, 2))  # [E, m, L]
    return torch.einsum("me,eml->ml", dense_w, y.to(accumulation_dtype))


class GroupedRoutedExperts(nn.Module):
    """All routed SiTU-GLU experts as stacked weights for grouped GEMMs."""

    def __init__(self, num_experts: int, width: int, hidden_dim: int, beta_gate: float, beta_up: float,
                 init_std: float):
        super().__init__()
        self.num_experts, self.width, self.hidden_dim = num_experts, width, hidden_dim
        self.beta_gate, self.beta_up = float(beta_gate), float(beta_up)
        self.gate_proj = nn.Parameter(torch.empty(num_experts, hidden_dim, width))
        self.up_proj = nn.Parameter(torch.empty(num_experts, hidden_dim, width))
        self.down_proj = nn.Parameter(torch.empty(num_experts, width, hidden_dim))
        for p in (self.gate_proj, self.up_proj, self.down_proj):
            nn.init.normal_(p, mean=0.0, std=init_std)
        self._register_state_dict_hook(GroupedRoutedExperts._export_per_expert)
        self._register_load_state_dict_pre_hook(GroupedRoutedExperts._import_per_expert, with_module=True)

    def __len__(self) -> int:
        return self.num_experts

    _NAMES = ("gate_proj", "up_proj", "down_proj")

    @staticmethod
    def _export_per_expert(module, state_dict, prefix, local_metadata):
        for name in GroupedRoutedExperts._NAMES:
            key = prefix + name
            if key in state_dict:
                stacked = state_dict.pop(key)
                for e in range(stacked.shape[0]):
                    state_dict[f"{prefix}{e}.transform.{name}.weight"] = stacked[e]
        return state_dict

    def _import_per_expert(self, state_dict, prefix, local_metadata, strict, missing, unexpected, errors):
        for name in GroupedRoutedExperts._NAMES:
            keys = [f"{prefix}{e}.transform.{name}.weight" for e in range(self.num_experts)]
            if all(k in state_dict for k in keys):
                state_dict[prefix + name] = torch.stack([state_dict.pop(k) for k in keys])

    def expert_forward(self, e: int, x: torch.Tensor) -> torch.Tensor:
        dt = x.dtype
        if torch.is_autocast_enabled(x.device.type):
            dt = torch.get_autocast_dtype(x.device.type)
        xc = x.to(dt)
        g = xc @ self.gate_proj[e].to(dt).t()
        u = xc @ self.up_proj[e].to(dt).t()
        return situ_glu_activation(g, u, self.beta_gate, self.beta_up) @ self.down_proj[e].to(dt).t()


def vectorized_sparse_dispatch(latent, experts: GroupedRoutedExperts, selected_experts, selected_weights, *,
                               accumulation_dtype):
    """Sort assignments by expert, run each expert once, scatter-add weighted outputs."""
    m, l = latent.shape
    k = selected_experts.shape[1]
    flat_e = selected_experts.reshape(-1)
    flat_t = torch.arange(m, device=latent.device)[:, None].expand(m, k).reshape(-1)
    flat_w = selected_weights.reshape(-1)
    order = torch.argsort(flat_e, stable=True)
    se, st, sw = flat_e[order], flat_t[order], flat_w[order]
    counts = torch.bincount(se, minlength=experts.num_experts).tolist()
    agg = torch.zeros(m, l, device=latent.device, dtype=accumulation_dtype)
    start = 0
    for e, cnt in enumerate(counts):
        if cnt == 0:
            continue
        tok = st[start:start + cnt]
        out = experts.expert_forward(e, latent.index_select(0, tok))
        agg = agg.index_add(0, tok, out.to(accumulation_dtype) * sw[start:start + cnt, None].to(accumulation_dtype))
        start += cnt
    return agg


def reference_sparse_dispatch(latent, experts: GroupedRoutedExperts, selected_experts, selected_weights, *,
                              accumulation_dtype):
    """Token-by-token, slot-by-slot dispatch (oracle for the grouped path)."""
    m, l = latent.shape
    agg = torch.zeros(m, l, device=latent.device, dtype=accumulation_dtype)
    for t in range(m):
        for s in range(selected_experts.shape[1]):
            e = int(selected_experts[t, s])
            out = experts.expert_forward(e, latent[t:t + 1])
            agg = agg.index_add(0, torch.tensor([t], device=latent.device),
                                out.to(accumulation_dtype) * selected_weights[t, s].to(accumulation_dtype))
    return agg


# --------------------------------------------------------------------------- quantile balancing
class ExactQuantileBalancer:
    def __init__(self, num_experts: int, top_k: int):
        if num_experts <= 1 or not 1 <= top_k < num_experts:
            raise ValueError("exact balancing requires 1 <= k < n")
        self.num_experts, self.top_k = num_experts, top_k
        self.target_quantile = 1.0 - top_k / num_experts

    @torch.no_grad()
    def compute_next_bias(self, raw_scores, biased_cutoffs, old_bias) -> QuantileBalanceUpdate:
        if raw_scores.ndim != 2 or raw_scores.shape[1] != self.num_experts:
            raise ValueError("raw_scores must have shape [M,E]")
        cd = torch.float64 if raw_scores.dtype == torch.float64 else torch.float32
        margins = raw_scores.to(cd) - biased_cutoffs.to(cd)[:, None]
        q = torch.quantile(margins, self.target_quantile, dim=0, interpolation="linear")
        prov = -q
        return QuantileBalanceUpdate(prov - prov.mean(), self.target_quantile, q, margins.amin(0), margins.amax(0),
                                     raw_scores.shape[0])


class HistogramQuantileBalancer(nn.Module):
    """Bounded-memory per-expert margin histograms (counts are all-reducible)."""

    def __init__(self, num_experts, top_k, num_bins, min_margin, max_margin):
        super().__init__()
        if num_experts <= 1 or not 1 <= top_k < num_experts or num_bins < 2 or max_margin <= min_margin:
            raise ValueError("invalid histogram balancer configuration")
        self.num_experts, self.top_k, self.num_bins = num_experts, top_k, num_bins
        self.min_margin, self.max_margin = float(min_margin), float(max_margin)
        self.target_quantile = 1.0 - top_k / num_experts
        self.register_buffer("counts", torch.zeros(num_experts, num_bins, dtype=torch.int64), persistent=False)
        self.register_buffer("underflow", torch.zeros(num_experts, dtype=torch.int64), persistent=False)
        self.register_buffer("overflow", torch.zeros(num_experts, dtype=torch.int64), persistent=False)

    @property
    def bin_width(self) -> float:
        return (self.max_margin - self.min_margin) / self.num_bins

    @torch.no_grad()
    def reset(self) -> None:
        self.counts.zero_()
        self.underflow.zero_()
        self.overflow.zero_()

    @torch.no_grad()
    def accumulate(self, raw_scores, biased_cutoffs) -> None:
        if raw_scores.ndim != 2 or raw_scores.shape[1] != self.num_experts:
            raise ValueError("raw_scores must have shape [M,E]")
        if _ops.use_kernels(raw_scores):
            _ops.qb_histogram(raw_scores, biased_cutoffs, self.counts, self.underflow, self.overflow,
                              self.min_margin, self.max_margin)
            return
        margins = raw_scores.float() - biased_cutoffs.float()[:, None]
        self.underflow.add_((margins < self.min_margin).sum(0))
        self.overflow.add_((margins >= self.max_margin).sum(0))
        idx = torch.floor((margins - self.min_margin) / self.bin_width).long().clamp_(0, self.num_bins - 1)
        flat = idx + torch.arange(self.num_experts, device=margins.device)[None, :] * self.num_bins
        add = torch.bincount(flat.reshape(-1), minlength=self.num_experts * self.num_bins)
        self.counts.add_(add.reshape(self.num_experts, self.num_bins).to(self.counts.device))

    @torch.no_grad()
    def compute_next_bias(self, old_bias) -> QuantileBalanceUpdate:
        totals = self.counts.sum(-1)
        if host_checks() and torch.any(totals == 0):
            raise ValueError("each expert histogram requires at least one margin")
        ranks = self.target_quantile * (totals.float() - 1)
        lo_r, hi_r = ranks.floor().long(), ranks.ceil().long()
        cum = self.counts.cumsum(-1)
        lo_b = (cum > lo_r[:, None]).long().argmax(-1)
        hi_b = (cum > hi_r[:, None]).long().argmax(-1)
        cd = torch.float64 if old_bias.dtype == torch.float64 else torch.float32
        lo_v = self.min_margin + (lo_b.float() + 0.5) * self.bin_width
        hi_v = self.min_margin + (hi_b.float() + 0.5) * self.bin_width
        q = (lo_v + (ranks - lo_r) * (hi_v - lo_v)).to(cd)
        prov = -q
        return QuantileBalanceUpdate(prov - prov.mean(), self.target_quantile, q,
                                     torch.full_like(q, self.min_margin), torch.full_like(q, self.max_margin),
                                     int(totals[0].item()) if host_checks() else totals[0])


# --------------------------------------------------------------------------- module
class StableLatentMoE(nn.Module):
    """``out = sum_shared(x) + W_up RMSNorm(sum_k w_k E_k(W_down x))``; no router aux loss."""

    def __init__(self, config: StableLatentMoEConfig):
        super().__init__()
        self.config = c = config
        self.shared_experts = nn.ModuleList(
            SharedExpert(c.d_model, c.shared_expert_hidden_dim, c.beta_gate, c.beta_up, c.expert_bias, c.init_std)
            for _ in range(c.num_shared_experts))
        self.down_projection = Linear(c.d_model, c.latent_dim, bias=c.projection_bias)
        self.router = TopKRouter(c)
        if c.expert_bias:
            raise ValueError("biased routed experts are not supported by the grouped expert layout")
        self.routed_experts = GroupedRoutedExperts(c.num_routed_experts, c.latent_dim, c.routed_expert_hidden_dim,
                                                   c.beta_gate, c.beta_up, c.init_std)
        self.routed_aggregate_norm = RMSNorm(c.latent_dim, eps=c.norm_eps)
        self.up_projection = Linear(c.latent_dim, c.d_model, bias=c.projection_bias)
        self.exact_balancer = (ExactQuantileBalancer(c.num_routed_experts, c.top_k)
                               if c.enable_quantile_balancing else None)
        self.histogram_balancer = (HistogramQuantileBalancer(c.num_routed_experts, c.top_k, c.histogram_num_bins,
                                                             c.histogram_min_margin, c.histogram_max_margin)
                                   if c.enable_quantile_balancing and c.quantile_backend == "histogram" else None)
        self._balance_accumulating = False
        self._balance_old_bias = None
        self._balance_exact_scores: list = []
        self._balance_exact_cutoffs: list = []
        for proj in (self.down_projection, self.up_projection):
            nn.init.normal_(proj.weight, mean=0.0, std=c.init_std)
            if proj.bias is not None:
                nn.init.zeros_(proj.bias)

    @property
    def routing_bias(self):
        return self.router.routing_bias

    # ---- Quantile Balancing windows
    @torch.no_grad()
    def begin_balance_accumulation(self) -> None:
        if not self.training:
            raise RuntimeError("routing-bias accumulation is training-only")
        if not self.config.enable_quantile_balancing:
            raise RuntimeError("Quantile Balancing is disabled")
        if self._balance_accumulating:
            raise RuntimeError("balance accumulation is already active")
        if self.histogram_balancer is not None:
            self.histogram_balancer.reset()
        self._balance_old_bias = self.routing_bias.detach().clone()
        self._balance_exact_scores.clear()
        self._balance_exact_cutoffs.clear()
        self._balance_accumulating = True

    @torch.no_grad()
    def finalize_and_commit_balance(self, reducer=None, keep_old=None) -> QuantileBalanceUpdate:
        """Close the window; ``reducer`` (EP/DP) makes the statistics global first.

        ``keep_old`` (device bool scalar) keeps the previous bias when True: the step whose
        window this is was skipped by a device-side finite check (no host branch needed).
        """
        if not self._balance_accumulating:
            raise RuntimeError("balance accumulation is not active")
        if self.config.quantile_backend == "exact":
            if not self._balance_exact_scores:
                raise RuntimeError("cannot finalize an empty QB window")
            scores = torch.cat(self._balance_exact_scores, 0)
            cutoffs = torch.cat(self._balance_exact_cutoffs, 0)
            if reducer is not None:
                scores, cutoffs = reducer.gather_exact(scores, cutoffs)
            update = self.exact_balancer.compute_next_bias(scores, cutoffs, self._balance_old_bias)
        else:
            if reducer is not None:
                reducer.reduce_histogram(self.histogram_balancer)
            update = self.histogram_balancer.compute_next_bias(self._balance_old_bias)
        if keep_old is not None:
            update.next_bias = torch.where(keep_old, self._balance_old_bias.to(update.next_bias.dtype),
                                           update.next_bias)
        self.router.commit_next_bias(update.next_bias)
        self.discard_balance_accumulation()
        return update

    @torch.no_grad()
    def discard_balance_accumulation(self) -> None:
        if self.histogram_balancer is not None:
            self.histogram_balancer.reset()
        self._balance_exact_scores.clear()
        self._balance_exact_cutoffs.clear()
        self._balance_old_bias = None
        self._balance_accumulating = False

    def _update_balance(self, ro: RouterOutput, *, commit: bool):
        if self.config.quantile_backend == "exact":
            if self._balance_accumulating:
                self._balance_exact_scores.append(ro.raw_scores.detach())
                self._balance_exact_cutoffs.append(ro.cutoff_k_plus_one.detach())
                return None
            update = self.exact_balancer.compute_next_bias(ro.raw_scores, ro.cutoff_k_plus_one, ro.routing_bias_before)
            if commit:
                self.router.commit_next_bias(update.next_bias)
            return update
        self.histogram_balancer.accumulate(ro.raw_scores, ro.cutoff_k_plus_one)
        if self._balance_accumulating:
            return None
        update = self.histogram_balancer.compute_next_bias(ro.routing_bias_before)
        if commit:
            self.router.commit_next_bias(update.next_bias)
        self.histogram_balancer.reset()
        return update

    # ---- routed path (overridable by expert parallelism)
    def routed_aggregate(self, latent, ro: RouterOutput, accumulation_dtype):
        m, k = ro.selected_experts.shape
        if latent.is_cuda and not torch.is_grad_enabled() and m * k <= _DENSE_DECODE_ROWS:
            return dense_small_batch_experts(latent, self.routed_experts, ro.selected_experts, ro.selected_weights,
                                             accumulation_dtype)
        if (_ops.use_kernels(latent) and accumulation_dtype == torch.float32 and latent.shape[-1] % 64 == 0
                and self.config.routed_expert_hidden_dim % 128 == 0):
            return _ops.moe_grouped_experts(latent, ro.selected_experts, ro.selected_weights,
                                            self.routed_experts.gate_proj, self.routed_experts.up_proj,
                                            self.routed_experts.down_proj, self.config.beta_gate, self.config.beta_up)
        fn = reference_sparse_dispatch if self.config.routing_backend == "reference" else vectorized_sparse_dispatch
        return fn(latent, self.routed_experts, ro.selected_experts, ro.selected_weights,
                  accumulation_dtype=accumulation_dtype)

    def shared_forward(self, flat, projected=None):
        """``projected``: the experts' (gate, up) linear outputs from a fused projection group."""
        out = None
        for i, expert in enumerate(self.shared_experts):
            if projected is None:
                y = expert(flat)
            else:
                t = expert.transform
                g, u = projected[2 * i], projected[2 * i + 1]
                y = t.down_proj(situ_glu_activation(g, u, t.beta_gate, t.beta_up))
            out = y if out is None else out + y
        return out

    def projection_groups(self):
        """Weights that read the block input and run as one fused GEMM on CUDA: every shared expert's
        gate and up projections, the latent down-projection, then the router (the ragged last)."""
        ws = []
        for expert in self.shared_experts:
            ws += [expert.transform.gate_proj.weight, expert.transform.up_proj.weight]
        return [ws + [self.down_projection.weight, self.router.projection.weight]]

    def _fused_projections(self, flat):
        group = self.projection_groups()[0]
        biases = [self.down_projection.bias, self.router.projection.bias]
        for expert in self.shared_experts:
            biases += [expert.transform.gate_proj.bias, expert.transform.up_proj.bias]
        if (not _ops.use_kernels(flat) or any(b is not None for b in biases)
                or not _ops.linear_group_supported(flat, group)):
            return None
        return _ops.linear_group(flat, group)

    def forward(self, inputs, *, update_routing_bias=False, return_router_diagnostics=False,
                return_branch_outputs=False):
        c = self.config
        if inputs.ndim < 1 or inputs.shape[-1] != c.d_model:
            raise ValueError(f"inputs must have shape [...,{c.d_model}]")
        if update_routing_bias and not self.training:
            raise RuntimeError("routing bias cannot update during eval")
        shape = inputs.shape
        flat = inputs.reshape(-1, c.d_model)
        fused = self._fused_projections(flat)
        if fused is None:
            shared = self.shared_forward(flat)
            latent = self.down_projection(flat)
            router_logits = None
        else:
            shared = self.shared_forward(flat, fused[:-2])
            latent, router_logits = fused[-2], fused[-1]
        need_balance = update_routing_bias or self._balance_accumulating
        ro = self.router(flat, need_qb_cutoff=need_balance, return_full_scores=need_balance, logits=router_logits)
        acc = policy_dtype(latent.dtype, c.routed_accumulation_dtype)
        agg = self.routed_aggregate(latent, ro, acc)
        normalized = self.routed_aggregate_norm(agg).to(latent.dtype)
        routed = self.up_projection(normalized)
        hidden = (shared + routed).reshape(shape)
        if need_balance:
            update = self._update_balance(ro, commit=update_routing_bias and not self._balance_accumulating)
            if update is not None and update_routing_bias:
                ro.routing_bias_after = self.routing_bias.detach().clone()
        want_router = return_router_diagnostics or c.return_router_diagnostics
        if not (want_router or return_branch_outputs):
            return hidden
        diagnostics = None
        if want_router:
            from .diagnostics import build_moe_diagnostics
            diagnostics = build_moe_diagnostics(ro, c.num_shared_experts, shared, routed, agg, normalized)
        ro.raw_logits = ro.raw_scores = ro.biased_scores = None
        return StableLatentMoEOutput(hidden, shared.reshape(shape) if return_branch_outputs else None,
                                     routed.reshape(shape) if return_branch_outputs else None,
                                     ro if want_router else None, diagnostics)


__all__ = [
    "StableLatentMoEConfig", "RouterOutput", "QuantileBalanceUpdate", "StableLatentMoEOutput", "TopKRouter",
    "SharedExpert", "RoutedExpert", "GroupedRoutedExperts", "vectorized_sparse_dispatch", "reference_sparse_dispatch",
    "ExactQuantileBalancer", "HistogramQuantileBalancer", "StableLatentMoE", "policy_dtype",
]
