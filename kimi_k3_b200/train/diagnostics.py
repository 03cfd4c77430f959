"""Tiered training diagnostics: metric extraction, sampled update monitor, alerts.

Parity: ``training/diagnostics/{config,collector,alerts,reducers,*_metrics}.py`` (reference):
the same schedule (cheap / standard / deep every N steps), layer sampling with anchors and
rotation, time and persistent-memory budgets that degrade standard/deep steps to cheap ones,
metric names, and alert rules with patience.

B200 design: every metric is first a 0-d device tensor in a :class:`MetricBatch`; a
diagnostic step copies them to the host in ONE transfer (``torch.stack(...).tolist()``)
instead of one ``.item()`` per scalar (the reference issues hundreds of syncs per step).
The update monitor keeps its parameter samples in one flat device buffer.
"""
from __future__ import annotations

import math
import time
from collections import defaultdict
from dataclasses import asdict, dataclass
from typing import Literal

import torch


# --------------------------------------------------------------------------- config
@dataclass(frozen=True)
class DiagnosticsConfig:
    enabled: bool = True
    cheap_every_steps: int = 1
    standard_every_steps: int = 10
    deep_every_steps: int = 500
    sample_layers_per_standard_step: int = 8
    rotate_sampled_layers: bool = True
    sample_tokens_per_layer: int = 256
    sample_parameters_per_group: int = 16
    sample_elements_per_parameter: int = 256
    max_diagnostic_time_fraction: float = 0.05
    max_persistent_gpu_bytes: int = 16 * 1024 * 1024
    alert_patience_steps: int = 5

    def __post_init__(self) -> None:
        for name in ("cheap_every_steps", "standard_every_steps", "deep_every_steps",
                     "sample_layers_per_standard_step", "sample_tokens_per_layer", "sample_parameters_per_group",
                     "sample_elements_per_parameter", "alert_patience_steps"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if not 0 < self.max_diagnostic_time_fraction <= 1:
            raise ValueError("max_diagnostic_time_fraction must be in (0, 1]")
        if self.max_persistent_gpu_bytes < 0:
            raise ValueError("max_persistent_gpu_bytes must be non-negative")

    def level_for_step(self, step: int) -> str | None:
        if not self.enabled or step <= 0:
            return None
        if step % self.deep_every_steps == 0:
            return "deep"
        if step % self.standard_every_steps == 0:
            return "standard"
        if step % self.cheap_every_steps == 0:
            return "cheap"
        return None

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "DiagnosticsConfig":
        return cls(**values)


# --------------------------------------------------------------------------- metric batch
class MetricBatch:
    """name -> python float or 0-d tensor; :meth:`materialize` does one device-to-host copy."""

    def __init__(self):
        self.values: dict = {}

    def __setitem__(self, name, value):
        self.values[name] = value

    def __contains__(self, name):
        return name in self.values

    def update(self, other):
        self.values.update(other.values if isinstance(other, MetricBatch) else other)

    def materialize(self) -> dict:
        """Under sharded data parallelism a metric computed from a DTensor parameter is a DTensor;
        it is completed with its collective here, in insertion order, which every rank shares."""
        try:
            from torch.distributed.tensor import DTensor
        except ImportError:  # pragma: no cover
            DTensor = ()
        for k, v in list(self.values.items()):
            if isinstance(v, DTensor):
                self.values[k] = v.full_tensor()
        dev_names = [k for k, v in self.values.items() if torch.is_tensor(v)]
        out = {k: float(v) for k, v in self.values.items() if not torch.is_tensor(v)}
        if dev_names:
            by_dev = defaultdict(list)
            for k in dev_names:
                by_dev[self.values[k].device].append(k)
            for _, names in by_dev.items():
                vals = torch.stack([self.values[k].detach().float().reshape(()) for k in names]).tolist()
                out.update(zip(names, vals))
        return out


def t_rms(x: torch.Tensor) -> torch.Tensor:
    return x.detach().float().square().mean().sqrt()


def t_ratio(a, b, eps: float = 1e-12):
    if torch.is_tensor(a) or torch.is_tensor(b):
        b = torch.as_tensor(b, dtype=torch.float32)
        return a / b.abs().clamp_min(eps)
    return float(a / max(abs(b), eps))


def t_cosine(a, b, eps=1e-12):
    return torch.nn.functional.cosine_similarity(a.detach().float().reshape(-1), b.detach().float().reshape(-1),
                                                 dim=0, eps=eps)


# --------------------------------------------------------------------------- extractors
KDA_KEYS = {"alpha_mean": "alpha_mean", "alpha_std": "alpha_std", "alpha_min_sampled": "alpha_min",
            "alpha_max_sampled": "alpha_max", "fraction_alpha_near_lower_bound": "fraction_alpha_near_lower_bound",
            "fraction_alpha_near_one": "fraction_alpha_near_one", "beta_mean": "beta_mean", "beta_std": "beta_std",
            "fraction_beta_near_zero": "beta_saturation_low", "fraction_beta_near_one": "beta_saturation_high",
            "log_decay_mean": "log_decay_mean", "cumulative_log_decay_min": "cumulative_log_decay_min",
            "cumulative_log_decay_mean": "cumulative_log_decay_mean", "state_rms": "state_rms",
            "state_absmax": "state_absmax", "recurrent_output_rms": "recurrent_output_rms",
            "gated_output_rms": "gated_output_rms", "output_gate_mean": "output_gate_mean",
            "output_gate_saturation_low": "output_gate_saturation_low",
            "output_gate_saturation_high": "output_gate_saturation_high"}
MLA_KEYS = {"attention_entropy_normalized_sampled": "attention_entropy_normalized",
            "max_attention_probability_sampled": "attention_max_probability", "output_rms": "attention_output_rms",
            "gated_output_rms": "gated_output_rms", "output_gate_mean": "gate_mean",
            "output_gate_saturation_low": "gate_saturation_low", "output_gate_saturation_high": "gate_saturation_high",
            "q_rms": "q_rms", "k_rms": "k_rms", "v_rms": "v_rms", "qk_scale_max": "qk_scale_max"}


def _scalar_like(v):
    return v.detach().float().reshape(()) if torch.is_tensor(v) and v.numel() == 1 else (
        float(v) if isinstance(v, (int, float)) else None)


def kda_metrics(diag: dict, prefix: str = "kda") -> dict:
    if not diag:
        return {}
    out = {}
    for public, src in KDA_KEYS.items():
        if src in diag and _scalar_like(diag[src]) is not None:
            out[f"{prefix}/{public}"] = _scalar_like(diag[src])
    return out


def mla_metrics(diag: dict, *, qk_clip_active: bool = False, prefix: str = "mla") -> dict:
    if not diag:
        return {}
    out = {f"{prefix}/{public}": _scalar_like(diag[src]) for public, src in MLA_KEYS.items()
           if src in diag and _scalar_like(diag[src]) is not None}
    out[f"{prefix}/qk_clip_active"] = float(qk_clip_active)
    return out


def moe_metrics(d, prefix: str = "moe") -> dict:
    if d is None:
        return {}
    e = int(d.expert_load.numel())
    top_k = max(int(d.num_assignments / max(d.num_tokens, 1)), 1)
    mean = d.mean_load.float()
    ent = d.routing_entropy_over_selected.float()
    return {f"{prefix}/load_mean": mean, f"{prefix}/load_std": d.std_load.float(),
            f"{prefix}/load_cv": d.coefficient_of_variation.float(),
            f"{prefix}/load_max_to_mean": d.max_load.float() / mean.clamp_min(1e-12),
            f"{prefix}/load_min_to_mean": d.min_load.float() / mean.clamp_min(1e-12),
            f"{prefix}/dead_expert_fraction_batch": d.zero_load_experts.float() / max(e, 1),
            f"{prefix}/router_entropy_normalized": ent / (math.log(top_k) if top_k > 1 else 1.0),
            f"{prefix}/top1_share": d.selected_weight_max.float(), f"{prefix}/topk_weight_entropy": ent,
            f"{prefix}/qb_bias_mean": d.routing_bias_mean.float(), f"{prefix}/qb_bias_std": d.routing_bias_std.float(),
            f"{prefix}/qb_bias_absmax": torch.maximum(d.routing_bias_min.float().abs(), d.routing_bias_max.float().abs()),
            f"{prefix}/qb_update_rms": d.qb_update_rms.float(),
            f"{prefix}/qb_quantile_error_estimate": d.qb_quantile_error_estimate.float(),
            f"{prefix}/shared_output_rms": d.shared_output_rms.float(),
            f"{prefix}/routed_pre_norm_rms": d.routed_aggregate_rms_before_norm.float(),
            f"{prefix}/routed_post_norm_rms": d.routed_aggregate_rms_after_norm.float(),
            f"{prefix}/routed_up_projection_rms": d.routed_output_rms.float(),
            f"{prefix}/shared_to_total_ratio": d.shared_to_total_ratio.float(),
            f"{prefix}/routed_to_total_ratio": d.routed_to_total_ratio.float(),
            f"{prefix}/shared_routed_cosine": d.shared_routed_cosine.float(), f"{prefix}/output_rms": d.output_rms.float()}


def attnres_metrics(depth_output, prefix: str = "attnres") -> dict:
    if depth_output is None:
        return {}
    stats = tuple(getattr(depth_output, "site_stats", ())) + (getattr(depth_output, "final_output_stats", None),)
    stats = tuple(s for s in stats if s is not None)
    if not stats:
        return {}

    def mean(attr):
        vals = [getattr(s, attr).float().reshape(()) if torch.is_tensor(getattr(s, attr)) else
                torch.tensor(float(getattr(s, attr))) for s in stats if getattr(s, attr, None) is not None]
        return torch.stack([v.cpu() if v.device.type != vals[0].device.type else v for v in vals]).mean() \
            if vals else 0.0
    out = {f"{prefix}/source_entropy_normalized": mean("normalized_entropy"),
           f"{prefix}/max_source_weight": mean("max_weight"),
           f"{prefix}/embedding_source_weight": mean("embedding_weight"),
           f"{prefix}/current_block_partial_weight": mean("current_partial_weight"),
           f"{prefix}/top1_source_index_mean": mean("dominant_source_index")}
    ent = [torch.exp(s.weight_entropy.float()) for s in stats if getattr(s, "weight_entropy", None) is not None]
    if ent:
        out[f"{prefix}/effective_num_sources"] = torch.stack([e.reshape(()) for e in ent]).mean()
    cvs, oldest = [], []
    for s in stats:
        w = getattr(s, "mean_weights", None)
        if w is None:
            continue
        w = w.detach().float()
        cvs.append(w.std(unbiased=False) / w.mean().clamp_min(1e-12))
        done = getattr(s, "number_of_completed_blocks", max(w.numel() - 1, 0))
        oldest.append(w[1] if done is not None and done > 0 and w.numel() > 1 else w.new_zeros(()))
    out[f"{prefix}/source_weight_cv"] = torch.stack(cvs).mean() if cvs else 0.0
    out[f"{prefix}/oldest_block_weight"] = torch.stack(oldest).mean() if oldest else 0.0
    return out


def loss_metrics(*, total_loss, ntp_loss, mtp_loss, ntp_tokens, mtp_tokens, lambda_mtp=0.0) -> dict:
    out = {"train/loss_total": total_loss, "train/loss_ntp": ntp_loss,
           "train/perplexity_ntp_clipped": torch.exp(torch.as_tensor(ntp_loss).float().clamp(max=20.0)),
           "train/valid_ntp_tokens": ntp_tokens, "train/valid_mtp_tokens": mtp_tokens,
           "mtp/loss_weight": float(lambda_mtp)}
    if mtp_loss is not None:
        m = torch.as_tensor(mtp_loss).float()
        out.update({"train/loss_mtp": m, "mtp/loss": m, "mtp/perplexity_clipped": torch.exp(m.clamp(max=20.0)),
                    "mtp/valid_tokens": mtp_tokens,
                    "mtp/main_to_mtp_loss_ratio": torch.as_tensor(ntp_loss).float() / m.clamp_min(1e-12)})
    return out


def mtp_metrics(d, *, loss_weight: float = 0.0, prefix: str = "mtp") -> dict:
    if d is None:
        return {}
    out = {f"{prefix}/valid_tokens": d.valid_token_count, f"{prefix}/token_accuracy": d.token_accuracy,
           f"{prefix}/logit_entropy": d.mean_logit_entropy, f"{prefix}/hidden_rms": d.hidden_rms,
           f"{prefix}/hidden_norm_mean": d.mean_hidden_norm, f"{prefix}/fusion_output_rms": d.fusion_output_rms,
           f"{prefix}/loss_weight": float(loss_weight)}
    ratios = []
    for layer in (d.block or {}).get("layers", ()):
        inp = layer.get("input_norm", layer.get("pre_attention_depth_norm"))
        br = layer.get("attention_output_norm")
        if inp is not None and br is not None:
            ratios.append(torch.as_tensor(br).float() / torch.as_tensor(inp).float().abs().clamp_min(1e-12))
    if ratios:
        out[f"{prefix}/block_branch_to_input_rms"] = torch.stack([r.reshape(()) for r in ratios]).mean()
    return out


def block_contribution(inp, branch, outp, *, prefix: str) -> dict:
    ir = t_rms(inp)
    return {f"{prefix}/branch_to_input_rms": t_rms(branch) / ir.clamp_min(1e-12),
            f"{prefix}/state_change_ratio": t_rms(outp.detach() - inp.detach()) / ir.clamp_min(1e-12),
            f"{prefix}/branch_input_cosine": t_cosine(branch, inp), f"{prefix}/output_rms": t_rms(outp),
            f"{prefix}/output_absmax": outp.detach().float().abs().max(),
            f"{prefix}/output_zero_fraction": (outp.detach() == 0).float().mean()}


def representation_metrics(hidden, *, max_tokens: int = 256, prefix: str = "representation") -> dict:
    s = hidden.detach().reshape(-1, hidden.shape[-1])[:max_tokens].float()
    if s.numel() == 0:
        return {}
    var = s.var(dim=0, unbiased=False)
    centered = s - s.mean(dim=-1, keepdim=True)
    if s.shape[0] > 1:
        n = torch.nn.functional.normalize(centered, dim=-1)
        cos = (n[:-1] * n[1:]).sum(-1)
        cm, cs = cos.mean(), cos.std(unbiased=False)
    else:
        cm = cs = 0.0
    return {f"{prefix}/rms": t_rms(s), f"{prefix}/feature_mean_abs": s.mean(0).abs().mean(),
            f"{prefix}/feature_std_mean": var.sqrt().mean(), f"{prefix}/dead_feature_fraction": (var <= 1e-12).float().mean(),
            f"{prefix}/token_cosine_mean_sampled": cm, f"{prefix}/token_cosine_std_sampled": cs,
            f"{prefix}/effective_variance_ratio_proxy": var.mean() / var.max().clamp_min(1e-12)}


def activation_metrics(x, *, max_elements: int = 8192, prefix: str = "activation") -> dict:
    v = x.detach().reshape(-1)[:max_elements].float()
    if v.numel() == 0:
        return {}
    ok = torch.isfinite(v)
    f = torch.where(ok, v, torch.zeros_like(v))
    return {f"{prefix}/rms": t_rms(f), f"{prefix}/mean": f.mean(), f"{prefix}/std": f.std(unbiased=False),
            f"{prefix}/absmax": f.abs().max(), f"{prefix}/zero_fraction": (f == 0).float().mean(),
            f"{prefix}/nonfinite_fraction": (~ok).float().mean()}


def vision_metrics(vision_outputs, meta, *, prefix: str = "vision") -> dict:
    if vision_outputs is None:
        return {}
    out = {}
    for name in ("images", "videos"):
        o = getattr(vision_outputs, name, None)
        if o is None:
            continue
        h = o.last_hidden_state
        out[f"{prefix}/{name}_hidden_rms"] = t_rms(h)
        out[f"{prefix}/{name}_hidden_absmax"] = h.detach().float().abs().max()
        out[f"{prefix}/{name}_items"] = float(h.shape[0])
    if meta is not None:
        for name in ("image_token_counts", "video_token_counts"):
            v = getattr(meta, name, None)
            if v is not None:
                out[f"{prefix}/{name}_total"] = v.sum().float()
                out[f"{prefix}/{name}_mean"] = v.float().mean()
    return out


# --------------------------------------------------------------------------- update monitor
def diagnostic_family(spec) -> str:
    name = spec.parameter_name.lower()
    role = getattr(spec, "role", "")
    if name.startswith("mtp.") or ".mtp." in name:
        return "mtp"
    table = {"embedding": "embeddings", "attention_q": "attention_qkv", "attention_k": "attention_qkv",
             "attention_v": "attention_qkv", "attention_o": "attention_output", "moe_router": "moe_router",
             "moe_shared_expert": "moe_shared_experts", "moe_routed_expert": "moe_routed_experts",
             "mtp_matrix": "mtp", "lm_head": "lm_head", "norm": "norms"}
    if role in table:
        return table[role]
    if "attnres" in name or "pseudo_query" in name:
        return "attnres"
    if ".attention." in name and "kda" in name:
        return "kda_internal"
    return "other"


class ParameterUpdateMonitor:
    """Samples the first ``max_elements`` entries of up to ``max_parameters`` tensors per
    family; before/after the optimizer step, all statistics stay on the device."""

    def __init__(self, specs, *, max_parameters_per_group: int = 16, max_elements_per_parameter: int = 256):
        self.specs = tuple(specs)
        self.max_parameters_per_group = int(max_parameters_per_group)
        self.max_elements_per_parameter = int(max_elements_per_parameter)
        self.before: dict = {}
        self.sampled = []
        self.persistent_bytes = 0

    def _grouped(self):
        g = defaultdict(list)
        for s in self.specs:
            g[diagnostic_family(s)].append(s)
        return g

    @torch.no_grad()
    def capture_before_step(self) -> dict:
        self.before.clear()
        self.sampled.clear()
        self.persistent_bytes = 0
        grouped = self._grouped()
        out = {}
        sums, counts, zero, nonfin, missing = {}, {}, {}, {}, {}
        for fam, specs in grouped.items():
            sq, cnt, zc, nf, miss = [], 0, [], [], 0
            for spec in specs[: self.max_parameters_per_group]:
                p = spec.parameter
                sample = p.detach().reshape(-1)[: self.max_elements_per_parameter].float().clone()
                self.before[spec.parameter_name] = sample
                self.sampled.append(spec)
                self.persistent_bytes += sample.numel() * sample.element_size()
                if p.grad is None:
                    miss += 1
                    continue
                gs = p.grad.detach().reshape(-1)[: self.max_elements_per_parameter].float()
                nf.append((~torch.isfinite(gs)).sum())
                fin = torch.nan_to_num(gs)
                sq.append(fin.square().sum())
                zc.append((fin == 0).sum())
                cnt += fin.numel()
            dev = specs[0].parameter.device
            sums[fam] = torch.stack(sq).sum() if sq else torch.zeros((), device=dev)
            counts[fam] = cnt
            zero[fam] = torch.stack(zc).sum().float() if zc else torch.zeros((), device=dev)
            nonfin[fam] = torch.stack(nf).sum().float() if nf else torch.zeros((), device=dev)
            missing[fam] = miss
            out[f"optimizer/{fam}/grad_rms"] = (sums[fam] / cnt).sqrt() if cnt else 0.0
            out[f"optimizer/{fam}/zero_grad_fraction"] = zero[fam] / cnt if cnt else 0.0
            out[f"optimizer/{fam}/nonfinite_grad_count"] = nonfin[fam]
            out[f"optimizer/{fam}/grad_none_tensors"] = float(miss)
        tot_c = sum(counts.values())
        if tot_c:
            devs = [v for v in sums.values()]
            out["train/gradient_rms_global_sampled"] = (torch.stack([d.to(devs[0].device) for d in devs]).sum()
                                                        / tot_c).sqrt()
        else:
            out["train/gradient_rms_global_sampled"] = 0.0
        if "mtp" in grouped:
            main = [f for f in grouped if f != "mtp"]
            mc = sum(counts[f] for f in main)
            main_rms = (torch.stack([sums[f] for f in main]).sum() / mc).sqrt() if mc else torch.zeros(())
            mtp_rms = out["optimizer/mtp/grad_rms"]
            out["mtp/gradient_rms"] = mtp_rms
            out["mtp/main_to_mtp_grad_ratio"] = main_rms / torch.as_tensor(mtp_rms).clamp_min(1e-12)
        return out

    @torch.no_grad()
    def capture_after_step(self) -> dict:
        upd, par, cnt = defaultdict(list), defaultdict(list), defaultdict(int)
        for spec in self.sampled:
            fam = diagnostic_family(spec)
            after = spec.parameter.detach().reshape(-1)[: self.max_elements_per_parameter].float()
            before = self.before[spec.parameter_name]
            upd[fam].append((after - before).square().sum())
            par[fam].append(after.square().sum())
            cnt[fam] += after.numel()
        out = {}
        tu, tp, tc = [], [], 0
        for fam, c in cnt.items():
            u, p = torch.stack(upd[fam]).sum(), torch.stack(par[fam]).sum()
            ur, pr = (u / c).sqrt(), (p / c).sqrt()
            out[f"optimizer/{fam}/parameter_rms"] = pr
            out[f"optimizer/{fam}/update_rms"] = ur
            out[f"optimizer/{fam}/update_to_parameter_ratio"] = ur / pr.clamp_min(1e-12)
            if fam == "mtp":
                out["mtp/update_rms"] = ur
                out["mtp/update_to_parameter_ratio"] = ur / pr.clamp_min(1e-12)
            tu.append(u)
            tp.append(p)
            tc += c
        if tc:
            gu, gp = (torch.stack(tu).sum() / tc).sqrt(), (torch.stack(tp).sum() / tc).sqrt()
            out.update({"train/parameter_norm_global_sampled": gp, "train/update_norm_global_sampled": gu,
                        "train/update_to_parameter_ratio_sampled": gu / gp.clamp_min(1e-12)})
        out["diagnostics/persistent_gpu_bytes"] = float(self.persistent_bytes)
        self.before.clear()
        self.sampled.clear()
        self.persistent_bytes = 0
        return out


# --------------------------------------------------------------------------- alerts
@dataclass(frozen=True)
class DiagnosticAlert:
    severity: Literal["info", "warning", "critical"]
    code: str
    message: str
    step: int
    metric_name: str
    observed_value: float
    reference_value: float | None
    patience_count: int

    def to_dict(self) -> dict:
        return asdict(self)


# (metric, predicate, code, message, severity, immediate, reference)
ALERT_RULES = (
    ("train/loss_total", lambda v: not math.isfinite(v), "NONFINITE_LOSS", "training loss is non-finite", "critical",
     True, None),
    ("diagnostics/budget_exceeded", lambda v: v > 0.5, "DIAGNOSTIC_BUDGET_EXCEEDED",
     "diagnostics exceeded the configured time or memory budget", "info", True, 0.0),
    ("block/branch_to_input_rms", lambda v: v < 1e-3, "INACTIVE_BLOCK",
     "a residual branch contribution is persistently negligible", "warning", False, 1e-3),
    ("attnres/source_entropy_normalized", lambda v: v < 0.05, "ATTNRES_SINGLE_SOURCE_COLLAPSE",
     "Attention Residuals collapsed to one depth source", "warning", False, 0.05),
    ("attnres/source_entropy_normalized", lambda v: v > 0.995, "ATTNRES_UNIFORM_COLLAPSE",
     "Attention Residuals remain nearly uniform across sources", "info", False, 0.995),
    ("kda/fraction_alpha_near_one", lambda v: v > 0.95, "KDA_RETENTION_SATURATION",
     "KDA decay is persistently near full retention", "warning", False, 0.95),
    ("kda/fraction_beta_near_zero", lambda v: v > 0.95, "KDA_STATE_WRITE_CLOSED",
     "KDA state writes are persistently closed", "warning", False, 0.95),
    ("kda/state_growth_ratio", lambda v: v > 2.0, "KDA_STATE_EXPLOSION", "KDA recurrent state RMS is growing abruptly",
     "warning", False, 2.0),
    ("moe/dead_expert_fraction_batch", lambda v: v > 0.5, "MOE_DEAD_EXPERTS_PERSISTENT",
     "more than half of routed experts are unused", "warning", False, 0.5),
    ("moe/routed_to_total_ratio", lambda v: v < 1e-3, "MOE_ROUTED_BRANCH_INACTIVE",
     "routed expert branch is negligible", "warning", False, 1e-3),
    ("kda/output_gate_saturation_low", lambda v: v > 0.95, "KDA_OUTPUT_GATE_CLOSED",
     "KDA output gate is persistently closed", "warning", False, 0.95),
    ("mla/output_gate_saturation_low", lambda v: v > 0.95, "MLA_OUTPUT_GATE_CLOSED",
     "MLA output gate is persistently closed", "warning", False, 0.95),
    ("qk_clip/fraction_layers_clipped", lambda v: v > 0.5, "QK_CLIP_PERSISTENT",
     "QK-Clip is active in most attention layers", "warning", False, 0.5),
    ("optimizer/mtp/grad_rms", lambda v: v <= 1e-12, "MTP_DISCONNECTED",
     "MTP parameters receive no measurable sampled gradient", "warning", False, 1e-12),
    ("mtp/valid_tokens", lambda v: v <= 0, "MTP_NO_VALID_TOKENS", "MTP repeatedly receives no valid target tokens",
     "warning", False, 0.0),
    ("representation/dead_feature_fraction", lambda v: v > 0.9, "REPRESENTATION_VARIANCE_COLLAPSE",
     "most sampled representation features have zero variance", "warning", False, 0.9),
)


class AlertManager:
    """Rules with patience over host scalars; a rule named ``family/metric`` also matches
    every ``family/<layer>/metric`` instance."""

    def __init__(self, patience_steps: int = 5, ema_decay: float = 0.95):
        if patience_steps <= 0 or not 0 <= ema_decay < 1:
            raise ValueError("invalid alert manager configuration")
        self.patience_steps = int(patience_steps)
        self.ema_decay = float(ema_decay)
        self.baselines: dict = {}
        self.counts: dict = {}

    @staticmethod
    def _matches(rule_name: str, key: str) -> bool:
        fam, leaf = rule_name.split("/", 1)[0], rule_name.rsplit("/", 1)[-1]
        return key == rule_name or (key.startswith(fam + "/") and key.endswith("/" + leaf))

    def evaluate(self, metrics: dict, step: int) -> tuple:
        alerts = []
        for name, value in metrics.items():
            value = float(value)
            if not math.isfinite(value):
                alerts.append(DiagnosticAlert("critical", "NONFINITE_METRIC", f"{name} is non-finite", step, name,
                                              value, None, 1))
                continue
            prev = self.baselines.get(name, value)
            self.baselines[name] = self.ema_decay * prev + (1 - self.ema_decay) * value
        for name, pred, code, msg, sev, immediate, ref in ALERT_RULES:
            cands = {k: float(v) for k, v in metrics.items() if self._matches(name, k)}
            if not cands:
                continue
            active = [(k, v) for k, v in cands.items() if pred(v)]
            self.counts[code] = self.counts.get(code, 0) + 1 if active else 0
            if self.counts[code] < (1 if immediate else self.patience_steps):
                continue
            metric, value = active[0] if active else next(iter(cands.items()))
            alerts.append(DiagnosticAlert(sev, code, msg, step, metric, value, ref, self.counts[code]))
        return tuple(alerts)

    def state_dict(self) -> dict:
        return {"patience_steps": self.patience_steps, "ema_decay": self.ema_decay,
                "baselines": dict(self.baselines), "counts": dict(self.counts)}

    def load_state_dict(self, state: dict) -> None:
        if int(state["patience_steps"]) != self.patience_steps:
            raise ValueError("alert patience is incompatible")
        self.baselines = {k: float(v) for k, v in state.get("baselines", {}).items()}
        self.counts = {k: int(v) for k, v in state.get("counts", {}).items()}


# --------------------------------------------------------------------------- collector
class KimiDiagnosticCollector:
    """Per-step diagnostics with a bounded time and memory budget (reference collector API)."""

    def __init__(self, model, config: DiagnosticsConfig | None = None, *, parameter_specs=()):
        self.model = model
        self.config = config or DiagnosticsConfig()
        self.alerts = AlertManager(self.config.alert_patience_steps)
        self.update_monitor = ParameterUpdateMonitor(parameter_specs,
                                                     max_parameters_per_group=self.config.sample_parameters_per_group,
                                                     max_elements_per_parameter=self.config.sample_elements_per_parameter)
        self.latest_metrics: dict = {}
        self.latest_alerts = ()
        self.rotation_index = 0
        self.last_diagnostic_time_ms = 0.0
        self.current_diagnostic_time_ms = 0.0
        self.degrade_until_step = 0
        self.metric_ema: dict = {}
        self.previous_state_rms: dict = {}
        self.active_level: str | None = None
        self._pending = MetricBatch()
        # Distributed runs: the budget decision is MAX-reduced over this group (on this device) so that
        # every rank degrades on the same steps and runs the same diagnostics (and their collectives).
        self.budget_group = None
        self.budget_device = None

    def level_for_step(self, step: int) -> str | None:
        level = self.config.level_for_step(step)
        if step <= self.degrade_until_step and level in ("standard", "deep"):
            return "cheap"
        return level

    def model_kwargs_for_step(self, step: int) -> dict:
        if self.level_for_step(step) not in ("standard", "deep"):
            return {}
        return {"output_hidden_states": True, "output_router_diagnostics": True, "output_attnres_diagnostics": True}

    def _sample_layer_indices(self, count: int, step: int) -> tuple:
        limit = min(self.config.sample_layers_per_standard_step, count)
        if count <= limit:
            return tuple(range(count))
        anchors = tuple(dict.fromkeys((0, count // 2, count - 1)))
        chosen = set(anchors[:limit])
        cursor = step // self.config.standard_every_steps if self.config.rotate_sampled_layers else 0
        idx = cursor % count
        while len(chosen) < limit:
            chosen.add(idx)
            idx = (idx + 1) % count
        return tuple(sorted(chosen))

    def collect_output(self, output, *, step: int) -> dict:
        self.active_level = self.level_for_step(step)
        if self.active_level is None:
            self.latest_metrics = {}
            return {}
        t0 = time.perf_counter()
        mb = MetricBatch()
        lo = getattr(output, "loss_output", None)
        if lo is not None:
            mtp = lo.mtp
            mb.update(loss_metrics(total_loss=lo.loss.detach(), ntp_loss=lo.ntp.loss.detach(),
                                   mtp_loss=None if mtp is None else mtp.loss.detach(),
                                   ntp_tokens=lo.ntp.normalizer, mtp_tokens=0.0 if mtp is None else mtp.normalizer,
                                   lambda_mtp=lo.lambda_mtp))
        state_rms = {}
        if self.active_level in ("standard", "deep"):
            mb.update(vision_metrics(getattr(output, "vision_outputs", None),
                                     getattr(output, "multimodal_metadata", None)))
            backbone = getattr(output, "backbone_diagnostics", None) or {}
            layers = tuple(backbone.get("layers", ()))
            sampled = self._sample_layer_indices(len(layers), step)
            for i in sampled:
                layer = layers[i]
                kind = layer.get("attention_type", "")
                if kind == "kda":
                    m = kda_metrics(layer.get("mechanism"), prefix=f"kda/layer_{i:02d}")
                    mb.update(m)
                    if f"kda/layer_{i:02d}/state_rms" in m:
                        state_rms[f"kda/layer_{i:02d}/state_rms"] = m[f"kda/layer_{i:02d}/state_rms"]
                elif kind in ("gated_mla", "gated_mla_final"):
                    mb.update(mla_metrics(layer.get("mechanism"), prefix=f"mla/layer_{i:02d}"))
                mb.update(moe_metrics(layer.get("channel_mixer"), prefix=f"moe/layer_{i:02d}"))
            trace = getattr(output, "backbone_trace", None)
            if trace is not None:
                for i in sampled:
                    a_in, a_br = trace.pre_attention[i], trace.attention_outputs[i]
                    bm = block_contribution(a_in, a_br, a_in + a_br, prefix=f"block/layer_{i:02d}/attention")
                    mb.update(bm)
                    arch = "kda" if layers[i].get("attention_type") == "kda" else "mla"
                    mb[f"{arch}/layer_{i:02d}/branch_to_input_rms"] = bm[f"block/layer_{i:02d}/attention/branch_to_input_rms"]
                    f_in, f_br = trace.pre_ffn[i], trace.ffn_outputs[i]
                    mb.update(block_contribution(f_in, f_br, f_in + f_br, prefix=f"block/layer_{i:02d}/moe"))
                mb.update(representation_metrics(trace.final_mixed, max_tokens=self.config.sample_tokens_per_layer))
                mb.update(activation_metrics(trace.final_mixed, max_elements=self.config.sample_tokens_per_layer
                                             * trace.final_mixed.shape[-1]))
            mb.update(attnres_metrics(getattr(output, "attnres_diagnostics", None)))
            mb.update(mtp_metrics(getattr(output, "mtp_diagnostics", None),
                                  loss_weight=0.0 if lo is None else lo.lambda_mtp))
            mb["diagnostics/layers_sampled"] = float(len(sampled))
        metrics = mb.materialize()  # the single device-to-host copy of this phase
        if "train/loss_mtp" in metrics and "mtp/loss" not in metrics:
            metrics["mtp/loss"] = metrics["train/loss_mtp"]
        for name in [k for k in metrics if k.endswith("/dead_expert_fraction_batch")]:
            ema_name = name.replace("_batch", "_ema")
            prev = self.metric_ema.get(ema_name, metrics[name])
            self.metric_ema[ema_name] = metrics[ema_name] = 0.95 * prev + 0.05 * metrics[name]
        for name in state_rms:
            cur = metrics[name]
            prev = self.previous_state_rms.get(name, cur)
            metrics[name.replace("/state_rms", "/state_growth_ratio")] = cur / max(prev, 1e-12)
            self.previous_state_rms[name] = cur
        ms = (time.perf_counter() - t0) * 1000.0
        self.last_diagnostic_time_ms = self.current_diagnostic_time_ms = ms
        metrics["diagnostics/time_ms"] = metrics["train/diagnostics_time_ms"] = ms
        metrics["diagnostics/scalars_emitted"] = float(len(metrics))
        self.latest_metrics = dict(metrics)
        return dict(metrics)

    def capture_before_optimizer_step(self) -> dict:
        if self.active_level is None:
            return {}
        t0 = time.perf_counter()
        self._pending = MetricBatch()
        self._pending.update(self.update_monitor.capture_before_step())
        self.current_diagnostic_time_ms += (time.perf_counter() - t0) * 1000.0
        return {}  # materialised together with the after-step statistics

    def capture_after_optimizer_step(self, *, step: int, step_time_ms: float | None = None):
        if self.active_level is None:
            return {}, ()
        t0 = time.perf_counter()
        self._pending.update(self.update_monitor.capture_after_step())
        metrics = self._pending.materialize()
        self._pending = MetricBatch()
        self.current_diagnostic_time_ms += (time.perf_counter() - t0) * 1000.0
        self.last_diagnostic_time_ms = self.current_diagnostic_time_ms
        metrics["diagnostics/time_ms"] = metrics["train/diagnostics_time_ms"] = self.last_diagnostic_time_ms
        if step_time_ms is not None:
            frac = self.last_diagnostic_time_ms / max(step_time_ms, 1e-12)
            metrics["diagnostics/time_fraction"] = metrics["train/diagnostics_time_fraction"] = frac
        over = (metrics.get("diagnostics/time_fraction", 0.0) > self.config.max_diagnostic_time_fraction or
                metrics.get("diagnostics/persistent_gpu_bytes", 0.0) > self.config.max_persistent_gpu_bytes)
        if self.budget_device is not None and torch.distributed.is_available() and torch.distributed.is_initialized() \
                and torch.distributed.get_world_size(self.budget_group) > 1:
            flag = torch.tensor([float(over)], device=self.budget_device)
            torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MAX, group=self.budget_group)
            over = bool(flag.item() > 0)
        if over:
            self.degrade_until_step = max(self.degrade_until_step, step + self.config.standard_every_steps)
        metrics["diagnostics/budget_exceeded"] = float(over)
        metrics["diagnostics/degradation_level"] = float(step <= self.degrade_until_step)
        combined = {**self.latest_metrics, **metrics}
        self.latest_alerts = self.alerts.evaluate(combined, step)
        self.latest_metrics = combined
        self.active_level = None
        return dict(metrics), self.latest_alerts

    def state_dict(self) -> dict:
        return {"config": self.config.to_dict(), "alerts": self.alerts.state_dict(),
                "rotation_index": self.rotation_index, "latest_metrics": dict(self.latest_metrics),
                "degrade_until_step": self.degrade_until_step, "metric_ema": dict(self.metric_ema),
                "previous_state_rms": dict(self.previous_state_rms)}

    def load_state_dict(self, state: dict) -> None:
        self.alerts.load_state_dict(state["alerts"])
        self.rotation_index = int(state.get("rotation_index", 0))
        self.latest_metrics = {k: float(v) for k, v in state.get("latest_metrics", {}).items()}
        self.degrade_until_step = int(state.get("degrade_until_step", 0))
        self.metric_ema = {k: float(v) for k, v in state.get("metric_ema", {}).items()}
        self.previous_state_rms = {k: float(v) for k, v in state.get("previous_state_rms", {}).items()}

    def diagnostic_snapshot(self, step: int) -> dict:
        return {"step": int(step), "metrics": dict(self.latest_metrics),
                "alerts": [a.to_dict() for a in self.latest_alerts]}


__all__ = ["DiagnosticsConfig", "MetricBatch", "KimiDiagnosticCollector", "ParameterUpdateMonitor", "AlertManager",
           "DiagnosticAlert", "ALERT_RULES", "diagnostic_family", "kda_metrics", "mla_metrics", "moe_metrics",
           "attnres_metrics", "loss_metrics", "mtp_metrics", "block_contribution", "representation_metrics",
           "activation_metrics", "vision_metrics"]
