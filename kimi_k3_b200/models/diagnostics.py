"""Per-mechanism diagnostics (KDA, MLA, Stable LatentMoE, backbone).

Parity targets (reference paths): ``src/kda/diagnostics.py:8-81``,
``src/mla/diagnostics.py:8-80``, ``src/stable_latent_moe/diagnostics.py:11-80``,
``src/hybrid_backbone/diagnostics.py:12-106``.  Key names match the reference so
the training diagnostics collector and its alerts read the same fields.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


def rms(x: torch.Tensor) -> torch.Tensor:
    return x.float().square().mean().sqrt()


def build_kda_diagnostics(q, k, beta, g, alpha, final_state, recurrent_output, gated_output, output_gate,
                          attention_mask, chunk_size, alpha_lower_bound) -> dict:
    valid = torch.ones(q.shape[:2], dtype=torch.bool, device=q.device) if attention_mask is None else attention_mask
    vh = valid[:, :, None].expand_as(beta)
    vhk = valid[:, :, None, None].expand_as(g)
    a, gg, bb = alpha[vhk].float(), g[vhk].float(), beta[vh].float()
    gate = output_gate[valid[:, :, None].expand_as(output_gate)].float()
    qe = (q.float().norm(dim=-1) - 1).abs()
    ke = (k.float().norm(dim=-1) - 1).abs()
    st = final_state.float()
    sn = st.flatten(-2).norm(dim=-1)
    cum = g.float().cumsum(dim=1)
    return {
        "alpha_min": a.min(), "alpha_max": a.max(), "alpha_mean": a.mean(), "alpha_std": a.std(unbiased=False),
        "fraction_alpha_near_lower_bound": (a <= alpha_lower_bound + 1e-3).float().mean(),
        "fraction_alpha_near_one": (a > 0.99).float().mean(),
        "log_decay_min": gg.min(), "log_decay_max": gg.max(), "log_decay_mean": gg.mean(),
        "cumulative_log_decay_min": cum[vhk].min(), "cumulative_log_decay_mean": cum[vhk].mean(),
        "beta_mean": bb.mean(), "beta_std": bb.std(unbiased=False),
        "beta_saturation_low": (bb < 0.01).float().mean(), "beta_saturation_high": (bb > 0.99).float().mean(),
        "state_norm_mean": sn.mean(), "state_norm_max": sn.max(), "state_rms": st.square().mean().sqrt(),
        "state_absmax": st.abs().max(), "recurrent_output_rms": rms(recurrent_output),
        "gated_output_rms": rms(gated_output), "q_norm_error": qe[vh].mean(), "k_norm_error": ke[vh].mean(),
        "output_gate_mean": gate.mean(), "output_gate_saturation_low": (gate < 0.01).float().mean(),
        "output_gate_saturation_high": (gate > 0.99).float().mean(),
        "output_gate_saturation": ((gate < 0.01) | (gate > 0.99)).float().mean(),
        "chunk_count": torch.tensor(math.ceil(q.shape[1] / chunk_size), dtype=torch.long, device=q.device),
    }


def build_mla_diagnostics(query, key, value, latent_kv, gate, attentions, key_mask, query_mask, cache_elements,
                          full_kv_width, attention_output, final_output, qk_scale) -> dict:
    p = attentions.float()
    pos = p > 0
    terms = torch.where(pos, -p * p.clamp_min(torch.finfo(torch.float32).tiny).log(), torch.zeros_like(p))
    rv = pos.any(dim=-1)
    ent = terms.sum(-1)[rv]
    support = pos.sum(-1)[rv].clamp_min(1)
    nent = torch.where(support > 1, ent / support.float().log().clamp_min(torch.finfo(torch.float32).tiny),
                       torch.zeros_like(ent))
    km = key_mask if key_mask is not None else torch.ones(latent_kv.shape[:2], dtype=torch.bool,
                                                          device=latent_kv.device)
    qm = query_mask
    lat = latent_kv[km].float().norm(dim=-1)
    gv = gate[qm].float()
    vq, vk, vv = query[qm], key[km], value[km]
    return {
        "attention_entropy": ent.mean(), "attention_entropy_normalized": nent.mean(),
        "attention_max_probability": p.max(dim=-1).values[rv].mean(),
        "gate_mean": gv.mean(), "gate_min": gv.min(), "gate_max": gv.max(),
        "gate_saturation_low": (gv < 0.01).float().mean(), "gate_saturation_high": (gv > 0.99).float().mean(),
        "latent_norm_mean": lat.mean(), "latent_norm_max": lat.max(),
        "query_norm_mean": vq.float().norm(dim=-1).mean(), "key_norm_mean": vk.float().norm(dim=-1).mean(),
        "q_rms": rms(vq), "k_rms": rms(vk), "v_rms": rms(vv), "attention_output_rms": rms(attention_output),
        "gated_output_rms": rms(final_output), "qk_scale_max": qk_scale.detach().float(),
        "cache_length": torch.tensor(latent_kv.shape[1], dtype=torch.long, device=query.device),
        "cache_elements": torch.tensor(cache_elements, dtype=torch.long, device=query.device),
        "compression_ratio": torch.tensor(full_kv_width / latent_kv.shape[-1], dtype=torch.float32,
                                          device=query.device),
    }


@dataclass
class MoEDiagnostics:
    num_tokens: int
    num_assignments: int
    shared_token_evaluations: int
    expert_load: torch.Tensor
    expert_load_fraction: torch.Tensor
    mean_load: torch.Tensor
    std_load: torch.Tensor
    min_load: torch.Tensor
    max_load: torch.Tensor
    coefficient_of_variation: torch.Tensor
    zero_load_experts: torch.Tensor
    selected_weight_mean: torch.Tensor
    selected_weight_min: torch.Tensor
    selected_weight_max: torch.Tensor
    routing_entropy_over_selected: torch.Tensor
    routing_bias_mean: torch.Tensor
    routing_bias_std: torch.Tensor
    routing_bias_min: torch.Tensor
    routing_bias_max: torch.Tensor
    qb_update_rms: torch.Tensor
    qb_quantile_error_estimate: torch.Tensor
    shared_output_rms: torch.Tensor
    routed_output_rms: torch.Tensor
    routed_aggregate_rms_before_norm: torch.Tensor
    routed_aggregate_rms_after_norm: torch.Tensor
    shared_to_total_ratio: torch.Tensor
    routed_to_total_ratio: torch.Tensor
    shared_routed_cosine: torch.Tensor
    output_rms: torch.Tensor


def build_moe_diagnostics(router, num_shared_experts, shared_output, routed_output, aggregate,
                          normalized_aggregate) -> MoEDiagnostics:
    loads = router.expert_load
    tokens, top_k = router.selected_experts.shape
    n_assign = tokens * top_k
    lf = loads.float()
    mean, std = lf.mean(), lf.std(unbiased=False)
    w = router.selected_weights.float()
    ent = -(w * w.clamp_min(torch.finfo(torch.float32).tiny).log()).sum(-1).mean()
    bias = router.routing_bias_before.float()
    after = router.routing_bias_after
    total = shared_output.float() + routed_output.float()
    trms = rms(total)
    srms, rrms = rms(shared_output), rms(routed_output)
    cos = F.cosine_similarity(shared_output.float().reshape(-1), routed_output.float().reshape(-1), dim=0, eps=1e-12)
    return MoEDiagnostics(
        tokens, n_assign, num_shared_experts * tokens, loads, lf / max(n_assign, 1), mean, std, lf.min(), lf.max(),
        std / mean.clamp_min(1e-12), (loads == 0).sum(), w.mean(), w.min(), w.max(), ent, bias.mean(),
        bias.std(unbiased=False), bias.min(), bias.max(),
        bias.new_zeros(()) if after is None else rms(after.float() - bias),
        (lf / max(n_assign, 1) - 1.0 / max(loads.numel(), 1)).abs().mean(), srms, rrms, rms(aggregate),
        rms(normalized_aggregate), srms / trms.clamp_min(1e-12), rrms / trms.clamp_min(1e-12), cos, trms)


def _count(module) -> int:
    return 0 if module is None else sum(p.numel() for p in module.parameters())


def parameter_counts(backbone) -> dict:
    layers = backbone.layers
    return {
        "kda": sum(_count(l.attention) for l in layers if l.attention_type == "kda"),
        "gated_mla": sum(_count(l.attention) for l in layers if l.attention_type == "gated_mla"),
        "ffn": sum(_count(l.ffn) for l in layers if l.ffn is not None),
        "norms": sum(_count(l.attention_norm) + _count(l.ffn_norm) for l in layers) + _count(backbone.final_norm),
        "attnres": sum(_count(s) for l in layers for s in (l.pre_attention_attnres, l.pre_ffn_attnres))
        + _count(backbone.final_output_attnres),
    }


def build_backbone_diagnostics(layer_diagnostics, backbone, cache, device) -> dict:
    counts = parameter_counts(backbone)
    counts["total"] = sum(counts.values())
    t = lambda v: torch.tensor(v, dtype=torch.long, device=device)  # noqa: E731
    return {
        "layers": layer_diagnostics,
        "num_kda_layers": sum(d["attention_type"] == "kda" for d in layer_diagnostics),
        "num_mla_layers": sum(d["attention_type"] in ("gated_mla", "gated_mla_final") for d in layer_diagnostics),
        "num_parameters_by_component": counts,
        "kda_cache_elements": t(0 if cache is None else cache.kda_elements),
        "mla_cache_elements": t(0 if cache is None else cache.mla_elements),
        "total_cache_elements": t(0 if cache is None else cache.total_elements),
    }
