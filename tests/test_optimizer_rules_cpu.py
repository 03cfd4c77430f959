"""Optimizer building blocks on CPU: config rules, Newton-Schulz properties, update-RMS matching, head
layouts and Per-Head orthogonalisation, the parameter registry, QK-Clip and the transactional skip.

Oracles: the quintic Newton-Schulz contract of ``training/optimizer/newton_schulz.py:11-74`` (scale-free,
near-orthogonal output, zero maps to zero, tall matrices via the transpose), the per-head rule of
``per_head_muon.py:310-326``, QK-Clip's ``sqrt(tau / s)`` factor (``qk_clip.py:87-144``) and the reference
registry (``parameter_registry.py:169``).
"""
import io

import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.train.optimizer import (HeadMatrixLayout, KimiOptimizerConfig, QKClipController,
                                          batched_newton_schulz, build_kimi_optimizer, build_parameter_registry,
                                          match_update_rms, merge_head_matrix, per_head_orthogonalize,
                                          split_head_matrix, zeropower_via_newton_schulz)

F64 = torch.float64


def _tiny(seed=0):
    torch.manual_seed(seed)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False))


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("bad", [dict(kind="sgd"), dict(adamw_lr=0.0), dict(adamw_betas=(0.9, 1.0)),
                                 dict(adamw_betas=(0.9,)), dict(muon_lr=-1.0), dict(muon_momentum=1.0),
                                 dict(muon_ns_steps=0), dict(weight_decay=-0.1), dict(qk_clip_threshold=0.0),
                                 dict(per_head_qkv=False), dict(muon_ns_dtype="float16")])
def test_config_rejects_invalid_values(bad):
    with pytest.raises(ValueError):
        KimiOptimizerConfig(**bad)


def test_config_resolution_and_round_trip():
    c = KimiOptimizerConfig(adamw_lr=1e-3, weight_decay=0.05)
    assert c.resolved_muon_lr == 1e-3 and c.resolved_muon_weight_decay == 0.05
    c2 = KimiOptimizerConfig(muon_lr=0.02, muon_weight_decay=0.0)
    assert c2.resolved_muon_lr == 0.02 and c2.resolved_muon_weight_decay == 0.0
    assert KimiOptimizerConfig.from_dict(c.to_dict()) == c


# --------------------------------------------------------------------------- Newton-Schulz
@pytest.mark.parametrize("shape", [(8, 8), (6, 16), (16, 6), (1, 9)])
def test_newton_schulz_is_near_orthogonal_and_scale_free(shape):
    torch.manual_seed(shape[0] * 31 + shape[1])
    x = torch.randn(*shape, dtype=F64)
    o = zeropower_via_newton_schulz(x)
    s = torch.linalg.svdvals(o.double())
    assert s.min().item() > 0.6 and s.max().item() < 1.25  # the quintic's convergence band
    assert max_diff(zeropower_via_newton_schulz(x * 123.0), o) < 1e-5
    # same singular vectors as the polar factor: o^T x is symmetric positive semi-definite
    m = (o.double().T @ x) if shape[0] <= shape[1] else (x.T @ o.double())
    assert max_diff(m, m.T) < 1e-4 * x.abs().max().item() * max(shape)


def test_newton_schulz_edge_cases():
    assert zeropower_via_newton_schulz(torch.zeros(4, 6)).abs().max().item() == 0.0
    x = torch.randn(9, 4)
    assert max_diff(zeropower_via_newton_schulz(x), zeropower_via_newton_schulz(x.T).T) < 1e-6
    with pytest.raises(ValueError):
        zeropower_via_newton_schulz(torch.randn(2, 3, 4))
    with pytest.raises(ValueError):
        zeropower_via_newton_schulz(x, steps=0)
    with pytest.raises(FloatingPointError):
        zeropower_via_newton_schulz(torch.full((3, 3), float("nan")))
    batch = torch.randn(5, 6, 10)
    batch[2] = 0
    b = batched_newton_schulz(batch)
    for i in range(5):
        assert max_diff(b[i], zeropower_via_newton_schulz(batch[i])) < 1e-5


def test_match_update_rms_modes():
    u = torch.randn(4, 9)
    assert max_diff(match_update_rms(u), u * 3.0) < 1e-6
    ref_t = torch.randn(4, 9) * 5
    out = match_update_rms(u, ref_t, mode="reference_rms")
    assert abs(out.square().mean().sqrt().item() - ref_t.square().mean().sqrt().item()) < 1e-4
    assert match_update_rms(torch.zeros(4, 9), ref_t, mode="reference_rms").abs().max().item() == 0.0
    with pytest.raises(ValueError):
        match_update_rms(u, None, mode="reference_rms")
    with pytest.raises(ValueError):
        match_update_rms(u, mode="spectral")


# --------------------------------------------------------------------------- head layouts
@pytest.mark.parametrize("axis", [0, 1])
def test_head_split_merge_round_trip(axis):
    out_dim, in_dim = (12, 5) if axis == 0 else (5, 12)
    lay = HeadMatrixLayout(3, 4, axis, in_dim, out_dim)
    w = torch.randn(out_dim, in_dim)
    blocks = split_head_matrix(w, lay)
    assert len(blocks) == 3
    if axis == 0:
        assert torch.equal(blocks[1], w[4:8])
    else:
        assert torch.equal(blocks[1], w[:, 4:8])
    assert torch.equal(merge_head_matrix(blocks, lay), w)
    with pytest.raises(ValueError):
        lay.validate(torch.randn(out_dim + 1, in_dim))
    with pytest.raises(ValueError):
        HeadMatrixLayout(0, 4, 0, 4, 4)
    with pytest.raises(ValueError):
        HeadMatrixLayout(2, 4, 0, 4, 8, packed_kind="fused_qkv")


def test_per_head_orthogonalize_equals_each_head_alone():
    torch.manual_seed(3)
    lay = HeadMatrixLayout(4, 3, 0, 10, 12)
    w = torch.randn(12, 10)
    w[3:6] *= 100.0                 # one head with a much larger scale
    out, metrics = per_head_orthogonalize(w, lay, steps=5, eps=1e-7)
    for h in range(4):
        want = zeropower_via_newton_schulz(w[3 * h:3 * h + 3]) * (10 ** 0.5)
        assert max_diff(out[3 * h:3 * h + 3], want) < 1e-5
    assert metrics["per_head_muon/fraction_heads_near_zero_update"] == 0.0
    assert metrics["per_head_muon/head_update_rms_max_to_median"] < 1.5  # equalised despite the 100x head


# --------------------------------------------------------------------------- registry
def test_registry_families_follow_the_rules():
    m = _tiny()
    rep = build_parameter_registry(m)
    fam = {s.parameter_name: s.optimizer_family for s in rep.specs}
    assert fam["embed_tokens.weight"] == "adamw_no_decay"
    assert "lm_head.weight" not in fam  # tied to the embedding: registered once
    kda = "backbone.backbone.groups.0.layers.0.attention.projections"
    assert fam[f"{kda}.q_proj.weight"] == "per_head_muon" and fam[f"{kda}.v_proj.weight"] == "per_head_muon"
    assert fam[f"{kda}.alpha_down.weight"] == "muon"
    assert fam[f"{kda}.b_alpha"] == "adamw_decay"        # a 2-D [H, K] tensor that is not a Linear
    assert fam[kda.replace("projections", "decay.A_log")] == "adamw_no_decay"
    assert all(f == "adamw_no_decay" for n, f in fam.items() if "norm" in n or "pseudo_query" in n)
    assert all(f != "muon" and f != "per_head_muon" for n, f in fam.items() if ".router." in n)
    assert any(f == "muon" and "routed_experts" in n for n, f in fam.items())
    assert not rep.missing and not rep.duplicates and not rep.ambiguous
    assert rep.total_numel == m.num_parameters()
    assert abs(sum(rep.percentages_by_family.values()) - 100.0) < 1e-9
    plain = build_parameter_registry(m, kind="muon_adamw")
    assert plain.tensor_count_by_family["per_head_muon"] == 0
    adam = build_parameter_registry(m, kind="adamw")
    assert adam.tensor_count_by_family["muon"] == 0 and adam.tensor_count_by_family["per_head_muon"] == 0
    assert build_parameter_registry(_tiny()).fingerprint == rep.fingerprint


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("kind", ["per_head_muon_adamw", "muon_adamw", "adamw"])
def test_registry_matches_reference(kind):
    ref()
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as rcfg
    from src.kimi_k3_mini import KimiK3 as RK
    from training.optimizer.parameter_registry import build_parameter_registry as rbuild
    theirs = rbuild(RK(rcfg(enable_vision=False)), kind=kind)
    ours = build_parameter_registry(_tiny(), kind=kind)
    tf = {s.parameter_name: s.optimizer_family for s in theirs.specs}
    of = {}
    for s in ours.specs:
        if s.parameter_name.endswith(("routed_experts.gate_proj", "routed_experts.up_proj",
                                      "routed_experts.down_proj")):
            pre, leaf = s.parameter_name.rsplit(".", 1)
            for e in range(s.parameter.shape[0]):
                of[f"{pre}.{e}.transform.{leaf}.weight"] = s.optimizer_family
        else:
            of[s.parameter_name] = s.optimizer_family
    assert of == tf


# --------------------------------------------------------------------------- QK-Clip
def _mla_layers(model):
    from kimi_k3_b200.models.mla import GatedMLA
    return [m for m in model.modules() if isinstance(m, GatedMLA)]


def test_qk_clip_scales_both_matrices_so_the_proxy_lands_on_tau():
    m = _tiny(1).double()
    layers = _mla_layers(m.backbone)  # the MTP block's layers run only with use_mtp
    with torch.no_grad():
        for layer in layers:
            layer.projections.query.weight.mul_(40.0)
            layer.projections.latent_kv.key_up.weight.mul_(40.0)
    ids = torch.randint(5, 128, (2, 9))
    with torch.no_grad():
        m(input_ids=ids)
    before = [float(layer._last_qk_scale) for layer in layers]
    wq0 = [layer.projections.query.weight.clone() for layer in layers]
    wk0 = [layer.projections.latent_kv.key_up.weight.clone() for layer in layers]
    tau = min(before) / 2
    ctl = QKClipController(m, threshold=tau)
    rep = ctl.apply(1)
    assert rep.applied and rep.events == len(layers)
    assert abs(rep.max_preclip_scale - max(before)) < 1e-6 * max(before) and rep.max_postclip_scale == tau
    assert abs(rep.min_rescale_factor - tau / max(before)) < 1e-6
    for layer, s, wq, wk in zip(layers, before, wq0, wk0):
        f = (tau / s) ** 0.5
        assert max_diff(layer.projections.query.weight, wq * f) < 1e-6 * wq.abs().max().item()
        assert max_diff(layer.projections.latent_kv.key_up.weight, wk * f) < 1e-6 * wk.abs().max().item()
    with torch.no_grad():
        m(input_ids=ids)
    # the first MLA layer sees unchanged inputs, so its proxy lands on tau (the proxy is computed in fp32)
    assert abs(float(layers[0]._last_qk_scale) - tau) < 1e-4 * tau
    assert ctl.total_events == len(layers)


def test_qk_clip_leaves_small_proxies_alone_and_honours_schedule_and_skip():
    m = _tiny(2).double()
    ids = torch.randint(5, 128, (2, 6))
    with torch.no_grad():
        m(input_ids=ids)
    layer = _mla_layers(m.backbone)[0]
    w = layer.projections.query.weight.clone()
    ctl = QKClipController(m, threshold=1e9)
    assert not ctl.apply(1).applied and torch.equal(layer.projections.query.weight, w)
    low = QKClipController(m, threshold=1e-6, every_steps=2)
    assert not low.apply(1).applied and torch.equal(layer.projections.query.weight, w)   # off-schedule step
    low.apply(2, skip=torch.tensor(True))                                              # skipped step
    assert torch.equal(layer.projections.query.weight, w)
    st = low.state_dict()
    QKClipController(m, threshold=1e-6, every_steps=2).load_state_dict(st)
    with pytest.raises(ValueError):
        QKClipController(m, threshold=2e-6, every_steps=2).load_state_dict(st)
    with pytest.raises(ValueError):
        QKClipController(m, threshold=0.0)


# --------------------------------------------------------------------------- hybrid step
def test_non_finite_gradient_skips_the_whole_step():
    m = _tiny(3)
    opt, _ = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=0.02))
    ids = torch.randint(5, 128, (2, 8))
    m(input_ids=ids, labels=ids).loss.backward()
    opt.step()
    snap = {n: p.detach().clone() for n, p in m.named_parameters()}
    state_before = {k: v.clone() if torch.is_tensor(v) else v for k, v in opt.state_dict().items()
                    if torch.is_tensor(v)}
    opt.zero_grad()
    m(input_ids=ids, labels=ids).loss.backward()
    next(p for p in m.parameters() if p.grad is not None).grad.view(-1)[0] = float("nan")
    opt.step()
    rep = opt.materialize_report()
    assert not rep.executed
    for n, p in m.named_parameters():
        assert torch.equal(p, snap[n]), n
    assert set(state_before) <= set(opt.state_dict())


def test_optimizer_state_round_trips():
    a, b = _tiny(4), _tiny(4)
    oa, _ = build_kimi_optimizer(a, KimiOptimizerConfig(muon_lr=0.02))
    ob, _ = build_kimi_optimizer(b, KimiOptimizerConfig(muon_lr=0.02))
    ids = torch.randint(5, 128, (2, 8))
    for _ in range(2):
        oa.zero_grad()
        a(input_ids=ids, labels=ids).loss.backward()
        oa.step()
    # through bytes, as a checkpoint file would (loading a live state dict shares its tensors)
    buf = io.BytesIO()
    torch.save({"model": a.state_dict(), "optimizer": oa.state_dict()}, buf)
    buf.seek(0)
    payload = torch.load(buf, weights_only=False)
    b.load_state_dict(payload["model"])
    ob.load_state_dict(payload["optimizer"])
    for m_, o in ((a, oa), (b, ob)):
        o.zero_grad()
        m_(input_ids=ids, labels=ids).loss.backward()
        o.step()
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert max_diff(pa, pb) < 1e-6, n


def test_optimizer_state_from_another_registry_is_rejected():
    a = _tiny(5)
    oa, _ = build_kimi_optimizer(a, KimiOptimizerConfig(muon_lr=0.02))
    other, _ = build_kimi_optimizer(_tiny(5), KimiOptimizerConfig(kind="muon_adamw", muon_lr=0.02))
    with pytest.raises(ValueError):
        oa.load_state_dict(other.state_dict())
