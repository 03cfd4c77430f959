"""Diagnostics on CPU: tier schedule, the single-copy metric batch, and every metric extractor against
the reference extractor fed the same module diagnostics (metric names and values), plus alerts.

Reference: ``training/diagnostics/{config,kda_metrics,mla_metrics,moe_metrics,attnres_metrics,loss_metrics,
mtp_metrics,block_metrics,representation_metrics,activation_metrics,alerts}.py``.
"""
import math

import pytest
import torch

from _oracle import needs_reference, ref
from kimi_k3_b200.train.diagnostics import (AlertManager, DiagnosticsConfig, MetricBatch, activation_metrics,
                                            attnres_metrics, block_contribution, kda_metrics, loss_metrics,
                                            mla_metrics, moe_metrics, representation_metrics, t_cosine, t_ratio,
                                            t_rms)

F64 = torch.float64


def _close(ours: dict, theirs: dict, rel=1e-5):
    assert set(ours) == set(theirs), set(ours) ^ set(theirs)
    for k, v in theirs.items():
        a = float(ours[k])
        b = float(v)
        if math.isnan(b):
            assert math.isnan(a), k
        else:
            assert abs(a - b) <= rel * (1.0 + abs(b)), (k, a, b)


def _mat(d: dict) -> dict:
    mb = MetricBatch()
    mb.update(d)
    return mb.materialize()


# --------------------------------------------------------------------------- config and batch
@pytest.mark.parametrize("bad", [dict(cheap_every_steps=0), dict(standard_every_steps=-1),
                                 dict(sample_tokens_per_layer=0), dict(max_diagnostic_time_fraction=0.0),
                                 dict(max_diagnostic_time_fraction=1.5), dict(max_persistent_gpu_bytes=-1),
                                 dict(alert_patience_steps=0)])
def test_config_rejects_invalid_values(bad):
    with pytest.raises(ValueError):
        DiagnosticsConfig(**bad)


@pytest.mark.parametrize("step,level", [(0, None), (1, "cheap"), (9, "cheap"), (10, "standard"), (500, "deep"),
                                        (1000, "deep"), (510, "standard")])
def test_level_schedule(step, level):
    assert DiagnosticsConfig().level_for_step(step) == level
    assert DiagnosticsConfig(enabled=False).level_for_step(step) is None
    assert DiagnosticsConfig.from_dict(DiagnosticsConfig().to_dict()) == DiagnosticsConfig()


@needs_reference
@pytest.mark.reference
def test_level_schedule_matches_reference():
    ref()
    from training.diagnostics.config import DiagnosticsConfig as RC
    kw = dict(cheap_every_steps=2, standard_every_steps=6, deep_every_steps=12)
    ours, theirs = DiagnosticsConfig(**kw), RC(**kw)
    for step in range(0, 40):
        assert ours.level_for_step(step) == theirs.level_for_step(step), step


def test_metric_batch_materialises_scalars_once():
    mb = MetricBatch()
    mb["a"] = torch.tensor(1.5)
    mb["b"] = 2
    mb.update({"c": torch.tensor([3.0])})
    other = MetricBatch()
    other["d"] = torch.tensor(4.0, dtype=F64)
    mb.update(other)
    assert "a" in mb and "z" not in mb
    assert mb.materialize() == {"a": 1.5, "b": 2.0, "c": 3.0, "d": 4.0}


def test_tensor_reducers():
    x = torch.tensor([3.0, 4.0])
    assert abs(t_rms(x).item() - (12.5 ** 0.5)) < 1e-6
    assert t_ratio(1.0, 0.0) == 1e12 and t_ratio(6.0, -3.0) == 2.0
    assert abs(t_ratio(torch.tensor(6.0), 3.0).item() - 2.0) < 1e-7
    assert abs(t_cosine(x, 2 * x).item() - 1.0) < 1e-6 and abs(t_cosine(x, -x).item() + 1.0) < 1e-6


# --------------------------------------------------------------------------- extractors vs the reference
def _kda_pair(seed=0):
    ref()
    from src.kda.config import KDAConfig as RC
    from src.kda.kda import KimiDeltaAttention as RK
    from kimi_k3_b200.models.kda import KDAConfig, KimiDeltaAttention
    torch.manual_seed(seed)
    kw = dict(d_model=16, num_heads=2, key_head_dim=4, value_head_dim=8, chunk_size=4, secondary_tile_size=4)
    ours = KimiDeltaAttention(KDAConfig(**kw)).double()
    theirs = RK(RC(**kw)).double()
    theirs.load_state_dict(ours.state_dict())
    return ours, theirs


@needs_reference
@pytest.mark.reference
def test_kda_and_block_metrics_match_reference():
    from training.diagnostics.block_metrics import compute_block_contribution
    from training.diagnostics.kda_metrics import compute_kda_metrics
    ours, theirs = _kda_pair()
    x = torch.randn(2, 9, 16, dtype=F64)
    mask = torch.ones(2, 9, dtype=torch.bool)
    mask[1, 6:] = False
    a = ours(x, attention_mask=mask, output_diagnostics=True)
    b = theirs(x, attention_mask=mask, output_diagnostics=True)
    _close(_mat(kda_metrics(a.diagnostics, prefix="layer0/kda")),
           compute_kda_metrics(b.diagnostics, prefix="layer0/kda"))
    y = x + a.hidden_states
    _close(_mat(block_contribution(x, a.hidden_states, y, prefix="blk")),
           compute_block_contribution(x, b.hidden_states, y, prefix="blk"))


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("clip", [False, True])
def test_mla_metrics_match_reference(clip):
    ref()
    from src.mla.config import GatedMLAConfig as RC
    from src.mla.gated_mla import GatedMLA as RM
    from training.diagnostics.mla_metrics import compute_mla_metrics
    from kimi_k3_b200.models.mla import GatedMLA, GatedMLAConfig
    torch.manual_seed(1)
    kw = dict(d_model=16, num_heads=2, q_head_dim=4, v_head_dim=8, kv_latent_dim=8)
    ours, theirs = GatedMLA(GatedMLAConfig(**kw)).double(), RM(RC(**kw)).double()
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(2, 7, 16, dtype=F64)
    a = ours(x, output_diagnostics=True).diagnostics
    b = theirs(x, output_diagnostics=True).diagnostics
    _close(_mat(mla_metrics(a, qk_clip_active=clip)), compute_mla_metrics(b, qk_clip_active=clip))


@needs_reference
@pytest.mark.reference
def test_moe_metrics_match_reference():
    ref()
    from src.stable_latent_moe.config import StableLatentMoEConfig as RC
    from src.stable_latent_moe.module import StableLatentMoE as RM
    from training.diagnostics.moe_metrics import compute_moe_metrics
    from kimi_k3_b200.models.moe import StableLatentMoE, StableLatentMoEConfig
    kw = dict(d_model=16, latent_dim=8, num_shared_experts=1, num_routed_experts=5, routed_experts_per_token=2,
              shared_expert_hidden_dim=12, routed_expert_hidden_dim=12)
    torch.manual_seed(2)
    theirs = RM(RC(**kw)).double()
    ours = StableLatentMoE(StableLatentMoEConfig(**kw)).double()
    ours.load_state_dict(theirs.state_dict())
    x = torch.randn(3, 6, 16, dtype=F64)
    a = ours(x, return_router_diagnostics=True).diagnostics
    b = theirs(x, return_router_diagnostics=True).diagnostics
    _close(_mat(moe_metrics(a)), compute_moe_metrics(b))


@needs_reference
@pytest.mark.reference
def test_attnres_metrics_match_reference():
    ref()
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as rcfg
    from src.kimi_k3_mini import KimiK3 as RK
    from training.diagnostics.attnres_metrics import compute_attnres_metrics
    from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
    torch.manual_seed(3)
    theirs = RK(rcfg(enable_vision=False)).double()
    ours = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double()
    ours.load_state_dict(theirs.state_dict())
    ids = torch.randint(5, 128, (2, 9))
    a = ours(input_ids=ids, output_attnres_diagnostics=True).attnres_diagnostics
    b = theirs(input_ids=ids, output_attnres_diagnostics=True).attnres_diagnostics
    _close(_mat(attnres_metrics(a)), compute_attnres_metrics(b))


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("mtp", [None, 2.5])
def test_loss_metrics_match_reference(mtp):
    ref()
    from training.diagnostics.loss_metrics import compute_loss_metrics
    kw = dict(total_loss=3.1 + (0 if mtp is None else 0.3 * mtp), ntp_loss=3.1, mtp_loss=mtp, ntp_tokens=120,
              mtp_tokens=0 if mtp is None else 100, lambda_mtp=0.3)
    _close(_mat(loss_metrics(**kw)), compute_loss_metrics(**kw))


@needs_reference
@pytest.mark.reference
def test_representation_and_activation_metrics_match_reference():
    ref()
    from training.diagnostics.activation_metrics import compute_activation_metrics
    from training.diagnostics.representation_metrics import compute_representation_metrics
    torch.manual_seed(4)
    h = torch.randn(3, 50, 16) * torch.linspace(0.1, 3.0, 16)
    _close(_mat(representation_metrics(h, max_tokens=100)), compute_representation_metrics(h, max_tokens=100),
           rel=1e-4)
    a = torch.randn(4000) * 3
    a[7] = float("inf")
    _close(_mat(activation_metrics(a, max_elements=3000)), compute_activation_metrics(a, max_elements=3000))


# --------------------------------------------------------------------------- alerts
@needs_reference
@pytest.mark.reference
def test_alerts_fire_after_the_same_patience_as_the_reference():
    ref()
    from training.diagnostics.alerts import AlertManager as RA
    ours, theirs = AlertManager(patience_steps=3), RA(patience_steps=3)
    series = ([{"train/loss_total": 2.0, "kda/layer0/fraction_alpha_near_one": 0.99,
                "moe/layer1/dead_expert_fraction_batch": 0.7, "mla/output_gate_saturation_low": 0.1}] * 5
              + [{"train/loss_total": float("nan"), "kda/layer0/fraction_alpha_near_one": 0.2}])
    for step, metrics in enumerate(series, 1):
        a = ours.evaluate(metrics, step)
        b = theirs.evaluate(metrics, step)
        assert sorted(x.code for x in a) == sorted(x.code for x in b), step
        if step == 3:
            assert {"KDA_RETENTION_SATURATION", "MOE_DEAD_EXPERTS_PERSISTENT"} <= {x.code for x in a}
    assert "NONFINITE_LOSS" in {x.code for x in a}
    fresh = AlertManager(patience_steps=3)
    fresh.load_state_dict(ours.state_dict())
    assert fresh.counts == ours.counts
    with pytest.raises(ValueError):
        AlertManager(patience_steps=4).load_state_dict(ours.state_dict())
