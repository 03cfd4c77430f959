"""Training services on CPU: diagnostics collector and alerts, EMA, checkpoints (format v2,
atomic, pruning, exact resume), progressive context curriculum."""
import math
import os

import pytest
import torch

from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.train.checkpoints import (list_checkpoints, load_checkpoint, prune_checkpoints,
                                            resolve_resume_path, save_checkpoint, write_latest_pointer)
from kimi_k3_b200.train.curriculum import (ContextCurriculumConfig, ContextStage, ProgressiveContextCollator,
                                           ProgressiveContextCurriculum, truncate_batch_to_context)
from kimi_k3_b200.train.diagnostics import AlertManager, DiagnosticsConfig, KimiDiagnosticCollector, MetricBatch
from kimi_k3_b200.train.ema import EMA, ema_health
from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer


def _model(seed=0):
    torch.manual_seed(seed)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False))


def test_diagnostics_standard_step_emits_finite_scalars():
    m = _model()
    opt, reg = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=0.01))
    col = KimiDiagnosticCollector(m, DiagnosticsConfig(standard_every_steps=2), parameter_specs=reg.specs)
    ids = torch.randint(5, 128, (2, 30))
    kw = col.model_kwargs_for_step(2)
    assert kw and col.level_for_step(2) == "standard"
    out = m(input_ids=ids, labels=ids, use_mtp=True, **kw)
    metrics = col.collect_output(out, step=2)
    assert "train/loss_total" in metrics and any(k.startswith("moe/layer_") for k in metrics)
    assert any(k.startswith("kda/layer_") for k in metrics) and any(k.startswith("attnres/") for k in metrics)
    out.loss.backward()
    col.capture_before_optimizer_step()
    opt.step()
    after, alerts = col.capture_after_optimizer_step(step=2, step_time_ms=1000.0)
    assert after["train/update_to_parameter_ratio_sampled"] > 0
    assert all(isinstance(v, float) for v in col.latest_metrics.values())
    assert all(math.isfinite(v) for v in col.latest_metrics.values())
    state = col.state_dict()
    col2 = KimiDiagnosticCollector(m, DiagnosticsConfig(standard_every_steps=2), parameter_specs=reg.specs)
    col2.load_state_dict(state)
    assert col2.latest_metrics == col.latest_metrics


def test_metric_batch_single_copy_and_alert_patience():
    mb = MetricBatch()
    mb["a"] = torch.tensor(2.0)
    mb["b"] = 3.0
    assert mb.materialize() == {"a": 2.0, "b": 3.0}
    am = AlertManager(patience_steps=3)
    for step in range(1, 3):
        assert not [a for a in am.evaluate({"moe/layer_01/dead_expert_fraction_batch": 0.9}, step)
                    if a.code == "MOE_DEAD_EXPERTS_PERSISTENT"]
    fired = [a for a in am.evaluate({"moe/layer_01/dead_expert_fraction_batch": 0.9}, 3)
             if a.code == "MOE_DEAD_EXPERTS_PERSISTENT"]
    assert fired and fired[0].patience_count == 3
    crit = am.evaluate({"train/loss_total": float("nan")}, 4)
    assert any(a.severity == "critical" for a in crit)


def test_ema_warmup_decay_and_swap():
    m = _model()
    ema = EMA(m, decay=0.9)
    p0 = {n: p.detach().clone() for n, p in m.named_parameters()}
    with torch.no_grad():
        for p in m.parameters():
            p.add_(1.0)
    assert ema.update(m)
    d = min(0.9, 2 / 11)  # first update: (1 + 1) / (10 + 1) with num_updates = 1
    name = next(iter(ema.shadow))
    assert torch.allclose(ema.shadow[name], d * p0[name] + (1 - d) * (p0[name] + 1), atol=1e-6)
    with ema.average_parameters(m):
        assert torch.allclose(dict(m.named_parameters())[name], ema.shadow[name])
    assert torch.allclose(dict(m.named_parameters())[name], p0[name] + 1)
    ok, status, _ = ema_health(ema, m)
    assert ok and status == "ok"
    e2 = EMA(_model(1), decay=0.9)
    e2.load_state_dict(ema.state_dict(), strict=True)
    assert e2.num_updates == 1 and torch.equal(e2.shadow[name], ema.shadow[name])


def test_checkpoint_roundtrip_and_exact_resume(tmp_path):
    from kimi_k3_b200.train.scheduler import WarmupCosineLR

    def build():
        m = _model()
        opt, _ = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=0.01, adamw_lr=1e-3))
        return m, opt, WarmupCosineLR(opt, total_steps=10, warmup_steps=2, prepare_first_update=True)

    def step(m, opt, sch, seed):
        ids = torch.randint(5, 128, (2, 20), generator=torch.Generator().manual_seed(seed))
        opt.zero_grad()
        m(input_ids=ids, labels=ids, use_mtp=True).loss.backward()
        opt.step()
        sch.step()

    a, oa, sa = build()
    for s in range(4):
        step(a, oa, sa, s)
    b, ob, sb = build()
    for s in range(2):
        step(b, ob, sb, s)
    path = save_checkpoint(tmp_path / "step_2.pt", b, optimizer=ob, scheduler=sb, global_step=2)
    c, oc, sc = build()
    info = load_checkpoint(path, c, optimizer=oc, scheduler=sc)
    assert info["format_version"] == 2 and info["global_step"] == 2
    for s in range(2, 4):
        step(c, oc, sc, s)
    for (n, p), (_, q) in zip(a.named_parameters(), c.named_parameters()):
        assert torch.equal(p, q), n  # bit-identical trajectory after resume


def test_checkpoint_pruning_and_latest(tmp_path):
    m = _model()
    for s in (1, 2, 3, 4):
        p = save_checkpoint(tmp_path / f"step_{s}.pt", m, global_step=s)
        write_latest_pointer(tmp_path, p)
    removed = prune_checkpoints(tmp_path, keep_last=2)
    assert [r.name for r in removed] == ["step_1.pt", "step_2.pt"]
    assert [p.name for p in list_checkpoints(tmp_path)] == ["step_3.pt", "step_4.pt"]
    assert resolve_resume_path("latest", tmp_path).name == "step_4.pt"
    assert not any(f.endswith(".tmp") for f in os.listdir(tmp_path))


def test_context_curriculum_transitions_and_state():
    cfg = ContextCurriculumConfig(enabled=True, stages=(ContextStage(16, 100), ContextStage(32, 300),
                                                        ContextStage(64, None)))
    cur = ProgressiveContextCurriculum(cfg, training_max_seq_len=64, mtp_min_seq_len=3)
    assert cur.current_max_seq_len() == 16
    assert not cur.update(50)
    assert cur.update(320) and cur.current_max_seq_len() == 64 and cur.last_transition.new_stage_index == 2
    st = cur.state_dict()
    fresh = ProgressiveContextCurriculum(cfg, training_max_seq_len=64, mtp_min_seq_len=3)
    fresh.load_state_dict(st)
    assert fresh.state == cur.state
    bad = dict(st, stage_index=1, max_seq_len=32)
    with pytest.raises(ValueError):
        ProgressiveContextCurriculum(cfg, training_max_seq_len=64, mtp_min_seq_len=3).load_state_dict(bad)
    with pytest.raises(ValueError):
        ContextCurriculumConfig(enabled=True, stages=(ContextStage(32, 10), ContextStage(16, None)))


def test_context_collator_pads_clips_and_trims():
    samples = [{"input_ids": torch.arange(1, 41), "labels": torch.arange(1, 41)},
               {"input_ids": torch.arange(1, 11), "labels": torch.arange(1, 11)}]
    col = ProgressiveContextCollator(24, pad_token_id=0)
    b = col(samples)
    assert b["input_ids"].shape == (2, 24) and b["attention_mask"][1].sum() == 10
    assert (b["labels"][1, 10:] == -100).all()
    short = ProgressiveContextCollator(24)([samples[1], samples[1]])
    assert short["input_ids"].shape == (2, 10)  # trimmed to the longest valid row
    bucketed = ProgressiveContextCollator(24, length_multiple=8)([samples[1], samples[1]])
    assert bucketed["input_ids"].shape == (2, 16)
    _, stats = truncate_batch_to_context(b, 12)
    assert stats["sequence_length"] == 12.0
