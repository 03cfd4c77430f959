"""The training loop's contract on CPU: token-exact accumulation windows, gradient clipping, the
non-finite skip (parameters, optimizer state and the Quantile-Balancing bias all untouched), batch
limits, scheduler and EMA hooks, and argument checks.

Reference behaviour: ``training/train_one_epoch.py:63-598`` (one optimizer step per window, global norm
and clip, transactional skip of a non-finite step, QB window committed only after an executed step).
"""
import math

import pytest
import torch

from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.train.ema import EMA
from kimi_k3_b200.train.engine import MoEController
from kimi_k3_b200.train.loop import train_one_epoch
from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
from kimi_k3_b200.train.scheduler import WarmupCosineLR


def _model(seed=0):
    torch.manual_seed(seed)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double()


def _batches(n=4, rows=2, t=12, seed=1):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        ids = torch.randint(5, 128, (rows, t), generator=g)
        mask = torch.ones(rows, t, dtype=torch.bool)
        mask[0, t - 1 - i:] = False                       # uneven valid-token counts per micro-batch
        out.append({"input_ids": ids, "labels": ids.clone(), "attention_mask": mask})
    return out


def _opt(model):
    return build_kimi_optimizer(model, KimiOptimizerConfig(kind="adamw", adamw_lr=1e-3, adamw_eps=1e-2,
                                                           weight_decay=0.0, qk_clip_enabled=False))[0]


def _params(m):
    return {n: p.detach().clone() for n, p in m.named_parameters()}


def test_accumulated_window_equals_one_step_on_the_concatenated_batch():
    parts = _batches(3)
    whole = {k: torch.cat([b[k] for b in parts], 0) for k in parts[0]}
    a, b = _model(), _model()
    ra = train_one_epoch(a, parts, _opt(a), grad_accum_steps=3, use_mtp=True)
    rb = train_one_epoch(b, [whole], _opt(b), grad_accum_steps=1, use_mtp=True)
    assert ra["optimizer_steps"] == rb["optimizer_steps"] == 1
    assert abs(ra["loss"] - rb["loss"]) < 1e-6
    pa, pb = _params(a), _params(b)
    worst = max((pa[n] - pb[n]).abs().max().item() for n in pa)
    assert worst < 1e-6


def test_gradient_clipping_bounds_the_applied_norm():
    m = _model()
    opt = _opt(m)
    res = train_one_epoch(m, _batches(1), opt, grad_clip=1e-3, use_mtp=True)
    pre, post = res["grad_norm_pre_clip"], res["grad_norm_post_clip"]
    assert pre > 1e-3 and post == pytest.approx(1e-3, rel=1e-3)
    m2 = _model()
    free = train_one_epoch(m2, _batches(1), _opt(m2), use_mtp=True)
    assert free["grad_norm_post_clip"] == pytest.approx(free["grad_norm_pre_clip"])
    with pytest.raises(ValueError):
        train_one_epoch(m, _batches(1), opt, grad_clip=0.0)


def test_a_non_finite_step_changes_nothing():
    m = _model()
    opt = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=1e-2))[0]
    ctl = MoEController(m)
    train_one_epoch(m, _batches(1), opt, use_mtp=True, moe_controller=ctl)   # optimizer state exists now
    before = _params(m)
    buffers = {n: b.clone() for n, b in m.named_buffers()}
    bad = _batches(1, seed=9)
    # a finite loss whose gradient is not finite (a non-finite logit would already fail the loss check)
    target = m.backbone.backbone.final_norm.weight
    handle = target.register_hook(lambda g: g * float("nan"))
    try:
        res = train_one_epoch(m, bad, opt, use_mtp=True, moe_controller=ctl)
    finally:
        handle.remove()
    assert res["optimizer_steps"] == 0 and res["skipped_optimizer_steps"] == 1
    after = _params(m)
    for n in before:
        assert torch.equal(before[n], after[n]), n
    for n, b in m.named_buffers():
        assert torch.equal(buffers[n], b), n                           # routing biases untouched
    # and training continues normally afterwards
    ok = train_one_epoch(m, _batches(1, seed=3), opt, use_mtp=True, moe_controller=ctl)
    assert ok["optimizer_steps"] == 1 and math.isfinite(ok["loss"])


def test_batch_limit_scheduler_and_ema_hooks():
    m = _model()
    opt = _opt(m)
    sched = WarmupCosineLR(opt.adamw if hasattr(opt, "adamw") else opt, 10, 2)
    ema = EMA(m, decay=0.5)
    steps_seen = []
    res = train_one_epoch(m, _batches(4), opt, scheduler=sched, ema=ema, max_batches=3, use_mtp=True,
                          on_optimizer_step=lambda info: steps_seen.append(info))
    assert res["optimizer_steps"] == 3 and len(steps_seen) == 3
    assert sched.step_num == 3 and ema.num_updates == 3
    none = train_one_epoch(m, _batches(2), opt, max_batches=0, use_mtp=True)
    assert none["optimizer_steps"] == 0
    with pytest.raises(ValueError):
        train_one_epoch(m, _batches(1), opt, grad_accum_steps=0)
    with pytest.raises(ValueError):
        train_one_epoch(m, _batches(1), opt, max_batches=-1)


def test_image_batches_train_and_evaluate_through_the_loop():
    """Batches carrying ``pixel_values`` (four placeholder tokens per image) pass through the training and
    evaluation loops; a video of two frames composes into its placeholders too."""
    from kimi_k3_b200.train.loop import eval_one_epoch
    torch.manual_seed(0)
    cfg = kimi_k3_cpu_tiny_config()
    m = KimiK3(cfg)
    opt = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=0.01))[0]
    batches = []
    for _ in range(3):
        ids = torch.randint(5, 128, (2, 16))
        ids[:, 2:6] = cfg.image_token_id
        batches.append({"input_ids": ids, "labels": ids.masked_fill(ids == cfg.image_token_id, -100),
                        "attention_mask": torch.ones(2, 16, dtype=torch.bool),
                        "pixel_values": torch.randn(2, 3, 16, 16)})
    vision_before = {n: p.detach().clone() for n, p in m.named_parameters() if n.startswith("vision_")}
    res = train_one_epoch(m, batches, opt, use_mtp=True, moe_controller=MoEController(m), grad_clip=1.0)
    assert res["optimizer_steps"] == 3 and math.isfinite(res["loss"])
    moved = [n for n, p in m.named_parameters() if n in vision_before and not torch.equal(p, vision_before[n])]
    assert moved                                    # the vision tower trains as well
    assert math.isfinite(eval_one_epoch(m, batches, use_mtp=True)["loss"])
    vids = torch.randint(5, 128, (1, 20))
    vids[0, 3:11] = cfg.video_token_id              # two frames of four tokens each
    out = m(input_ids=vids, video_values=torch.randn(1, 2, 3, 16, 16), labels=vids, use_mtp=True)
    assert math.isfinite(out.loss.item())
