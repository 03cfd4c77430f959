"""Training services on CPU: the warmup-cosine schedule, token-exact window loss accounting, checkpoint
files (pruning, latest pointer, resume resolution, RNG state), EMA and the loggers.

Oracles: the schedule of ``training/scheduler.py:13-324`` (linear warmup to the base rate, cosine to
``min_lr``, separate Muon floor), the window rule of ``training/loss_accounting.py:36-214`` (sum of loss
sums over the sum of normalisers), the EMA decay ``min(d, (1 + n) / (10 + n))`` of ``training/ema.py`` and
the checkpoint contract of ``training/checkpoints.py``.
"""
import json
import math

import pytest
import torch

from _oracle import needs_reference, ref
from kimi_k3_b200.train.checkpoints import (checkpoint_step, list_checkpoints, prune_checkpoints,
                                            resolve_resume_path, restore_rng_state, rng_state,
                                            write_latest_pointer)
from kimi_k3_b200.train.ema import EMA
from kimi_k3_b200.train.scheduler import WarmupCosineLR, build_warmup_cosine_scheduler
from kimi_k3_b200.train.state import (JSONLLogger, LossContribution, MemoryLogger, combine_window_loss,
                                      count_batch_tokens)


def _sgd(lr=1.0):
    return torch.optim.SGD([torch.nn.Parameter(torch.zeros(2))], lr=lr)


class _Hybrid:
    """The two-optimizer shape the scheduler drives (``.muon`` and ``.adamw``)."""

    def __init__(self):
        self.muon = _sgd(0.02)
        self.adamw = _sgd(3e-4)


# --------------------------------------------------------------------------- schedule
def _expected(step, base, floor, warmup, total):
    if warmup and step <= warmup:
        return base * step / warmup
    t = min(max(step, warmup), total)
    return floor + (base - floor) * 0.5 * (1 + math.cos(math.pi * (t - warmup) / (total - warmup)))


@pytest.mark.parametrize("warmup,total", [(0, 10), (3, 10), (5, 6)])
def test_schedule_follows_warmup_then_cosine(warmup, total):
    opt = _sgd(2.0)
    s = WarmupCosineLR(opt, total, warmup, min_lr=0.1)
    for step in range(1, total + 4):
        s.step()
        assert opt.param_groups[0]["lr"] == pytest.approx(_expected(step, 2.0, 0.1, warmup, total)), step
    assert opt.param_groups[0]["lr"] == pytest.approx(0.1)      # holds the floor after the end


def test_hybrid_schedule_has_separate_floors_and_prepared_first_update():
    opt = _Hybrid()
    s = build_warmup_cosine_scheduler(opt, 20, 4, min_lr=1e-5, min_muon_lr=2e-3, prepare_first_update=True)
    # the first update already runs at the step-1 rate
    assert opt.muon.param_groups[0]["lr"] == pytest.approx(0.02 / 4)
    for _ in range(20):
        s.step()
    assert opt.muon.param_groups[0]["lr"] == pytest.approx(2e-3)
    assert opt.adamw.param_groups[0]["lr"] == pytest.approx(1e-5)
    d = s.get_lr_dict()
    assert set(d) == {"adamw_lr", "muon_lr", "step"} and d["step"] == 20
    assert len(s.get_last_lr()) == 2


def test_schedule_state_round_trip_and_device_resident_rates():
    opt = _sgd(1.0)
    s = WarmupCosineLR(opt, 50, 5, min_lr=0.0)
    for _ in range(17):
        s.step()
    fresh_opt = _sgd(1.0)
    fresh = WarmupCosineLR(fresh_opt, 50, 5, min_lr=0.0)
    fresh.load_state_dict(s.state_dict())
    assert fresh_opt.param_groups[0]["lr"] == pytest.approx(opt.param_groups[0]["lr"])
    fresh.set_step(0)
    assert fresh_opt.param_groups[0]["lr"] == 0.0
    lr_t = torch.tensor(1.0)
    dev_opt = _sgd(1.0)
    dev_opt.param_groups[0]["lr"] = lr_t
    ds = WarmupCosineLR(dev_opt, 10, 2)
    ds.step()
    assert dev_opt.param_groups[0]["lr"] is lr_t and lr_t.item() == pytest.approx(0.5)  # updated in place
    with pytest.raises(ValueError):
        WarmupCosineLR(_sgd(), 0, 0)
    with pytest.raises(ValueError):
        s.set_step(-1)


@needs_reference
@pytest.mark.reference
def test_hybrid_schedule_matches_reference():
    ref()
    from training.scheduler import build_warmup_cosine_scheduler as rbuild
    a, b = _Hybrid(), _Hybrid()
    sa = build_warmup_cosine_scheduler(a, 30, 6, min_lr=1e-5, min_muon_lr=1e-3)
    sb = rbuild(b, total_steps=30, warmup_steps=6, min_lr=1e-5, min_muon_lr=1e-3)
    for _ in range(35):
        sa.step()
        sb.step()
        assert a.muon.param_groups[0]["lr"] == pytest.approx(b.muon.param_groups[0]["lr"])
        assert a.adamw.param_groups[0]["lr"] == pytest.approx(b.adamw.param_groups[0]["lr"])


# --------------------------------------------------------------------------- window accounting
def _contrib(loss_sum, n, mtp_sum=None, mtp_n=0.0, lam=0.3, tokens=0):
    return LossContribution(torch.tensor(float(loss_sum)), float(n), None if mtp_sum is None else
                            torch.tensor(float(mtp_sum)), float(mtp_n), lam, 0.0, tokens)


def test_window_loss_is_total_loss_over_total_tokens():
    parts = [_contrib(10.0, 4, 3.0, 2, tokens=5), _contrib(2.0, 1, 1.0, 2, tokens=2),
             _contrib(30.0, 10, 6.0, 4, tokens=11)]
    obj, m = combine_window_loss(parts)
    assert obj.item() == pytest.approx(42.0 / 15 + 0.3 * 10.0 / 8)
    assert m["ntp_loss"] == pytest.approx(42.0 / 15) and m["mtp_loss"] == pytest.approx(10.0 / 8)
    assert m["ntp_tokens"] == 15 and m["mtp_tokens"] == 8 and m["tokens"] == 18
    # the mean of micro-batch means would weight the 1-token batch like the 10-token one
    assert obj.item() != pytest.approx(sum(c.ntp_loss for c in parts) / 3 + 0.3 * 10.0 / 8)


def test_window_loss_contract_errors():
    with pytest.raises(ValueError):
        combine_window_loss([])
    with pytest.raises(ValueError):
        combine_window_loss([_contrib(0.0, 0)])
    with pytest.raises(ValueError):
        combine_window_loss([_contrib(1.0, 1, 1.0, 1, lam=0.3), _contrib(1.0, 1, 1.0, 1, lam=0.5)])
    obj, m = combine_window_loss([_contrib(4.0, 2)])
    assert obj.item() == 2.0 and math.isnan(m["mtp_loss"])


def test_count_batch_tokens_uses_every_mask():
    ids = torch.arange(12).reshape(2, 6)
    batch = {"input_ids": ids, "attention_mask": torch.tensor([[1] * 6, [1] * 4 + [0] * 2]),
             "labels": ids.masked_fill(ids == 3, -100), "loss_mask": torch.ones(2, 6, dtype=torch.bool)}
    batch["loss_mask"][0, 0] = False
    assert count_batch_tokens(batch) == 12 - 2 - 1 - 1
    assert count_batch_tokens({"labels": ids}) == 0


# --------------------------------------------------------------------------- checkpoint files
def test_prune_list_and_latest_pointer(tmp_path):
    for step in (1, 5, 12, 30):
        (tmp_path / f"step_{step}.pt").write_bytes(b"x")
    (tmp_path / "step_40.pt.tmp").write_bytes(b"x")          # an unfinished write is never listed
    names = [p.name for p in list_checkpoints(tmp_path)]
    assert names == ["step_1.pt", "step_5.pt", "step_12.pt", "step_30.pt"]
    assert checkpoint_step(tmp_path / "step_12.pt") == 12 and checkpoint_step("best.pt") == -1
    removed = prune_checkpoints(tmp_path, 2, protect=[tmp_path / "step_1.pt"])
    assert sorted(p.name for p in removed) == ["step_5.pt"]
    assert sorted(p.name for p in list_checkpoints(tmp_path)) == ["step_1.pt", "step_12.pt", "step_30.pt"]
    assert prune_checkpoints(tmp_path, 0) == []
    write_latest_pointer(tmp_path, tmp_path / "step_12.pt")
    assert resolve_resume_path("latest", tmp_path).name == "step_12.pt"
    (tmp_path / "latest").unlink()
    assert resolve_resume_path("latest", tmp_path).name == "step_30.pt"
    assert resolve_resume_path(None) is None and resolve_resume_path("") is None
    assert resolve_resume_path(tmp_path / "step_1.pt").name == "step_1.pt"
    with pytest.raises(FileNotFoundError):
        resolve_resume_path(tmp_path / "missing.pt")
    with pytest.raises(ValueError):
        resolve_resume_path("latest")


def test_rng_state_restores_every_generator():
    import random

    import numpy as np
    st = rng_state()
    a = (random.random(), float(np.random.rand()), torch.rand(3))
    restore_rng_state(st)
    b = (random.random(), float(np.random.rand()), torch.rand(3))
    assert a[0] == b[0] and a[1] == b[1] and torch.equal(a[2], b[2])


# --------------------------------------------------------------------------- EMA
def test_ema_warmup_decay_and_update_rule():
    m = torch.nn.Linear(3, 2, bias=False)
    ema = EMA(m, decay=0.9)
    for n in range(1, 6):
        with torch.no_grad():
            m.weight.add_(1.0)
        before = ema.shadow["weight"].clone()
        assert ema.update(m)
        d = min(0.9, (1.0 + n) / (10.0 + n))
        assert torch.allclose(ema.shadow["weight"], d * before + (1 - d) * m.weight.detach(), atol=1e-6)
    live = m.weight.detach().clone()
    with ema.average_parameters(m):
        assert torch.equal(m.weight, ema.shadow["weight"])
    assert torch.equal(m.weight, live)                  # restored after the context
    with pytest.raises(ValueError):
        EMA(m, decay=1.0)


def test_ema_schedule_and_exclusions():
    m = torch.nn.Linear(3, 2)
    ema = EMA(m, decay=0.5, update_after_step=2, update_every=2, exclude_names=("bias",))
    assert set(ema.shadow) == {"weight"}
    done = [ema.update(m) for _ in range(6)]
    assert done == [False, True, False, True, False, True] and ema.num_updates == 3


def test_ema_state_round_trip():
    m = torch.nn.Linear(3, 2)
    ema = EMA(m, decay=0.5)
    with torch.no_grad():
        m.weight.mul_(2)
    ema.update(m)
    other = EMA(torch.nn.Linear(3, 2), decay=0.5)
    other.load_state_dict(ema.state_dict())
    a, b = torch.nn.Linear(3, 2), torch.nn.Linear(3, 2)
    ema.copy_to(a)
    other.copy_to(b)
    assert torch.equal(a.weight, b.weight) and torch.equal(a.bias, b.bias)
    assert other.num_updates == 1


# --------------------------------------------------------------------------- loggers
def test_jsonl_and_memory_loggers(tmp_path):
    log = JSONLLogger(tmp_path / "logs" / "train.jsonl")
    log.log(1, {"loss": torch.tensor(2.5), "name": "a", "skip": [1, 2]})
    log.log(2, {"loss": 1.5})
    lines = [json.loads(x) for x in (tmp_path / "logs" / "train.jsonl").read_text().splitlines()]
    assert lines == [{"step": 1, "loss": 2.5, "name": "a"}, {"step": 2, "loss": 1.5}]
    JSONLLogger(tmp_path / "off.jsonl", enabled=False).log(1, {"a": 1})
    assert not (tmp_path / "off.jsonl").exists()
    mem = MemoryLogger()
    mem.log(3, {"x": 1})
    assert mem.records == [{"step": 3, "x": 1}]


@needs_reference
@pytest.mark.reference
def test_checkpoints_move_between_the_implementations(tmp_path):
    """A format-v2 checkpoint written by the reference loads into this package's model (and the
    reverse) with identical logits afterwards."""
    ref()
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as rcfg
    from src.kimi_k3_mini import KimiK3 as RK
    from training.checkpoints import load_checkpoint as ref_load
    from training.checkpoints import save_checkpoint as ref_save
    from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
    from kimi_k3_b200.train.checkpoints import load_checkpoint, save_checkpoint
    torch.manual_seed(0)
    theirs = RK(rcfg(enable_vision=False))
    ours = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False))
    with torch.no_grad():
        for p in theirs.parameters():
            p.add_(0.01 * torch.randn_like(p))
    ref_save(tmp_path / "ref.pt", theirs, epoch=1, global_step=7)
    load_checkpoint(tmp_path / "ref.pt", ours)
    ids = torch.randint(5, 128, (2, 9))
    theirs.eval()
    ours.eval()
    with torch.no_grad():
        assert torch.equal(ours(input_ids=ids).logits, theirs(input_ids=ids).logits)
        for p in ours.parameters():
            p.mul_(0.5)
    save_checkpoint(tmp_path / "ours.pt", ours, epoch=2, global_step=9)
    back = RK(rcfg(enable_vision=False)).eval()
    ref_load(tmp_path / "ours.pt", back)
    with torch.no_grad():
        assert torch.equal(back(input_ids=ids).logits, ours(input_ids=ids).logits)
