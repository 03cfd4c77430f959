"""Optimizer oracles on CPU: Newton-Schulz, bucketed Muon vs per-matrix Muon, device-flag skip,
per-head orthogonalisation, scheduler; reference parity where the reference is installed."""
import math

import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.train.optimizer import (KimiOptimizerConfig, batched_newton_schulz, build_kimi_optimizer,
                                          zeropower_via_newton_schulz)
from kimi_k3_b200.train.scheduler import WarmupCosineLR


def _model(seed=0, vision=False):
    torch.manual_seed(seed)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=vision)).double()


def _loss(model, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(5, 128, (2, 24), generator=g)
    return model(input_ids=ids, labels=ids, use_mtp=True).loss


def test_batched_ns_equals_single_matrix():
    torch.manual_seed(0)
    x = torch.randn(5, 12, 20)
    b = batched_newton_schulz(x, dtype=torch.float32)
    for i in range(5):
        assert max_diff(b[i], zeropower_via_newton_schulz(x[i], output_dtype=torch.float32)) < 1e-5
    tall = batched_newton_schulz(x.transpose(1, 2).contiguous(), dtype=torch.float32)
    assert max_diff(tall, b.transpose(1, 2)) < 1e-5
    assert batched_newton_schulz(torch.zeros(2, 4, 6), dtype=torch.float32).abs().max() == 0


@needs_reference
@pytest.mark.reference
def test_ns_matches_reference():
    ref()
    from training.optimizer.newton_schulz import zeropower_via_newton_schulz as rns
    torch.manual_seed(1)
    for shape in ((16, 40), (40, 16), (7, 7)):
        x = torch.randn(*shape)
        assert max_diff(zeropower_via_newton_schulz(x), rns(x)) < 1e-5


def test_bucketed_step_equals_per_matrix_step():
    """All gradients present -> bucket path; forcing the sparse path must give identical params."""
    a, b = _model(), _model()
    oa, _ = build_kimi_optimizer(a, KimiOptimizerConfig(muon_lr=0.02, adamw_lr=1e-3))
    ob, _ = build_kimi_optimizer(b, KimiOptimizerConfig(muon_lr=0.02, adamw_lr=1e-3))
    for step in range(2):
        for model, opt, sparse in ((a, oa, False), (b, ob, True)):
            opt.zero_grad()
            _loss(model, step).backward()
            if sparse:
                opt.muon.step = opt.muon._step_sparse  # force the matrix-by-matrix path
            opt.step()
        # fp32 Newton-Schulz: batched and single-matrix GEMMs round differently
        assert max(max_diff(p, q) for p, q in zip(a.parameters(), b.parameters())) < 1e-5


def test_device_skip_flag_is_a_no_op():
    m = _model()
    opt, _ = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=0.02, kind="muon_adamw"))
    _loss(m, 0).backward()
    opt.step()  # creates momentum state
    before = [p.detach().clone() for p in opt.muon.param_groups[0]["params"]]
    mom = [opt.muon.state[p]["momentum_buffer"].clone() for p in opt.muon.param_groups[0]["params"]]
    opt.zero_grad()
    _loss(m, 1).backward()
    for p in opt.muon.param_groups[0]["params"]:
        p.grad[..., 0] = float("nan")
    opt.muon.step(skip=torch.tensor(True))
    for p, b0, m0 in zip(opt.muon.param_groups[0]["params"], before, mom):
        assert torch.equal(p, b0)
        assert torch.equal(opt.muon.state[p]["momentum_buffer"], m0)


@needs_reference
@pytest.mark.reference
def test_text_only_training_matches_reference_optimizer():
    """No unused parameters: every Muon matrix goes through the bucketed path."""
    import dataclasses
    ref()
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as ref_cfg
    from src.kimi_k3_mini import KimiK3 as RefK3
    from training.optimizer.config import KimiOptimizerConfig as RefCfg
    from training.optimizer.hybrid import build_kimi_optimizer as ref_build
    torch.manual_seed(2)
    theirs = RefK3(dataclasses.replace(ref_cfg(), enable_vision=False)).double()
    ours = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double()
    ours.load_state_dict(theirs.state_dict())
    kw = dict(adamw_lr=1e-3, muon_lr=2e-2, weight_decay=0.1)
    o1, _ = ref_build(theirs, RefCfg(**kw))
    o2, _ = build_kimi_optimizer(ours, KimiOptimizerConfig(**kw))
    # One step: later steps amplify fp32 Newton-Schulz rounding through the gradients.
    for step in range(1):
        for model, opt in ((theirs, o1), (ours, o2)):
            opt.zero_grad()
            _loss(model, step).backward()
            opt.step()
    theirs_p = dict(theirs.named_parameters())
    from _oracle import expand_expert_grads
    ours_p = expand_expert_grads((n, p.detach()) for n, p in ours.named_parameters())
    assert max(max_diff(theirs_p[n], ours_p[n]) for n in theirs_p) < 1e-6


def test_warmup_cosine_schedule_shape():
    m = _model()
    opt, _ = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=0.02, adamw_lr=1e-3))
    sch = WarmupCosineLR(opt, total_steps=100, warmup_steps=10, min_lr=1e-4, prepare_first_update=True)
    lrs = []
    for _ in range(100):
        lrs.append(opt.get_lrs()["adamw_lr"])
        sch.step()
    assert lrs[0] < lrs[9] and max(lrs) <= 1e-3 + 1e-12 and lrs[-1] < lrs[50] and min(lrs[10:]) >= 1e-4 - 1e-12


@needs_reference
@pytest.mark.reference
def test_scheduler_matches_reference():
    ref()
    from training.scheduler import WarmupCosineLR as RefLR
    from training.optimizer.config import KimiOptimizerConfig as RefCfg
    from training.optimizer.hybrid import build_kimi_optimizer as ref_build
    m1, m2 = _model(), _model()
    import inspect
    o1, _ = ref_build(m1, RefCfg(muon_lr=0.02, adamw_lr=1e-3))
    o2, _ = build_kimi_optimizer(m2, KimiOptimizerConfig(muon_lr=0.02, adamw_lr=1e-3))
    params = inspect.signature(RefLR.__init__).parameters
    kw = {k: v for k, v in dict(total_steps=50, warmup_steps=5, min_lr=1e-4).items() if k in params}
    s1, s2 = RefLR(o1, **kw), WarmupCosineLR(o2, **kw)
    for _ in range(50):
        a, b = o1.get_lrs() if hasattr(o1, "get_lrs") else None, o2.get_lrs()
        if a is not None:
            assert abs(a["adamw_lr"] - b["adamw_lr"]) < 1e-15 and abs(a["muon_lr"] - b["muon_lr"]) < 1e-15
        s1.step()
        s2.step()


def test_newton_schulz_reformulation_and_transposed_output():
    """``(aI + bG + cG^2) X`` equals ``aX + (bG + cG^2) X`` (fp64), and ``transpose_out`` returns
    the transpose of the plain result."""
    import torch
    from kimi_k3_b200.train.optimizer import NS_COEFFS, newton_schulz_iterations
    torch.manual_seed(0)
    x = torch.randn(3, 16, 40, dtype=torch.float64)
    x = x / x.flatten(1).norm(dim=1)[:, None, None]
    a, b, c = NS_COEFFS
    w = x.clone()
    for _ in range(5):
        g = w @ w.transpose(-2, -1)
        w = a * w + (b * g + c * g @ g) @ w
    got = newton_schulz_iterations(x.clone(), 5)
    assert torch.allclose(got, w, atol=1e-10, rtol=1e-10)
    got_t = newton_schulz_iterations(x.clone(), 5, transpose_out=True)
    assert got_t.is_contiguous() and torch.allclose(got_t, w.transpose(-2, -1), atol=1e-10, rtol=1e-10)
