"""The generic Muon / Muon + AdamW / AdamW optimizers against the reference's
(``training/muon_optimizer.py``, ``training/adam_optimizer.py``)."""
import pytest
import torch
import torch.nn as nn

from _oracle import needs_reference, ref


def _model():
    from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
    torch.manual_seed(0)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False))


class _Toy(nn.Module):
    def __init__(self):
        super().__init__()
        self.embed = nn.Embedding(11, 6)
        self.proj_a = nn.Linear(6, 8)
        self.proj_b = nn.Linear(6, 8, bias=False)
        self.tall = nn.Linear(3, 9, bias=False)
        self.norm = nn.LayerNorm(8)
        self.lm_head = nn.Linear(8, 11, bias=False)
        self.alpha_gate = nn.Parameter(torch.ones(4, 4))
        self.frozen = nn.Parameter(torch.ones(2, 2), requires_grad=False)


@needs_reference
@pytest.mark.parametrize("make", [_model, _Toy])
def test_parameter_groups_match_reference(make):
    ref()
    from training.adam_optimizer import build_adamw_parameter_groups as ref_adamw_groups
    from training.muon_optimizer import build_muon_adamw_parameter_groups as ref_groups
    from kimi_k3_b200.train.legacy import build_adamw_parameter_groups, build_muon_adamw_parameter_groups
    model = make()
    _, _, meta = build_muon_adamw_parameter_groups(model, 0.1, 0.01)
    _, _, ref_meta = ref_groups(model, 0.1, 0.01)
    for key in ("muon_names", "adamw_decay_names", "adamw_no_decay_names", "num_muon_params", "num_adamw_params",
                "total_trainable_params"):
        assert meta[key] == ref_meta[key], key
    _, info = build_adamw_parameter_groups(model, 0.1)
    _, ref_info = ref_adamw_groups(model, 0.1)
    assert info == ref_info


@needs_reference
@pytest.mark.parametrize("shape", [(5, 7), (9, 3), (4, 4)])
def test_zeropower_matches_reference(shape):
    ref()
    from training.muon_optimizer import zeropower_via_newtonschulz5 as ref_zp
    from kimi_k3_b200.train.legacy import zeropower_via_newtonschulz5
    torch.manual_seed(1)
    g = torch.randn(*shape)
    assert (zeropower_via_newtonschulz5(g) - ref_zp(g)).abs().max().item() < 2e-5
    assert torch.equal(zeropower_via_newtonschulz5(torch.zeros(shape)), torch.zeros(shape))
    with pytest.raises(FloatingPointError):
        zeropower_via_newtonschulz5(torch.full(shape, float("nan")))


@needs_reference
def test_hybrid_steps_match_reference():
    """Three Muon + AdamW steps from the same weights and gradients land on the same parameters
    (equal-shape matrices are orthogonalised as one batch here, one by one in the reference)."""
    ref()
    from training.muon_optimizer import build_muon_adamw_optimizer as ref_build
    from kimi_k3_b200.train.legacy import build_muon_adamw_optimizer
    a, b = _Toy(), _Toy()
    b.load_state_dict(a.state_dict())
    opt, _ = build_muon_adamw_optimizer(a, learning_rate=1e-2, muon_lr=2e-2, muon_weight_decay=0.01)
    ref_opt, _ = ref_build(b, learning_rate=1e-2, muon_lr=2e-2, muon_weight_decay=0.01)
    g = torch.Generator().manual_seed(3)
    for step in range(3):
        for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
            if pa.requires_grad:
                grad = torch.randn(pa.shape, generator=g)
                pa.grad, pb.grad = grad.clone(), grad.clone()
        opt.step()
        ref_opt.step()
        if step == 1:
            opt.set_lr(5e-3, muon_lr=1e-2)
            ref_opt.set_lr(5e-3, muon_lr=1e-2)
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert (pa - pb).abs().max().item() < 1e-5, n


def test_hybrid_state_dict_roundtrip_and_validation():
    from kimi_k3_b200.train.legacy import HybridMuonAdamW, Muon, build_muon_adamw_optimizer
    model = _Toy()
    opt, meta = build_muon_adamw_optimizer(model, learning_rate=1e-3)
    assert meta["optimizer_type"] == "muon_adamw" and meta["num_muon_tensors"] == 3
    for p in model.parameters():
        if p.requires_grad:
            p.grad = torch.ones_like(p)
    opt.step()
    state = opt.state_dict()
    fresh, _ = build_muon_adamw_optimizer(model, learning_rate=1e-3)
    fresh.load_state_dict(state)
    assert isinstance(fresh, HybridMuonAdamW)
    assert len(fresh.muon.state) == len(opt.muon.state) and len(fresh.adamw.state) == len(opt.adamw.state)
    with pytest.raises(ValueError):
        Muon([nn.Parameter(torch.ones(3))])
    with pytest.raises(ValueError):
        opt.set_lr(-1.0)
