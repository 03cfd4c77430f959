"""Stable LatentMoE checks on CPU: config, router equations, Quantile Balancing, expert layout, module.

Oracles: the router equations of ``src/stable_latent_moe/router.py:54-109`` (biased selection,
unbiased renormalised weights, top-(k+1) cutoff), the QB rule of ``quantile_balancing.py:19-57``
(``b = -q + mean(q)`` at quantile ``1 - k/E``), the histogram approximation of ``histogram.py`` and the
reference modules in float64.
"""
import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.moe import (ExactQuantileBalancer, GroupedRoutedExperts, HistogramQuantileBalancer,
                                     StableLatentMoE, StableLatentMoEConfig, TopKRouter, policy_dtype)

F64 = torch.float64


def _cfg(**kw):
    base = dict(d_model=16, latent_dim=8, num_shared_experts=2, num_routed_experts=6, routed_experts_per_token=2,
                shared_expert_hidden_dim=20, routed_expert_hidden_dim=12)
    base.update(kw)
    return StableLatentMoEConfig(**base)


def _module(seed=0, **kw):
    torch.manual_seed(seed)
    return StableLatentMoE(_cfg(**kw)).double()


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("bad", [
    dict(num_shared_experts=0),
    dict(routed_experts_per_token=7),
    dict(routed_experts_per_token=6),            # QB needs k < E
    dict(latent_dim=0),
    dict(beta_gate=0.0),
    dict(router_eps=0.0),
    dict(routing_backend="loop"),
    dict(quantile_backend="sketch"),
    dict(router_logits_dtype="bfloat16"),
    dict(histogram_num_bins=1),
    dict(histogram_min_margin=1.0, histogram_max_margin=1.0),
])
def test_config_rejects_invalid_values(bad):
    with pytest.raises(ValueError):
        _cfg(**bad)


def test_config_canonical_and_round_trip():
    k3 = StableLatentMoEConfig.kimi_k3()
    assert (k3.d_model, k3.latent_dim, k3.num_routed_experts, k3.top_k) == (7168, 3584, 896, 16)
    assert k3.num_shared_experts == 2
    c = _cfg(quantile_backend="histogram")
    assert StableLatentMoEConfig.from_dict(c.to_dict()) == c
    # without QB, k == E is allowed
    assert _cfg(routed_experts_per_token=6, enable_quantile_balancing=False).top_k == 6
    assert policy_dtype(torch.bfloat16, "float32") == torch.float32
    assert policy_dtype(torch.bfloat16, "input") == torch.bfloat16
    assert policy_dtype(torch.float64, "float32") == torch.float64


@needs_reference
@pytest.mark.reference
def test_config_dict_matches_reference_schema():
    ref()
    from src.stable_latent_moe.config import StableLatentMoEConfig as RC
    ours = _cfg(quantile_backend="histogram", histogram_num_bins=64).to_dict()
    assert RC(**ours).to_dict() == ours
    assert RC.kimi_k3().to_dict() == StableLatentMoEConfig.kimi_k3().to_dict()


# --------------------------------------------------------------------------- router
def _router(seed=1, **kw):
    torch.manual_seed(seed)
    return TopKRouter(_cfg(**kw)).double()


def test_router_selects_by_biased_scores_and_weights_by_raw_scores():
    r = _router()
    with torch.no_grad():
        r.routing_bias.copy_(torch.tensor([0.5, -0.5, 0.0, 0.2, -0.1, 0.3]))
    x = torch.randn(30, 16, dtype=F64)
    out = r(x, need_qb_cutoff=True, return_full_scores=True)
    raw = torch.sigmoid(x @ r.projection.weight.T)
    biased = raw + r.routing_bias.double()
    vals, idx = biased.topk(3, dim=-1)
    assert torch.equal(out.selected_experts, idx[:, :2])
    sel_raw = raw.gather(1, idx[:, :2])
    assert max_diff(out.selected_raw_scores, sel_raw) < 1e-14
    assert max_diff(out.selected_weights, sel_raw / sel_raw.sum(-1, keepdim=True)) < 1e-14
    assert max_diff(out.selected_weights.sum(-1), torch.ones(30, dtype=F64)) < 1e-14
    assert max_diff(out.cutoff_k_plus_one, vals[:, 2]) < 1e-14
    assert torch.equal(out.expert_load, torch.bincount(idx[:, :2].reshape(-1), minlength=6))
    assert out.expert_load.sum().item() == 60
    assert max_diff(out.biased_scores, biased) < 1e-14 and max_diff(out.raw_scores, raw) < 1e-14


def test_router_bias_is_a_buffer_and_commit_validates():
    r = _router()
    assert "routing_bias" in dict(r.named_buffers())
    assert "routing_bias" not in dict(r.named_parameters())
    r.commit_next_bias(torch.arange(6, dtype=F64))
    assert r.routing_bias.tolist() == list(range(6))
    with pytest.raises(ValueError):
        r.commit_next_bias(torch.zeros(5))
    with pytest.raises(ValueError):
        r.commit_next_bias(torch.full((6,), float("nan")))
    with pytest.raises(ValueError):
        r(torch.randn(3, 15, dtype=F64))
    with pytest.raises(ValueError):
        TopKRouter(_cfg(routed_experts_per_token=6, enable_quantile_balancing=False))(
            torch.randn(2, 16), need_qb_cutoff=True)


def test_a_large_bias_forces_an_expert_into_every_selection():
    r = _router()
    with torch.no_grad():
        r.routing_bias[4] = 10.0
    out = r(torch.randn(25, 16, dtype=F64))
    assert (out.selected_experts == 4).any(-1).all()
    assert out.expert_load[4].item() == 25


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("router_bias", [False, True])
def test_router_matches_reference(router_bias):
    ref()
    from src.stable_latent_moe.config import StableLatentMoEConfig as RC
    from src.stable_latent_moe.router import TopKRouter as RR
    ours = _router(2, router_bias=router_bias)
    theirs = RR(RC(**_cfg(router_bias=router_bias).to_dict())).double()
    if router_bias:
        torch.nn.init.normal_(ours.projection.bias)
    with torch.no_grad():
        ours.routing_bias.normal_(0, 0.1)
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(17, 16, dtype=F64)
    a = ours(x, need_qb_cutoff=True, return_full_scores=True)
    b = theirs(x, need_qb_cutoff=True, return_full_scores=True)
    assert torch.equal(a.selected_experts, b.selected_experts)
    assert torch.equal(a.expert_load, b.expert_load)
    for name in ("selected_raw_scores", "selected_weights", "cutoff_k_plus_one", "raw_scores", "biased_scores"):
        assert max_diff(getattr(a, name), getattr(b, name)) < 1e-14, name


# --------------------------------------------------------------------------- Quantile Balancing
def _scores(m=200, e=6, seed=3):
    g = torch.Generator().manual_seed(seed)
    raw = torch.sigmoid(torch.randn(m, e, generator=g, dtype=F64) + torch.linspace(-1, 1, e, dtype=F64))
    return raw


def _cutoffs(raw, bias, k):
    return (raw + bias).topk(k + 1, dim=-1).values[:, k]


def test_exact_balancer_equation_and_zero_mean():
    raw = _scores()
    bias = torch.zeros(6, dtype=F64)
    cut = _cutoffs(raw, bias, 2)
    qb = ExactQuantileBalancer(6, 2)
    assert qb.target_quantile == pytest.approx(1 - 2 / 6)
    up = qb.compute_next_bias(raw, cut, bias)
    margins = raw - cut[:, None]
    q = torch.quantile(margins, 1 - 2 / 6, dim=0)
    assert max_diff(up.quantiles, q) < 1e-14
    assert max_diff(up.next_bias, -q + q.mean()) < 1e-14
    assert abs(up.next_bias.sum().item()) < 1e-12
    assert max_diff(up.margin_min, margins.amin(0)) == 0.0 and up.num_tokens == 200
    with pytest.raises(ValueError):
        ExactQuantileBalancer(6, 6)
    with pytest.raises(ValueError):
        qb.compute_next_bias(raw[:, :5], cut, bias)


def test_exact_balancing_evens_out_the_expert_load():
    raw = _scores(m=3000)
    k = 2
    bias = torch.zeros(6, dtype=F64)
    load0 = torch.bincount((raw + bias).topk(k, -1).indices.reshape(-1), minlength=6).double()
    qb = ExactQuantileBalancer(6, k)
    for _ in range(4):
        bias = qb.compute_next_bias(raw, _cutoffs(raw, bias, k), bias).next_bias
    load = torch.bincount((raw + bias).topk(k, -1).indices.reshape(-1), minlength=6).double()
    cv = lambda x: (x.std() / x.mean()).item()  # noqa: E731
    assert cv(load) < 0.25 * cv(load0)
    assert (load - 1000).abs().max().item() < 150


@pytest.mark.parametrize("bins", [64, 256, 1024])
def test_histogram_balancer_approximates_exact_within_a_bin(bins):
    raw = _scores(m=500)
    bias = torch.zeros(6, dtype=F64)
    cut = _cutoffs(raw, bias, 2)
    hist = HistogramQuantileBalancer(6, 2, bins, -2.0, 2.0)
    hist.accumulate(raw[:250], cut[:250])
    hist.accumulate(raw[250:], cut[250:])
    assert hist.counts.sum(-1).tolist() == [500] * 6
    assert hist.underflow.sum().item() == 0 and hist.overflow.sum().item() == 0
    approx = hist.compute_next_bias(bias)
    exact = ExactQuantileBalancer(6, 2).compute_next_bias(raw, cut, bias)
    assert max_diff(approx.quantiles, exact.quantiles) <= 2 * hist.bin_width
    assert abs(approx.next_bias.sum().item()) < 1e-5
    hist.reset()
    assert hist.counts.sum().item() == 0
    with pytest.raises(ValueError):
        hist.compute_next_bias(bias)


def test_histogram_counts_out_of_range_margins():
    hist = HistogramQuantileBalancer(2, 1, 8, -1.0, 1.0)
    raw = torch.tensor([[0.0, 5.0], [0.0, -5.0], [0.0, 0.999]], dtype=F64)
    hist.accumulate(raw, torch.zeros(3, dtype=F64))
    assert hist.overflow.tolist() == [0, 1] and hist.underflow.tolist() == [0, 1]
    assert hist.counts.sum(-1).tolist() == [3, 3]  # clamped into the edge bins as well
    assert hist.counts[1, -1].item() == 2 and hist.counts[1, 0].item() == 1


@needs_reference
@pytest.mark.reference
def test_balancers_match_reference():
    ref()
    from src.stable_latent_moe.histogram import HistogramQuantileBalancer as RH
    from src.stable_latent_moe.quantile_balancing import ExactQuantileBalancer as RE
    raw = _scores(m=300)
    bias = torch.linspace(-0.1, 0.1, 6, dtype=F64)
    cut = _cutoffs(raw, bias, 2)
    a, b = ExactQuantileBalancer(6, 2).compute_next_bias(raw, cut, bias), RE(6, 2).compute_next_bias(raw, cut, bias)
    assert max_diff(a.next_bias, b.next_bias) < 1e-14
    ours, theirs = HistogramQuantileBalancer(6, 2, 128, -2.0, 2.0), RH(6, 2, 128, -2.0, 2.0)
    ours.accumulate(raw, cut)
    theirs.accumulate(raw, cut)
    assert torch.equal(ours.counts, theirs.counts)
    assert max_diff(ours.compute_next_bias(bias).next_bias, theirs.compute_next_bias(bias).next_bias) < 1e-6


def test_balance_window_lifecycle():
    m = _module(4)
    x = torch.randn(3, 5, 16, dtype=F64)
    m.eval()
    with pytest.raises(RuntimeError):
        m.begin_balance_accumulation()
    with pytest.raises(RuntimeError):
        m(x, update_routing_bias=True)
    m.train()
    with pytest.raises(RuntimeError):
        m.finalize_and_commit_balance()
    m.begin_balance_accumulation()
    with pytest.raises(RuntimeError):
        m.begin_balance_accumulation()
    with pytest.raises(RuntimeError):
        m.finalize_and_commit_balance()  # nothing accumulated yet
    assert m._balance_accumulating  # a failed finalize leaves the window open
    before = m.routing_bias.clone()
    m(x)
    assert max_diff(m.routing_bias, before) == 0.0  # accumulation never commits by itself
    m.discard_balance_accumulation()
    assert not m._balance_accumulating
    with pytest.raises(RuntimeError):
        _module(4, enable_quantile_balancing=False).begin_balance_accumulation()


@pytest.mark.parametrize("backend", ["exact", "histogram"])
def test_window_over_micro_batches_equals_one_update_on_their_union(backend):
    a, b = _module(5, quantile_backend=backend), _module(5, quantile_backend=backend)
    xs = [torch.randn(2, 7, 16, dtype=F64) for _ in range(3)]
    a.begin_balance_accumulation()
    for x in xs:
        a(x)
    up = a.finalize_and_commit_balance()
    b(torch.cat(xs, 0), update_routing_bias=True)
    assert max_diff(a.routing_bias, b.routing_bias) < 1e-12
    assert max_diff(up.next_bias.to(F64), a.routing_bias.to(F64)) == 0.0


def test_keep_old_leaves_the_bias_unchanged():
    m = _module(6)
    with torch.no_grad():
        m.router.routing_bias.copy_(torch.linspace(-0.2, 0.2, 6))
    before = m.routing_bias.clone()
    m.begin_balance_accumulation()
    m(torch.randn(2, 6, 16, dtype=F64))
    m.finalize_and_commit_balance(keep_old=torch.tensor(True))
    assert max_diff(m.routing_bias, before) == 0.0


# --------------------------------------------------------------------------- experts and module
def test_grouped_experts_state_dict_uses_per_expert_keys():
    ex = GroupedRoutedExperts(3, 4, 5, 4.0, 25.0, 0.02)
    sd = ex.state_dict()
    assert sorted(sd) == sorted(f"{e}.transform.{n}.weight" for e in range(3) for n in ("gate_proj", "up_proj",
                                                                                       "down_proj"))
    assert sd["1.transform.gate_proj.weight"].shape == (5, 4)
    assert sd["2.transform.down_proj.weight"].shape == (4, 5)
    ex2 = GroupedRoutedExperts(3, 4, 5, 4.0, 25.0, 0.02)
    ex2.load_state_dict(sd)
    x = torch.randn(7, 4)
    for e in range(3):
        assert max_diff(ex.expert_forward(e, x), ex2.expert_forward(e, x)) == 0.0
    assert len(ex) == 3


def test_module_output_is_shared_plus_normalised_routed_branch():
    m = _module(7)
    x = torch.randn(2, 5, 16, dtype=F64)
    out = m(x, return_branch_outputs=True, return_router_diagnostics=True)
    assert max_diff(out.hidden_states, out.shared_output + out.routed_output) < 1e-14
    flat = x.reshape(-1, 16)
    shared = sum(e.transform(flat) for e in m.shared_experts)
    assert max_diff(out.shared_output.reshape(-1, 16), shared) < 1e-14
    latent = m.down_projection(flat)
    ro = out.router_output
    agg = torch.zeros_like(latent)
    for t in range(flat.shape[0]):
        for j in range(2):
            agg[t] += ro.selected_weights[t, j] * m.routed_experts.expert_forward(int(ro.selected_experts[t, j]),
                                                                                  latent[t:t + 1])[0]
    want = m.up_projection(m.routed_aggregate_norm(agg))
    assert max_diff(out.routed_output.reshape(-1, 16), want) < 1e-13
    diag = vars(out.diagnostics)
    assert diag and all(torch.isfinite(v).all() for v in diag.values() if torch.is_tensor(v))
    assert diag["num_tokens"] == 10 and diag["num_assignments"] == 20


def test_every_parameter_receives_a_gradient():
    m = _module(8, num_routed_experts=3, routed_experts_per_token=2)
    x = torch.randn(4, 8, 16, dtype=F64)
    m(x).square().sum().backward()
    for name, p in m.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name
        assert p.grad.abs().sum() > 0, name


def test_bf16_dtype_policies():
    m = _module(9).to(torch.bfloat16)
    x = torch.randn(2, 4, 16).to(torch.bfloat16)
    out = m(x, return_router_diagnostics=True)
    assert out.hidden_states.dtype == torch.bfloat16
    assert out.router_output.selected_weights.dtype == torch.float32
    m2 = StableLatentMoE(_cfg(routing_weights_dtype="input", router_logits_dtype="input")).to(torch.bfloat16)
    assert m2(x, return_router_diagnostics=True).router_output.selected_weights.dtype == torch.bfloat16


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("routing_backend", ["reference", "vectorized"])
def test_module_outputs_diagnostics_and_gradients_match_reference(routing_backend):
    ref()
    from src.stable_latent_moe.config import StableLatentMoEConfig as RC
    from src.stable_latent_moe.module import StableLatentMoE as RM
    kw = dict(routing_backend=routing_backend, projection_bias=True, router_bias=True)
    torch.manual_seed(10)
    theirs = RM(RC(**_cfg(**kw).to_dict())).double()
    ours = StableLatentMoE(_cfg(**kw)).double()
    ours.load_state_dict(theirs.state_dict())
    x = torch.randn(3, 5, 16, dtype=F64)
    a = ours(x, return_router_diagnostics=True, return_branch_outputs=True)
    b = theirs(x, return_router_diagnostics=True, return_branch_outputs=True)
    assert max_diff(a.hidden_states, b.hidden_states) < 1e-13
    assert max_diff(a.shared_output, b.shared_output) < 1e-13
    da, db = vars(a.diagnostics), vars(b.diagnostics)
    assert set(da) == set(db)
    for key, want in db.items():
        if torch.is_tensor(want):
            assert max_diff(da[key], want) < 1e-6 * (1 + want.double().abs().max().item()), key
        else:
            assert da[key] == want, key
    g = torch.randn_like(a.hidden_states)
    a.hidden_states.backward(g)
    b.hidden_states.backward(g)
    from _oracle import expand_expert_grads
    ours_g = expand_expert_grads((n, p.grad) for n, p in ours.named_parameters())
    for n, p in theirs.named_parameters():
        if p.grad is not None:
            assert max_diff(ours_g[n], p.grad) < 1e-12, n
