"""Layer oracles on CPU (float64) against the reference modules: MLA, Stable LatentMoE, AttnRes."""
import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.mla import GatedMLA, GatedMLAConfig, absorbed_latent_decode, manual_causal_attention
from kimi_k3_b200.models.moe import (GroupedRoutedExperts, StableLatentMoE, StableLatentMoEConfig,
                                     reference_sparse_dispatch, vectorized_sparse_dispatch)


# --------------------------------------------------------------------------- MLA
def _mla_cfg(**kw):
    return dict(d_model=32, num_heads=4, q_head_dim=8, v_head_dim=8, kv_latent_dim=16, **kw)


def test_mla_prefill_decode_equals_full():
    torch.manual_seed(0)
    m = GatedMLA(GatedMLAConfig(**_mla_cfg())).double().eval()
    x = torch.randn(2, 15, 32, dtype=torch.float64)
    full = m(x).hidden_states
    pre = m(x[:, :9], use_cache=True)
    cache, outs = pre.cache, [pre.hidden_states]
    for i in range(9, 15):
        st = m(x[:, i:i + 1], cache=cache, use_cache=True)
        cache = st.cache
        outs.append(st.hidden_states)
    assert max_diff(torch.cat(outs, 1), full) < 1e-12


def test_mla_right_padding_matches_unpadded():
    torch.manual_seed(1)
    m = GatedMLA(GatedMLAConfig(**_mla_cfg())).double()
    x = torch.randn(2, 12, 32, dtype=torch.float64)
    mask = torch.ones(2, 12, dtype=torch.bool)
    mask[1, 7:] = False
    out = m(x, attention_mask=mask).hidden_states
    short = m(x[1:, :7]).hidden_states
    assert max_diff(out[1:, :7], short) < 1e-12
    assert out[1, 7:].abs().max().item() == 0.0


def test_absorbed_decode_equals_expanded_attention():
    torch.manual_seed(2)
    m = GatedMLA(GatedMLAConfig(**_mla_cfg())).double().eval()
    x = torch.randn(2, 10, 32, dtype=torch.float64)
    proj = m.projections(x)
    b, t, h = 2, 10, 4
    mask = torch.ones(b, t, dtype=torch.bool)
    mask[1, 8:] = False
    kv = m.projections.latent_kv
    got = absorbed_latent_decode(proj.query[:, -1:], proj.latent_kv, mask, kv.key_up.weight, kv.value_up.weight, h)
    s = torch.einsum("bhd,bkhd->bhk", proj.query[:, -1], proj.key) / 8 ** 0.5
    s = s.masked_fill(~mask[:, None, :], float("-inf"))
    want = torch.einsum("bhk,bkhd->bhd", torch.softmax(s, -1), proj.value)
    assert max_diff(got[:, 0], want) < 1e-12


@needs_reference
@pytest.mark.reference
def test_mla_module_matches_reference():
    ref()
    from src.mla.config import GatedMLAConfig as RC
    from src.mla.gated_mla import GatedMLA as RM
    torch.manual_seed(3)
    theirs = RM(RC(**_mla_cfg())).double()
    ours = GatedMLA(GatedMLAConfig(**_mla_cfg())).double()
    ours.load_state_dict(theirs.state_dict())
    x = torch.randn(3, 11, 32, dtype=torch.float64, requires_grad=True)
    mask = torch.ones(3, 11, dtype=torch.bool)
    mask[2, 5:] = False
    a = theirs(x, attention_mask=mask).hidden_states
    b = ours(x, attention_mask=mask).hidden_states
    assert max_diff(a, b) < 1e-12
    ga = torch.autograd.grad(a.sum(), x)[0]
    gb = torch.autograd.grad(b.sum(), x)[0]
    assert max_diff(ga, gb) < 1e-12


def test_manual_attention_is_causal():
    torch.manual_seed(4)
    q, k, v = (torch.randn(1, 2, 9, 4, dtype=torch.float64) for _ in range(3))
    o = manual_causal_attention(q, k, v)
    v2 = v.clone()
    v2[:, :, 6:] += 3
    o2 = manual_causal_attention(q, k, v2)
    o = o if torch.is_tensor(o) else o[0]
    o2 = o2 if torch.is_tensor(o2) else o2[0]
    assert max_diff(o[:, :, :6], o2[:, :, :6]) == 0.0


# --------------------------------------------------------------------------- MoE
def _moe_cfg(**kw):
    base = dict(d_model=16, latent_dim=8, num_shared_experts=1, num_routed_experts=6, routed_experts_per_token=2,
                shared_expert_hidden_dim=20, routed_expert_hidden_dim=12)
    base.update(kw)
    return base


def test_reference_and_vectorized_dispatch_agree():
    torch.manual_seed(5)
    ex = GroupedRoutedExperts(6, 8, 12, 4.0, 25.0, 0.3).double()
    lat = torch.randn(40, 8, dtype=torch.float64)
    sel = torch.stack([torch.randperm(6)[:2] for _ in range(40)])
    w = torch.rand(40, 2, dtype=torch.float64)
    a = reference_sparse_dispatch(lat, ex, sel, w, accumulation_dtype=torch.float64)
    b = vectorized_sparse_dispatch(lat, ex, sel, w, accumulation_dtype=torch.float64)
    assert max_diff(a, b) < 1e-12


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("backend", ["exact", "histogram"])
def test_moe_module_and_quantile_balancing_match_reference(backend):
    ref()
    from src.stable_latent_moe.config import StableLatentMoEConfig as RC
    from src.stable_latent_moe.module import StableLatentMoE as RM
    torch.manual_seed(6)
    theirs = RM(RC(**_moe_cfg(quantile_backend=backend))).double()
    ours = StableLatentMoE(StableLatentMoEConfig(**_moe_cfg(quantile_backend=backend))).double()
    ours.load_state_dict(theirs.state_dict())
    for step in range(3):
        x = torch.randn(4, 9, 16, dtype=torch.float64, requires_grad=True)
        for m in (theirs, ours):
            m.begin_balance_accumulation()
        a = theirs(x, update_routing_bias=True)
        b = ours(x, update_routing_bias=True)
        a = a if torch.is_tensor(a) else a.hidden_states
        b = b if torch.is_tensor(b) else b.hidden_states
        assert max_diff(a, b) < 1e-12
        ga = torch.autograd.grad(a.square().sum(), x)[0]
        gb = torch.autograd.grad(b.square().sum(), x)[0]
        assert max_diff(ga, gb) < 1e-12
        theirs.finalize_and_commit_balance()
        ours.finalize_and_commit_balance()
        assert max_diff(theirs.router.routing_bias, ours.router.routing_bias) < 1e-12, step


# --------------------------------------------------------------------------- AttnRes
@needs_reference
@pytest.mark.reference
def test_depth_softmax_mix_matches_reference():
    ref()
    from src.attention_residuals.site import depth_softmax_mix_reference as rmix
    from kimi_k3_b200.models.attnres import depth_softmax_mix_reference as omix
    torch.manual_seed(7)
    srcs = torch.randn(2, 5, 4, 16, dtype=torch.float64)
    q = torch.randn(16, dtype=torch.float64)
    norm = torch.nn.RMSNorm(16, dtype=torch.float64) if hasattr(torch.nn, "RMSNorm") else None
    if norm is None:
        pytest.skip("torch without nn.RMSNorm")
    from kimi_k3_b200.models.primitives import RMSNorm
    ours_norm = RMSNorm(16).double()
    ra = rmix(srcs, q, ours_norm)
    oa = omix(srcs, q, ours_norm)
    ra = ra if torch.is_tensor(ra) else ra[0]
    oa = oa if torch.is_tensor(oa) else oa[0]
    assert max_diff(ra, oa) < 1e-12


def test_dense_small_batch_experts_matches_sparse_dispatch():
    """The decode-size expert path (every expert on every token, unselected weights zero) equals
    the routed dispatch (fp64)."""
    import torch
    from kimi_k3_b200.models.moe import GroupedRoutedExperts, dense_small_batch_experts, vectorized_sparse_dispatch
    torch.manual_seed(0)
    ex = GroupedRoutedExperts(6, 32, 48, 4.0, 25.0, 0.2).double()
    x = torch.randn(5, 32, dtype=torch.float64)
    sel = torch.stack([torch.randperm(6)[:2] for _ in range(5)])
    w = torch.rand(5, 2, dtype=torch.float64)
    with torch.no_grad():
        got = dense_small_batch_experts(x, ex, sel, w, torch.float64)
        ref = vectorized_sparse_dispatch(x, ex, sel, w, accumulation_dtype=torch.float64)
    assert torch.allclose(got, ref, atol=1e-10, rtol=1e-9)
