"""KDA module-level checks on CPU: config, decay bounds, projections, modes, masks, state handling.

Oracles: the equations of ``src/kda/decay.py:7-43`` (lower-bounded decay), ``src/kda/projections.py:144-225``
(normalised q / k, clamped beta, low-rank decay logits) and the reference modules themselves in float64.
"""
import io
import math

import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.kda import (KDAConfig, KDAState, KimiDeltaAttention, LowerBoundedDecay,
                                     validate_attention_mask)
from kimi_k3_b200.models.primitives import ShortConvState

F64 = torch.float64


def _cfg(**kw):
    base = dict(d_model=24, num_heads=3, key_head_dim=6, value_head_dim=8)
    base.update(kw)
    return KDAConfig(**base)


def _module(seed=0, **kw):
    torch.manual_seed(seed)
    return KimiDeltaAttention(_cfg(**kw)).double()


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("bad", [
    dict(d_model=25),                              # d_model != H * Dv
    dict(num_heads=0, d_model=0),
    dict(key_head_dim=0),
    dict(short_conv_kernel_size=0),
    dict(chunk_size=8, secondary_tile_size=16),    # secondary tile larger than the chunk
    dict(g_min=0.0),
    dict(g_min=1.0),
    dict(decay_rank=0),
    dict(eps=0.0),
    dict(init_std=-1.0),
    dict(decay_initializer="uniform"),
])
def test_config_rejects_invalid_values(bad):
    with pytest.raises(ValueError):
        _cfg(**bad)


def test_config_properties_and_round_trip():
    c = _cfg(decay_rank=5)
    assert c.resolved_decay_rank == 5 and c.key_width == 18 and c.value_width == 24
    assert _cfg().resolved_decay_rank == 8
    assert KDAConfig.from_dict(c.to_dict()) == c


@needs_reference
@pytest.mark.reference
def test_config_dict_matches_reference_schema():
    ref()
    from src.kda.config import KDAConfig as RC
    ours = _cfg(decay_rank=4, chunk_size=32).to_dict()
    theirs = RC(**ours).to_dict()
    assert ours == theirs


# --------------------------------------------------------------------------- decay
@pytest.mark.parametrize("g_min", [-5.0, -1.0, -0.25])
def test_decay_is_bounded_by_g_min_and_zero(g_min):
    torch.manual_seed(1)
    d = LowerBoundedDecay(4, g_min).double()
    with torch.no_grad():
        d.A_log.copy_(torch.tensor([-1.0, 0.0, 0.5, 2.0]))
    z = torch.randn(2, 5, 4, 3, dtype=F64) * 40
    g, a = d(z)
    assert (g < 0).all() and (g > g_min).all()
    assert max_diff(a, torch.exp(g)) == 0.0
    want = g_min * torch.sigmoid(d.A_log.exp()[None, None, :, None] * z).clamp(2.3e-16, 1 - 2.3e-16)
    assert max_diff(g, want) < 1e-12
    # saturating logits stay strictly inside the open interval
    g_hi, _ = d(torch.full((1, 1, 4, 1), 1e4, dtype=F64))
    g_lo, _ = d(torch.full((1, 1, 4, 1), -1e4, dtype=F64))
    assert (g_hi > g_min).all() and (g_lo < 0).all()


def test_decay_is_monotone_in_logits():
    d = LowerBoundedDecay(2).double()
    z = torch.linspace(-6, 6, 50, dtype=F64).reshape(1, 50, 1, 1).expand(1, 50, 2, 1)
    g, _ = d(z.contiguous())
    assert (g[:, 1:] < g[:, :-1]).all()


def test_decay_validation():
    with pytest.raises(ValueError):
        LowerBoundedDecay(0)
    with pytest.raises(ValueError):
        LowerBoundedDecay(2, g_min=0.5)
    with pytest.raises(ValueError):
        LowerBoundedDecay(2)(torch.zeros(1, 2, 3, 4))


@needs_reference
@pytest.mark.reference
def test_decay_matches_reference():
    ref()
    from src.kda.decay import LowerBoundedDecay as RD
    torch.manual_seed(2)
    ours, theirs = LowerBoundedDecay(3, -3.0).double(), RD(3, -3.0).double()
    with torch.no_grad():
        ours.A_log.normal_()
    theirs.load_state_dict(ours.state_dict())
    z = torch.randn(2, 4, 3, 5, dtype=F64) * 5
    (g, a), (gr, ar) = ours(z), theirs(z)
    assert max_diff(g, gr) == 0.0 and max_diff(a, ar) == 0.0


# --------------------------------------------------------------------------- projections
def test_projection_outputs_are_normalised_and_clamped():
    m = _module(3)
    x = torch.randn(2, 9, 24, dtype=F64) * 3
    p = m.projections(x)
    assert p.q.shape == (2, 9, 3, 6) and p.v.shape == (2, 9, 3, 8)
    assert max_diff(p.q.norm(dim=-1), torch.ones(2, 9, 3, dtype=F64)) < 1e-10
    assert max_diff(p.k.norm(dim=-1), torch.ones(2, 9, 3, dtype=F64)) < 1e-10
    assert (p.beta > 0).all() and (p.beta < 1).all() and p.beta.shape == (2, 9, 3)
    proj = m.projections
    want = (x @ proj.alpha_down.weight.T @ proj.alpha_up.weight.T).reshape(2, 9, 3, 6) + proj.b_alpha
    assert max_diff(p.decay_logits, want) < 1e-12


def test_official_fla_decay_bias_maps_to_log_uniform_dt():
    torch.manual_seed(4)
    m = KimiDeltaAttention(_cfg(num_heads=8, d_model=64, key_head_dim=16))
    dt = torch.nn.functional.softplus(m.projections.b_alpha.double())
    assert dt.min().item() >= 1e-4 - 1e-9 and dt.max().item() <= 0.1 + 1e-6
    logs = dt.log()
    assert logs.min().item() < math.log(0.01) < logs.max().item()
    z = KimiDeltaAttention(_cfg(decay_initializer="zeros"))
    assert z.projections.b_alpha.abs().max().item() == 0.0


def test_projection_conv_state_continues_across_calls():
    m = _module(5)
    x = torch.randn(2, 12, 24, dtype=F64)
    full = m.projections(x, output_final_state=True)
    a = m.projections(x[:, :7], output_final_state=True)
    b = m.projections(x[:, 7:], q_conv_state=a.q_conv_state, k_conv_state=a.k_conv_state,
                      v_conv_state=a.v_conv_state, output_final_state=True)
    for name in ("q", "k", "v", "beta", "decay_logits"):
        assert max_diff(torch.cat((getattr(a, name), getattr(b, name)), 1), getattr(full, name)) < 1e-12
    assert max_diff(b.k_conv_state.buffer, full.k_conv_state.buffer) == 0.0


@needs_reference
@pytest.mark.reference
def test_projections_match_reference_with_padding():
    ref()
    from src.kda.config import KDAConfig as RC
    from src.kda.projections import KDAProjections as RP
    torch.manual_seed(6)
    ours = _module(6, projection_bias=True, beta_bias=True).projections
    theirs = RP(RC(**_cfg(projection_bias=True, beta_bias=True).to_dict())).double()
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(3, 10, 24, dtype=F64)
    mask = torch.ones(3, 10, dtype=torch.bool)
    mask[1, 6:] = False
    mask[2, 3:] = False
    a = ours(x, attention_mask=mask, output_final_state=True)
    b = theirs(x, attention_mask=mask, output_final_state=True)
    for name in ("q", "k", "v", "beta", "decay_logits"):
        assert max_diff(getattr(a, name), getattr(b, name)) < 1e-13, name
    for name in ("q_conv_state", "k_conv_state", "v_conv_state"):
        assert max_diff(getattr(a, name).buffer, getattr(b, name).buffer) == 0.0, name


# --------------------------------------------------------------------------- module
@pytest.mark.parametrize("chunk,tile", [(4, 4), (8, 4), (16, 16), (64, 16)])
def test_recurrent_and_chunkwise_modes_agree(chunk, tile):
    m = _module(7, chunk_size=chunk, secondary_tile_size=tile)
    x = torch.randn(2, 21, 24, dtype=F64)
    a = m(x, mode="recurrent", output_final_state=True)
    b = m(x, mode="chunkwise", output_final_state=True)
    assert max_diff(a.hidden_states, b.hidden_states) < 1e-11
    assert max_diff(a.state.recurrent_state, b.state.recurrent_state) < 1e-11
    assert a.state.sequence_offset.tolist() == [21, 21]


def test_padded_rows_match_their_unpadded_runs_and_are_zeroed():
    m = _module(8)
    x = torch.randn(3, 11, 24, dtype=F64)
    lengths = [11, 6, 2]
    mask = torch.arange(11)[None] < torch.tensor(lengths)[:, None]
    out = m(x, attention_mask=mask, output_final_state=True)
    assert out.state.sequence_offset.tolist() == lengths
    for i, n in enumerate(lengths):
        alone = m(x[i:i + 1, :n], output_final_state=True)
        assert max_diff(out.hidden_states[i, :n], alone.hidden_states[0]) < 1e-11
        assert max_diff(out.state.recurrent_state[i], alone.state.recurrent_state[0]) < 1e-11
        assert out.hidden_states[i, n:].abs().max().item() == 0.0 if n < 11 else True


def test_module_is_causal():
    m = _module(9)
    x = torch.randn(1, 16, 24, dtype=F64)
    y = m(x).hidden_states
    x2 = x.clone()
    x2[:, 10:] += torch.randn(1, 6, 24, dtype=F64)
    assert max_diff(m(x2).hidden_states[:, :10], y[:, :10]) < 1e-13


def test_decode_continues_a_padded_prefill():
    m = _module(10)
    x = torch.randn(2, 9, 24, dtype=F64)
    mask = torch.ones(2, 6, dtype=torch.bool)
    mask[1, 4:] = False
    pre = m(x[:, :6], attention_mask=mask, output_final_state=True)
    st = m(x[:, 6:7], state=pre.state, mode="decode").state
    # row 1 saw 4 prompt tokens, then the decode token
    alone = m(torch.cat((x[1:, :4], x[1:, 6:7]), 1), output_final_state=True)
    assert max_diff(st.recurrent_state[1], alone.state.recurrent_state[0]) < 1e-11
    assert st.sequence_offset.tolist() == [7, 5]


def test_state_clone_reorder_and_validation():
    m = _module(11)
    x = torch.randn(3, 5, 24, dtype=F64)
    st = m(x, output_final_state=True).state
    c = st.clone()
    assert c.recurrent_state is not st.recurrent_state and max_diff(c.recurrent_state, st.recurrent_state) == 0.0
    idx = torch.tensor([2, 0], dtype=torch.long)
    r = st.reorder(idx)
    assert max_diff(r.recurrent_state, st.recurrent_state[idx]) == 0.0
    assert max_diff(r.v_conv_state.buffer, st.v_conv_state.buffer[idx]) == 0.0
    assert r.sequence_offset.tolist() == [5, 5]
    # a reordered state decodes exactly like the selected rows of the original
    tok = torch.randn(3, 1, 24, dtype=F64)
    full = m(tok, state=st, mode="decode").hidden_states
    sub = m(tok[idx], state=r, mode="decode").hidden_states
    assert max_diff(sub, full[idx]) < 1e-13
    with pytest.raises(ValueError):
        st.reorder(torch.tensor([0.0]))
    with pytest.raises(ValueError):
        KDAState(st.recurrent_state[0], st.q_conv_state, st.k_conv_state, st.v_conv_state, st.sequence_offset)
    with pytest.raises(TypeError):
        KDAState(st.recurrent_state, st.q_conv_state, st.k_conv_state, st.v_conv_state,
                 st.sequence_offset.to(torch.int32))
    with pytest.raises(ValueError):
        m(x[:2], state=st)
    bad = KDAState(st.recurrent_state, ShortConvState(st.q_conv_state.buffer[:, :2]), st.k_conv_state,
                   st.v_conv_state, st.sequence_offset)
    with pytest.raises(ValueError):
        m(x, state=bad)


def test_module_argument_validation():
    m = _module(12)
    x = torch.randn(2, 3, 24, dtype=F64)
    with pytest.raises(ValueError):
        m(x, mode="decode")
    with pytest.raises(ValueError):
        m(x, mode="parallel")
    with pytest.raises(ValueError):
        m(x[:, :0])
    with pytest.raises(ValueError):
        m(torch.randn(2, 3, 23, dtype=F64))
    with pytest.raises(ValueError):
        m(x, attention_mask=torch.ones(2, 4, dtype=torch.bool))
    with pytest.raises(ValueError):
        validate_attention_mask(torch.zeros(2, 3, dtype=torch.bool), 2, 3)


def test_state_round_trips_through_serialization():
    m = _module(13)
    x = torch.randn(2, 7, 24, dtype=F64)
    st = m(x, output_final_state=True).state
    buf = io.BytesIO()
    torch.save({"model": m.state_dict(), "state": st}, buf)
    buf.seek(0)
    payload = torch.load(buf, weights_only=False)
    m2 = KimiDeltaAttention(_cfg()).double()
    m2.load_state_dict(payload["model"])
    tok = torch.randn(2, 1, 24, dtype=F64)
    a = m(tok, state=st, mode="decode")
    b = m2(tok, state=payload["state"], mode="decode")
    assert max_diff(a.hidden_states, b.hidden_states) == 0.0
    assert max_diff(a.state.recurrent_state, b.state.recurrent_state) == 0.0


def test_every_parameter_receives_a_finite_gradient():
    m = _module(14, projection_bias=True, short_conv_bias=True, beta_bias=True, output_gate_bias=True,
                output_bias=True)
    x = torch.randn(2, 10, 24, dtype=F64)
    m(x).hidden_states.square().sum().backward()
    for name, p in m.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name
        assert p.grad.abs().sum().item() > 0, name


def test_bf16_forward_is_finite_and_close_to_fp64():
    m = _module(15)
    x = torch.randn(2, 12, 24, dtype=F64)
    want = m(x).hidden_states
    got = m.to(torch.bfloat16)(x.to(torch.bfloat16)).hidden_states
    assert got.dtype == torch.bfloat16 and torch.isfinite(got).all()
    rel = (got.double() - want).norm() / want.norm()
    assert rel.item() < 0.1  # the reference module in bf16 lands at the same distance (tested below)


def test_diagnostics_are_finite_scalars():
    m = _module(16)
    x = torch.randn(2, 8, 24, dtype=F64)
    mask = torch.ones(2, 8, dtype=torch.bool)
    mask[1, 5:] = False
    d = m(x, attention_mask=mask, output_diagnostics=True).diagnostics
    assert d and all(torch.is_tensor(v) and v.numel() == 1 and torch.isfinite(v).all() for v in d.values())


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("mode", ["recurrent", "chunkwise"])
def test_module_outputs_gradients_and_diagnostics_match_reference(mode):
    ref()
    from src.kda.config import KDAConfig as RC
    from src.kda.kda import KimiDeltaAttention as RK
    kw = dict(chunk_size=8, secondary_tile_size=4, decay_rank=5, short_conv_bias=True)
    ours = _module(17, **kw)
    theirs = RK(RC(**_cfg(**kw).to_dict())).double()
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(2, 13, 24, dtype=F64)
    mask = torch.ones(2, 13, dtype=torch.bool)
    mask[0, 9:] = False
    a = ours(x, attention_mask=mask, mode=mode, output_final_state=True, output_diagnostics=True)
    b = theirs(x, attention_mask=mask, mode=mode, output_final_state=True, output_diagnostics=True)
    assert max_diff(a.hidden_states, b.hidden_states) < 1e-11
    assert max_diff(a.state.recurrent_state, b.state.recurrent_state) < 1e-11
    assert a.state.sequence_offset.tolist() == b.state.sequence_offset.tolist()
    assert set(a.diagnostics) == set(b.diagnostics)
    for key in a.diagnostics:  # diagnostics are reported in fp32
        want = b.diagnostics[key].double()
        assert max_diff(a.diagnostics[key], want) < 1e-6 * (1.0 + want.abs().item()), key
    g = torch.randn_like(a.hidden_states)
    a.hidden_states.backward(g)
    b.hidden_states.backward(g)
    theirs_grads = dict(theirs.named_parameters())
    for name, p in ours.named_parameters():
        assert max_diff(p.grad, theirs_grads[name].grad) < 1e-9, name


@needs_reference
@pytest.mark.reference
def test_bf16_forward_is_bitwise_equal_to_reference():
    ref()
    from src.kda.config import KDAConfig as RC
    from src.kda.kda import KimiDeltaAttention as RK
    ours = _module(18)
    theirs = RK(RC(**_cfg().to_dict())).double()
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(2, 12, 24).to(torch.bfloat16)
    a = ours.to(torch.bfloat16)(x).hidden_states
    b = theirs.to(torch.bfloat16)(x).hidden_states
    assert torch.equal(a, b)


@pytest.mark.parametrize("g_scale", [-5.0, -0.01])
def test_fp32_chunkwise_is_stable_under_extreme_decay(g_scale):
    """Full 64-token chunks at the strongest (g near g_min = -5) and weakest decays: the fp32 chunk form
    stays finite and within fp32 round-off of the fp64 recurrence (no exp(+|cumulative decay|) blow-up)."""
    from kimi_k3_b200.models.kda import chunkwise_kda, recurrent_kda
    import torch.nn.functional as F
    torch.manual_seed(0)
    b, t, h, k, v = 1, 256, 2, 16, 16
    q = F.normalize(torch.randn(b, t, h, k), dim=-1)
    kk = F.normalize(torch.randn(b, t, h, k), dim=-1)
    vv = torch.randn(b, t, h, v)
    g = g_scale * torch.rand(b, t, h, k).clamp_min(0.5)
    beta = torch.rand(b, t, h)
    want = recurrent_kda(q.double(), kk.double(), vv.double(), g.double(), beta.double(), None, True)
    got = chunkwise_kda(q, kk, vv, g, beta, None, True, chunk_size=64)
    assert torch.isfinite(got.hidden_states).all() and torch.isfinite(got.final_state).all()
    assert max_diff(got.hidden_states, want.hidden_states) < 1e-5
    assert max_diff(got.final_state, want.final_state) < 1e-5
