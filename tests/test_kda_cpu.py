"""KDA operator oracles on CPU in float64: recurrence vs chunk form, ragged T, masks, state carry, reference."""
import pytest
import torch
import torch.nn.functional as F

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.kda import (KDAConfig, KimiDeltaAttention, chunkwise_kda, recurrent_kda, ut_transform)


def _core(b=2, t=37, h=3, kd=8, vd=5, seed=0, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(b, t, h, kd, generator=g, dtype=dtype), dim=-1)
    k = F.normalize(torch.randn(b, t, h, kd, generator=g, dtype=dtype), dim=-1)
    v = torch.randn(b, t, h, vd, generator=g, dtype=dtype)
    gg = -torch.rand(b, t, h, kd, generator=g, dtype=dtype) * 2.0
    beta = torch.rand(b, t, h, generator=g, dtype=dtype)
    h0 = torch.randn(b, h, kd, vd, generator=g, dtype=dtype) * 0.1
    return q, k, v, gg, beta, h0


@pytest.mark.parametrize("chunk", [1, 3, 8, 16, 64])
@pytest.mark.parametrize("t", [1, 17, 37])
def test_chunkwise_matches_recurrent(chunk, t):
    q, k, v, g, beta, h0 = _core(t=t)
    r = recurrent_kda(q, k, v, g, beta, h0, True)
    c = chunkwise_kda(q, k, v, g, beta, h0, True, chunk_size=chunk, secondary_tile_size=min(chunk, 16))
    assert max_diff(r.hidden_states, c.hidden_states) < 1e-11
    assert max_diff(r.final_state, c.final_state) < 1e-11


def test_state_carry_equals_one_pass():
    q, k, v, g, beta, h0 = _core(t=40)
    full = recurrent_kda(q, k, v, g, beta, h0, True)
    a = chunkwise_kda(q[:, :23], k[:, :23], v[:, :23], g[:, :23], beta[:, :23], h0, True, chunk_size=8)
    b = chunkwise_kda(q[:, 23:], k[:, 23:], v[:, 23:], g[:, 23:], beta[:, 23:], a.final_state, True, chunk_size=8)
    assert max_diff(torch.cat([a.hidden_states, b.hidden_states], 1), full.hidden_states) < 1e-11
    assert max_diff(b.final_state, full.final_state) < 1e-11


def test_right_padding_mask_freezes_state():
    q, k, v, g, beta, h0 = _core(t=20)
    mask = torch.ones(2, 20, dtype=torch.bool)
    mask[1, 12:] = False
    m = chunkwise_kda(q, k, v, g, beta, h0, True, mask, chunk_size=8)
    short = recurrent_kda(q[1:, :12], k[1:, :12], v[1:, :12], g[1:, :12], beta[1:, :12], h0[1:], True)
    assert max_diff(m.final_state[1:], short.final_state) < 1e-11
    assert max_diff(m.hidden_states[1:, :12], short.hidden_states) < 1e-11


def test_prefix_causality():
    q, k, v, g, beta, _ = _core(t=30)
    o = chunkwise_kda(q, k, v, g, beta, chunk_size=8).hidden_states
    v2 = v.clone()
    v2[:, 20:] += 5.0
    o2 = chunkwise_kda(q, k, v2, g, beta, chunk_size=8).hidden_states
    assert max_diff(o[:, :20], o2[:, :20]) == 0.0


def test_gradcheck_chunkwise():
    q, k, v, g, beta, h0 = _core(b=1, t=6, h=1, kd=3, vd=2)
    leaves = [x.clone().requires_grad_() for x in (q, k, v, g, beta, h0)]
    assert torch.autograd.gradcheck(lambda *a: chunkwise_kda(*a, True, chunk_size=4).hidden_states, leaves)


@needs_reference
@pytest.mark.reference
def test_operators_match_reference():
    ref()
    from src.kda.chunkwise import chunkwise_kda as rc
    from src.kda.recurrent import recurrent_kda as rr
    q, k, v, g, beta, h0 = _core(t=45)
    mask = torch.ones(2, 45, dtype=torch.bool)
    mask[0, 30:] = False
    ours = chunkwise_kda(q, k, v, g, beta, h0, True, mask, chunk_size=16)
    theirs = rc(q, k, v, g, beta, h0, True, mask, chunk_size=16)
    assert max_diff(ours.hidden_states, theirs.hidden_states) < 1e-11
    assert max_diff(ours.final_state, theirs.final_state) < 1e-11
    rr_out = rr(q, k, v, g, beta, h0, True, mask)
    assert max_diff(ours.hidden_states, rr_out.hidden_states) < 1e-11


@needs_reference
@pytest.mark.reference
def test_ut_transform_matches_reference():
    ref()
    from src.kda.ut_transform import ut_transform as rut
    _, k, v, g, beta, _ = _core(b=1, t=16, h=2)
    kc = k[:, :16].permute(0, 2, 1, 3)
    vc = v[:, :16].permute(0, 2, 1, 3)
    gc = g[:, :16].permute(0, 2, 1, 3)
    bc = beta[:, :16].permute(0, 2, 1)
    a, b = ut_transform(kc, vc, gc, bc), rut(kc, vc, gc, bc)
    for name in ("u", "w"):
        if hasattr(a, name) and hasattr(b, name):
            assert max_diff(getattr(a, name), getattr(b, name)) < 1e-11


@needs_reference
@pytest.mark.reference
def test_module_forward_prefill_decode_matches_reference():
    ref()
    from src.kda.config import KDAConfig as RC
    from src.kda.kda import KimiDeltaAttention as RK
    torch.manual_seed(3)
    rk = RK(RC(d_model=32, num_heads=4, key_head_dim=8, value_head_dim=8)).double()
    ok = KimiDeltaAttention(KDAConfig(d_model=32, num_heads=4, key_head_dim=8, value_head_dim=8)).double()
    ok.load_state_dict(rk.state_dict())
    x = torch.randn(2, 19, 32, dtype=torch.float64)
    a, b = ok(x), rk(x)
    assert max_diff(a.hidden_states, b.hidden_states) < 1e-11
    # prefill 11 tokens then decode one at a time equals the full forward
    pre = ok(x[:, :11], output_final_state=True)
    state, outs = pre.state, [pre.hidden_states]
    for i in range(11, 19):
        st = ok(x[:, i:i + 1], state=state, mode="decode")
        state = st.state
        outs.append(st.hidden_states)
    assert max_diff(torch.cat(outs, 1), a.hidden_states) < 1e-11
