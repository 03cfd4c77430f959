"""L0 primitive oracles on CPU: short conv, SiTU-GLU, RMSNorms, output gate, postprocess.

Each module is checked against the reference module of the same name (same weights, float64), and
against the equation it implements (lag-ordered causal conv, softcap bounds, RMS over the head axis).
Reference modules: ``src/kimi_primitives/{short_conv,situ_glu,headwise_rmsnorm,output_gate,
postprocess}.py`` and ``src/transformer_modules/rms_norm.py``.
"""
import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.primitives import (CausalShortConv1D, FullRankOutputGate, HeadwiseRMSNorm,
                                            PrimitiveAttentionPostprocess, RMSNorm, ShortConvState, SiTUGLU,
                                            combine_heads, situ_glu_activation, softcap, split_heads)

F64 = torch.float64


def _conv_by_definition(x, weight, bias=None, history=None):
    """``y[t, c] = sum_j weight[c, j] * x[t - j, c]`` with zeros (or the history) before t = 0."""
    b, t, c = x.shape
    k = weight.shape[1]
    hist = x.new_zeros(b, k - 1, c) if history is None else history
    full = torch.cat((hist, x), 1)
    y = x.new_zeros(b, t, c)
    for i in range(t):
        for j in range(k):
            y[:, i] += weight[:, j] * full[:, i + k - 1 - j]
    if bias is not None:
        y = y + bias
    return y


# --------------------------------------------------------------------------- short conv
@pytest.mark.parametrize("kernel_size", [1, 2, 3, 4, 5])
@pytest.mark.parametrize("bias", [False, True])
def test_short_conv_matches_lag_ordered_definition(kernel_size, bias):
    torch.manual_seed(kernel_size)
    conv = CausalShortConv1D(6, kernel_size, bias=bias).double()
    if bias:
        torch.nn.init.normal_(conv.bias)
    x = torch.randn(2, 9, 6, dtype=F64)
    assert max_diff(conv(x), _conv_by_definition(x, conv.weight, conv.bias)) < 1e-13


@pytest.mark.parametrize("split", [0, 1, 3, 7, 11])
def test_short_conv_state_carry_equals_one_pass(split):
    torch.manual_seed(3)
    conv = CausalShortConv1D(5, 4).double()
    x = torch.randn(3, 11, 5, dtype=F64)
    full, st_full = conv(x, return_state=True)
    a, st = conv(x[:, :split], return_state=True)
    b, st2 = conv(x[:, split:], state=st, return_state=True)
    assert max_diff(torch.cat((a, b), 1), full) < 1e-13
    assert max_diff(st2.buffer, st_full.buffer) == 0.0
    assert st_full.buffer.shape == (3, 3, 5)


def test_short_conv_token_by_token_equals_full():
    torch.manual_seed(4)
    conv = CausalShortConv1D(4, 3, bias=True).double()
    x = torch.randn(2, 8, 4, dtype=F64)
    full = conv(x)
    st, outs = None, []
    for i in range(8):
        y, st = conv(x[:, i:i + 1], state=st, return_state=True)
        outs.append(y)
    assert max_diff(torch.cat(outs, 1), full) < 1e-13


def test_short_conv_is_causal():
    torch.manual_seed(5)
    conv = CausalShortConv1D(4, 4).double()
    x = torch.randn(1, 10, 4, dtype=F64)
    y = conv(x)
    x2 = x.clone()
    x2[:, 6:] = torch.randn(1, 4, 4, dtype=F64)
    assert max_diff(conv(x2)[:, :6], y[:, :6]) == 0.0


def test_short_conv_state_is_not_mutated_and_empty_input():
    conv = CausalShortConv1D(3, 4).double()
    st = ShortConvState(torch.randn(1, 3, 3, dtype=F64))
    before = st.buffer.clone()
    y, nxt = conv(torch.zeros(1, 0, 3, dtype=F64), state=st, return_state=True)
    assert y.shape == (1, 0, 3)
    assert max_diff(st.buffer, before) == 0.0
    assert max_diff(nxt.buffer, before) == 0.0 and nxt.buffer is not st.buffer
    clone = st.clone()
    assert clone.buffer is not st.buffer and max_diff(clone.buffer, st.buffer) == 0.0


def test_short_conv_rejects_bad_state_and_shapes():
    conv = CausalShortConv1D(3, 4)
    x = torch.randn(2, 5, 3)
    with pytest.raises(ValueError):
        conv(x, state=ShortConvState(torch.zeros(2, 2, 3)))
    with pytest.raises(ValueError):
        conv(x, state=ShortConvState(torch.zeros(2, 3, 3, dtype=F64)))
    with pytest.raises(ValueError):
        conv(torch.randn(2, 5, 4))
    with pytest.raises(ValueError):
        ShortConvState(torch.zeros(3, 3))
    with pytest.raises(ValueError):
        CausalShortConv1D(0, 4)
    with pytest.raises(ValueError):
        CausalShortConv1D(3, 0)


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("kernel_size,bias", [(1, False), (4, False), (4, True), (6, True)])
def test_short_conv_matches_reference(kernel_size, bias):
    ref()
    from src.kimi_primitives.short_conv import CausalShortConv1D as RefConv
    from src.kimi_primitives.states import ShortConvState as RefState
    torch.manual_seed(6)
    ours = CausalShortConv1D(7, kernel_size, bias=bias).double()
    theirs = RefConv(7, kernel_size, bias=bias).double()
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(2, 13, 7, dtype=F64, requires_grad=True)
    xr = x.detach().clone().requires_grad_(True)
    hist = torch.randn(2, kernel_size - 1, 7, dtype=F64)
    y, s = ours(x, state=ShortConvState(hist), return_state=True)
    yr, sr = theirs(xr, state=RefState(hist), return_state=True)
    assert max_diff(y, yr) < 1e-14 and torch.equal(s.buffer, sr.buffer)
    g = torch.randn_like(y)
    y.backward(g)
    yr.backward(g)
    assert max_diff(x.grad, xr.grad) < 1e-14
    assert max_diff(ours.weight.grad, theirs.weight.grad) < 1e-13


# --------------------------------------------------------------------------- SiTU-GLU
@pytest.mark.parametrize("beta", [0.5, 4.0, 25.0])
def test_softcap_is_bounded_odd_and_identity_near_zero(beta):
    x = torch.linspace(-200, 200, 2001, dtype=F64)
    y = softcap(x, beta)
    assert y.abs().max().item() <= beta
    assert max_diff(softcap(-x, beta), -y) == 0.0
    small = torch.linspace(-1e-4, 1e-4, 11, dtype=F64)
    assert max_diff(softcap(small, beta), small) < 1e-12 / beta
    with pytest.raises(ValueError):
        softcap(x, 0.0)


def test_situ_activation_equation_and_bounds():
    torch.manual_seed(7)
    g = torch.randn(4, 33, dtype=F64) * 10
    u = torch.randn(4, 33, dtype=F64) * 50
    want = 4.0 * torch.tanh(g / 4.0) * torch.sigmoid(g) * 25.0 * torch.tanh(u / 25.0)
    assert max_diff(situ_glu_activation(g, u), want) < 1e-13
    # |softcap(g,4)·σ(g)| < 4 and |softcap(u,25)| < 25
    big = situ_glu_activation(torch.full((3,), 1e6, dtype=F64), torch.full((3,), -1e6, dtype=F64))
    assert (big.abs() <= 100.0).all()
    with pytest.raises(ValueError):
        situ_glu_activation(g, u[:, :5])
    with pytest.raises(ValueError):
        situ_glu_activation(g, u, beta_gate=-1.0)


def test_situ_glu_gradcheck():
    torch.manual_seed(8)
    m = SiTUGLU(5, 7, bias=True).double()
    x = torch.randn(2, 3, 5, dtype=F64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda t: m(t), (x,))


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("bias,output_bias", [(False, None), (True, None), (True, False), (False, True)])
def test_situ_glu_matches_reference(bias, output_bias):
    ref()
    from src.kimi_primitives.situ_glu import SiTUGLU as RefGLU
    torch.manual_seed(9)
    ours = SiTUGLU(12, 20, bias=bias, output_bias=output_bias).double()
    theirs = RefGLU(12, 20, bias=bias, output_bias=output_bias).double()
    assert sorted(ours.state_dict()) == sorted(theirs.state_dict())
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(3, 5, 12, dtype=F64) * 3
    assert max_diff(ours(x), theirs(x)) < 1e-14


def test_situ_glu_init_and_validation():
    torch.manual_seed(10)
    m = SiTUGLU(64, 256, init_std=0.05)
    for p in (m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight):
        assert abs(p.std().item() - 0.05) < 0.01
    with pytest.raises(ValueError):
        SiTUGLU(0, 4)
    with pytest.raises(ValueError):
        SiTUGLU(4, 4, init_std=0.0)
    with pytest.raises(ValueError):
        m(torch.randn(2, 63))


# --------------------------------------------------------------------------- norms
@pytest.mark.parametrize("dtype", [torch.float64, torch.float32, torch.bfloat16])
def test_rms_norm_equation(dtype):
    torch.manual_seed(11)
    n = RMSNorm(24, eps=1e-5)
    torch.nn.init.normal_(n.weight)
    x = (torch.randn(3, 4, 24) * 7).to(dtype)
    y = n.to(dtype)(x) if dtype == torch.float64 else n(x)
    xf = x.double()
    want = xf / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)
    want = want.to(dtype).double() * n.weight.to(dtype).double()
    tol = {torch.float64: 1e-12, torch.float32: 1e-5, torch.bfloat16: 3e-2}[dtype]
    assert y.dtype == dtype
    assert max_diff(y, want) < tol


def test_rms_norm_is_scale_invariant_and_validates():
    torch.manual_seed(12)
    n = RMSNorm(16, eps=1e-14).double()
    x = torch.randn(2, 16, dtype=F64)
    assert max_diff(n(x * 37.0), n(x)) < 1e-12
    with pytest.raises(ValueError):
        n(torch.randn(2, 15, dtype=F64))
    with pytest.raises(ValueError):
        RMSNorm(0)
    with pytest.raises(ValueError):
        RMSNorm(4, eps=0.0)


@needs_reference
@pytest.mark.reference
def test_rms_norm_matches_reference():
    ref()
    from src.transformer_modules.rms_norm import RMSNorm as RefNorm
    torch.manual_seed(13)
    ours, theirs = RMSNorm(20, eps=1e-6).double(), RefNorm(20, eps=1e-6).double()
    torch.nn.init.normal_(ours.weight)
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(2, 7, 20, dtype=F64)
    assert max_diff(ours(x), theirs(x)) < 1e-14
    xb = x.to(torch.bfloat16)
    assert max_diff(ours.to(torch.bfloat16)(xb), theirs.to(torch.bfloat16)(xb)) == 0.0


@pytest.mark.parametrize("affine,per_head", [(True, True), (True, False), (False, True)])
def test_headwise_rms_norm_normalises_each_head(affine, per_head):
    torch.manual_seed(14)
    n = HeadwiseRMSNorm(3, 8, eps=1e-14, elementwise_affine=affine, per_head_affine=per_head).double()
    if affine:
        torch.nn.init.normal_(n.weight)
        assert n.weight.shape == ((3, 8) if per_head else (8,))
    else:
        assert n.weight is None
    x = torch.randn(2, 5, 3, 8, dtype=F64)
    # scaling one head leaves every head's output unchanged
    x2 = x.clone()
    x2[:, :, 1] *= 9.0
    assert max_diff(n(x2), n(x)) < 1e-12
    y = n(x)
    if not affine:
        rms = y.pow(2).mean(-1).sqrt()
        assert max_diff(rms, torch.ones_like(rms)) < 1e-5


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("affine,per_head", [(True, True), (True, False), (False, False)])
@pytest.mark.parametrize("dtype", [torch.float64, torch.bfloat16])
def test_headwise_rms_norm_matches_reference(affine, per_head, dtype):
    ref()
    from src.kimi_primitives.headwise_rmsnorm import HeadwiseRMSNorm as RefHN
    torch.manual_seed(15)
    ours = HeadwiseRMSNorm(4, 6, elementwise_affine=affine, per_head_affine=per_head)
    theirs = RefHN(4, 6, elementwise_affine=affine, per_head_affine=per_head)
    if affine:
        torch.nn.init.normal_(ours.weight)
    theirs.load_state_dict(ours.state_dict())
    ours, theirs = ours.to(dtype), theirs.to(dtype)
    x = torch.randn(2, 3, 4, 6).to(dtype)
    assert max_diff(ours(x), theirs(x)) == 0.0


def test_split_combine_heads_round_trip_and_validation():
    x = torch.randn(2, 3, 12)
    h = split_heads(x, 4)
    assert h.shape == (2, 3, 4, 3)
    assert torch.equal(combine_heads(h), x)
    assert torch.equal(h[:, :, 1], x[:, :, 3:6])
    with pytest.raises(ValueError):
        split_heads(x, 5)
    with pytest.raises(ValueError):
        split_heads(x[0], 4)
    with pytest.raises(ValueError):
        combine_heads(x)


# --------------------------------------------------------------------------- gates
def test_output_gate_equation_and_return_gate():
    torch.manual_seed(16)
    g = FullRankOutputGate(8, bias=True, output_bias=True).double()
    torch.nn.init.normal_(g.gate_proj.bias)
    torch.nn.init.normal_(g.output_proj.bias)
    a = torch.randn(2, 5, 8, dtype=F64)
    r = torch.randn(2, 5, 8, dtype=F64)
    out, gate = g(a, r, return_gate=True)
    want_gate = torch.sigmoid(r @ g.gate_proj.weight.T + g.gate_proj.bias)
    assert max_diff(gate, want_gate) < 1e-14
    assert max_diff(out, (want_gate * a) @ g.output_proj.weight.T + g.output_proj.bias) < 1e-14
    assert max_diff(g.gate_values(r), want_gate) < 1e-14
    # precomputed gate logits (a fused projection group) give the same output
    logits = g.gate_proj(r)
    assert max_diff(g(a, r, gate_logits=logits), out) == 0.0
    with pytest.raises(ValueError):
        g(a[:, :4], r)
    with pytest.raises(ValueError):
        g(a, r[..., :7])


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("norm_affine,per_head", [(True, True), (False, True), (True, False)])
def test_postprocess_matches_reference(norm_affine, per_head):
    ref()
    from src.kimi_primitives.postprocess import PrimitiveAttentionPostprocess as RefPost
    torch.manual_seed(17)
    kw = dict(norm_affine=norm_affine, per_head_affine=per_head, gate_bias=True)
    ours = PrimitiveAttentionPostprocess(3, 4, **kw).double()
    theirs = RefPost(3, 4, **kw).double()
    assert sorted(ours.state_dict()) == sorted(theirs.state_dict())
    theirs.load_state_dict(ours.state_dict())
    heads = torch.randn(2, 6, 3, 4, dtype=F64)
    resid = torch.randn(2, 6, 12, dtype=F64)
    o, gte = ours(heads, resid, return_gate=True)
    orf, gr = theirs(heads, resid, return_gate=True)
    assert max_diff(o, orf) < 1e-14 and max_diff(gte, gr) < 1e-14
