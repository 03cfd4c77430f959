"""Gated MLA module-level checks on CPU: config, attention backends and masks, NoPE, latent caches,
gradients and diagnostics.

Oracles: the masked-softmax attention equation (``src/mla/attention.py:35-195``), the cache repacking
rule of ``src/mla/cache.py:106-163`` and the reference modules in float64.
"""
import io
import math

import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.mla import (GatedMLA, GatedMLAConfig, MLACache, StaticMLACache, manual_causal_attention,
                                     mla_attention)

F64 = torch.float64


def _cfg(**kw):
    base = dict(d_model=24, num_heads=3, q_head_dim=4, v_head_dim=8, kv_latent_dim=12)
    base.update(kw)
    return GatedMLAConfig(**base)


def _module(seed=0, **kw):
    torch.manual_seed(seed)
    return GatedMLA(_cfg(**kw)).double()


def _attention_by_definition(q, k, v, allowed):
    """``softmax(q k^T / sqrt(d))`` over the allowed keys of each query; rows with none give 0."""
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(q.shape[-1])
    s = s.masked_fill(~allowed[:, None], -torch.inf)
    p = torch.softmax(s, -1).nan_to_num(0.0)
    return torch.einsum("bhqk,bkhd->bqhd", p, v)


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("bad", [
    dict(d_model=25),
    dict(kv_latent_dim=37),                 # above H * (Dq + Dv) = 36
    dict(kv_latent_dim=0),
    dict(attention_dropout=1.0),
    dict(output_dropout=-0.1),
    dict(use_nope=False),
    dict(attention_backend="flash"),
    dict(attention_backend="sdpa", use_sdpa=False),
    dict(init_std=0.0),
])
def test_config_rejects_invalid_values(bad):
    with pytest.raises(ValueError):
        _cfg(**bad)


def test_config_properties_and_backend_resolution():
    c = _cfg()
    assert (c.query_width, c.value_width, c.full_kv_width) == (12, 24, 36)
    assert c.cache_compression_ratio == 3.0
    assert c.resolved_backend == "sdpa"
    assert _cfg(use_sdpa=False).resolved_backend == "manual"
    assert _cfg(attention_backend="manual").resolved_backend == "manual"
    assert GatedMLAConfig.from_dict(c.to_dict()) == c


@needs_reference
@pytest.mark.reference
def test_config_dict_matches_reference_schema():
    ref()
    from src.mla.config import GatedMLAConfig as RC
    ours = _cfg(attention_backend="manual", kv_latent_dim=20).to_dict()
    assert RC(**ours).to_dict() == ours
    assert RC(**ours).cache_compression_ratio == _cfg(attention_backend="manual", kv_latent_dim=20).cache_compression_ratio


# --------------------------------------------------------------------------- attention math
@pytest.mark.parametrize("backend", ["manual", "sdpa"])
@pytest.mark.parametrize("tq,tk", [(5, 5), (1, 7), (3, 9)])
def test_attention_matches_definition_with_key_and_query_masks(backend, tq, tk):
    torch.manual_seed(tq * 10 + tk)
    q = torch.randn(2, tq, 3, 4, dtype=F64)
    k = torch.randn(2, tk, 3, 4, dtype=F64)
    v = torch.randn(2, tk, 3, 6, dtype=F64)
    key_mask = torch.ones(2, tk, dtype=torch.bool)
    key_mask[1, tk - 2:] = False
    query_mask = torch.ones(2, tq, dtype=torch.bool)
    query_mask[0, -1] = tq == 1  # keep at least one valid query in row 0
    pos = torch.arange(tq)[None].expand(2, tq) + (tk - tq)
    out = mla_attention(q, k, v, key_mask, True, backend=backend, query_mask=query_mask, query_positions=pos)
    allowed = key_mask[:, None, :] & (torch.arange(tk)[None, None, :] <= pos[:, :, None]) & query_mask[:, :, None]
    assert max_diff(out, _attention_by_definition(q, k, v, allowed)) < 1e-12


def test_fully_masked_query_rows_are_zero_and_finite():
    torch.manual_seed(1)
    q, k, v = (torch.randn(1, 4, 2, 4, dtype=F64) for _ in range(3))
    qmask = torch.tensor([[True, False, True, False]])
    for backend in ("manual", "sdpa"):
        out = mla_attention(q, k, v, None, True, backend=backend, query_mask=qmask)
        assert torch.isfinite(out).all()
        assert out[0, 1].abs().max().item() == 0.0 and out[0, 3].abs().max().item() == 0.0


def test_attention_probabilities_are_causal_and_normalised():
    torch.manual_seed(2)
    q, k, v = (torch.randn(2, 6, 2, 4, dtype=F64) for _ in range(3))
    out, probs = manual_causal_attention(q, k, v, return_attentions=True)
    assert probs.shape == (2, 2, 6, 6)
    assert max_diff(probs.sum(-1), torch.ones(2, 2, 6, dtype=F64)) < 1e-12
    assert probs.triu(1).abs().max().item() == 0.0
    assert max_diff(out, mla_attention(q, k, v, backend="sdpa")) < 1e-12


def test_bf16_attention_keeps_fp32_output_when_asked():
    q, k, v = (torch.randn(1, 5, 2, 4).to(torch.bfloat16) for _ in range(3))
    assert mla_attention(q, k, v, keep_output_fp32=True).dtype == torch.float32
    assert mla_attention(q, k, v, keep_output_fp32=False).dtype == torch.bfloat16
    with pytest.raises(ValueError):
        mla_attention(q, k, v, backend="flash")


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("backend", ["manual", "sdpa"])
def test_attention_matches_reference(backend):
    ref()
    from src.mla.attention import mla_attention as ra
    torch.manual_seed(3)
    q = torch.randn(2, 3, 2, 4, dtype=F64)
    k, v = torch.randn(2, 8, 2, 4, dtype=F64), torch.randn(2, 8, 2, 5, dtype=F64)
    km = torch.ones(2, 8, dtype=torch.bool)
    km[0, 6:] = False
    qm = torch.tensor([[True, True, False], [True, True, True]])
    pos = torch.tensor([[3, 4, 5], [5, 6, 7]])
    kw = dict(backend=backend, query_mask=qm, query_positions=pos)
    assert max_diff(mla_attention(q, k, v, km, True, **kw), ra(q, k, v, km, True, **kw)) < 1e-13
    a, pa = mla_attention(q, k, v, km, True, return_attentions=True, **kw)
    b, pb = ra(q, k, v, km, True, return_attentions=True, **kw)
    assert max_diff(a, b) < 1e-13 and max_diff(pa, pb) < 1e-13


# --------------------------------------------------------------------------- caches
def _packed_by_definition(old, old_mask, new, new_mask):
    """Each row keeps its valid old tokens then its valid new tokens, left-packed, zeros after."""
    rows = []
    for i in range(old.shape[0]):
        rows.append(torch.cat((old[i][old_mask[i]], new[i][new_mask[i]]), 0))
    n = max(r.shape[0] for r in rows)
    out = old.new_zeros(old.shape[0], n, old.shape[2])
    for i, r in enumerate(rows):
        out[i, :r.shape[0]] = r
    return out, torch.tensor([r.shape[0] for r in rows])


def test_cache_append_packs_ragged_rows():
    torch.manual_seed(4)
    c = MLACache.empty(3, 5, dtype=F64)
    assert c.cache_length == 0 and c.sequence_offset.tolist() == [0, 0, 0]
    x1 = torch.randn(3, 4, 5, dtype=F64)
    m1 = torch.tensor([[1, 1, 1, 1], [1, 1, 0, 0], [1, 0, 0, 0]], dtype=torch.bool)
    c1 = c.append(x1, m1)
    x2 = torch.randn(3, 2, 5, dtype=F64)
    m2 = torch.tensor([[1, 0], [1, 1], [1, 1]], dtype=torch.bool)
    c2 = c1.append(x2, m2)
    want, lengths = _packed_by_definition(c1.latent_kv, c1.attention_mask, x2, m2)
    assert c2.sequence_offset.tolist() == lengths.tolist() == [5, 4, 3]
    assert max_diff(c2.latent_kv, want) == 0.0
    assert c2.attention_mask.tolist() == (torch.arange(5)[None] < lengths[:, None]).tolist()
    assert c2.cache_elements == 3 * 5 * 5


def test_cache_clone_reorder_and_validation():
    c = MLACache.empty(2, 4, dtype=F64).append(torch.randn(2, 3, 4, dtype=F64))
    d = c.clone()
    assert d.latent_kv is not c.latent_kv and max_diff(d.latent_kv, c.latent_kv) == 0.0
    r = c.reorder(torch.tensor([1, 0]))
    assert max_diff(r.latent_kv, c.latent_kv.flip(0)) == 0.0
    with pytest.raises(ValueError):
        c.reorder(torch.tensor([[0]]))
    with pytest.raises(TypeError):
        c.append(torch.randn(2, 1, 4, dtype=torch.float32))
    with pytest.raises(ValueError):
        c.append(torch.randn(3, 1, 4, dtype=F64))
    with pytest.raises(ValueError):
        c.append(torch.randn(2, 1, 4, dtype=F64), torch.ones(2, 2, dtype=torch.bool))
    with pytest.raises(ValueError):
        c.append(torch.randn(2, 1, 4, dtype=F64), torch.ones(2, 1, dtype=torch.long))
    with pytest.raises(ValueError):
        MLACache(torch.zeros(2, 3), None, torch.zeros(2, dtype=torch.long))
    with pytest.raises(ValueError):
        MLACache(torch.zeros(2, 3, 4), torch.ones(2, 2, dtype=torch.bool), torch.zeros(2, dtype=torch.long))
    with pytest.raises(ValueError):
        MLACache.empty(0, 4)


@needs_reference
@pytest.mark.reference
def test_cache_append_matches_reference():
    ref()
    from src.mla.cache import MLACache as RCache
    torch.manual_seed(5)
    ours, theirs = MLACache.empty(3, 6, dtype=F64), RCache.empty(3, 6, dtype=F64)
    for t in (4, 1, 3):
        x = torch.randn(3, t, 6, dtype=F64)
        m = torch.rand(3, t) < 0.7
        m[:, 0] = True
        ours, theirs = ours.append(x, m), theirs.append(x, m)
        assert max_diff(ours.latent_kv, theirs.latent_kv) == 0.0
        assert torch.equal(ours.attention_mask, theirs.attention_mask)
        assert torch.equal(ours.sequence_offset, theirs.sequence_offset)


def test_static_cache_appends_in_place_and_matches_dynamic_decode():
    m = _module(6).eval()
    x = torch.randn(2, 9, 24, dtype=F64)
    mask = torch.ones(2, 6, dtype=torch.bool)
    mask[1, 4:] = False
    pre = m(x[:, :6], attention_mask=mask, use_cache=True)
    static = StaticMLACache.from_cache(pre.cache, 12)
    buf = static.latent_kv
    dyn = pre.cache
    for i in range(6, 9):
        a = m(x[:, i:i + 1], cache=dyn, use_cache=True)
        b = m(x[:, i:i + 1], cache=static, use_cache=True)
        dyn, static = a.cache, b.cache
        assert max_diff(a.hidden_states, b.hidden_states) < 1e-12
    assert static.latent_kv is buf
    assert static.sequence_offset.tolist() == [9, 7]
    assert static.valid_mask().sum(1).tolist() == [9, 7]
    with pytest.raises(ValueError):
        StaticMLACache.from_cache(pre.cache, 3)
    with pytest.raises(ValueError):
        static.append(torch.randn(2, 2, 12, dtype=F64))


# --------------------------------------------------------------------------- module
def test_nope_attention_is_permutation_invariant_over_the_visible_prefix():
    m = _module(7).eval()
    x = torch.randn(1, 8, 24, dtype=F64)
    perm = torch.cat((torch.randperm(7), torch.tensor([7])))
    a = m(x).hidden_states[:, -1]
    b = m(x[:, perm]).hidden_states[:, -1]
    assert max_diff(a, b) < 1e-12
    with pytest.raises(ValueError):
        m(x, position_ids=torch.arange(8)[None])


@pytest.mark.parametrize("absorbed", [True, False])
def test_prefill_then_decode_equals_full_forward(absorbed):
    m = _module(8).eval()
    m.absorbed_decode = absorbed
    x = torch.randn(2, 11, 24, dtype=F64)
    full = m(x).hidden_states
    pre = m(x[:, :5], use_cache=True)
    cache, outs = pre.cache, [pre.hidden_states]
    for i in range(5, 11):
        st = m(x[:, i:i + 1], cache=cache, use_cache=True)
        cache, _ = st.cache, outs.append(st.hidden_states)
    assert max_diff(torch.cat(outs, 1), full) < 1e-12
    assert cache.sequence_offset.tolist() == [11, 11]


def test_multi_token_chunks_with_a_cache_equal_full_forward():
    m = _module(9).eval()
    x = torch.randn(2, 12, 24, dtype=F64)
    full = m(x).hidden_states
    cache, outs = None, []
    for lo, hi in ((0, 4), (4, 9), (9, 12)):
        st = m(x[:, lo:hi], cache=cache, use_cache=True)
        cache, _ = st.cache, outs.append(st.hidden_states)
    assert max_diff(torch.cat(outs, 1), full) < 1e-12


def test_backends_agree_and_qk_scale_is_recorded():
    a, b = _module(10, attention_backend="manual"), _module(10, attention_backend="sdpa")
    x = torch.randn(2, 7, 24, dtype=F64)
    assert max_diff(a(x).hidden_states, b(x).hidden_states) < 1e-12
    p = a.projections(x)
    want = p.query.square().mean().sqrt() * p.key.square().mean().sqrt() * math.sqrt(4)
    assert abs(a._last_qk_scale.item() - want.item()) < 1e-5


def test_dropout_only_in_training_mode():
    m = _module(11, attention_dropout=0.5, output_dropout=0.5)
    x = torch.randn(1, 6, 24, dtype=F64)
    m.eval()
    assert max_diff(m(x).hidden_states, m(x).hidden_states) == 0.0
    m.train()
    torch.manual_seed(0)
    y1 = m(x).hidden_states
    torch.manual_seed(1)
    y2 = m(x).hidden_states
    assert max_diff(y1, y2) > 0.0


def test_cache_round_trips_through_serialization():
    m = _module(12).eval()
    x = torch.randn(2, 6, 24, dtype=F64)
    cache = m(x, use_cache=True).cache
    buf = io.BytesIO()
    torch.save(cache, buf)
    buf.seek(0)
    loaded = torch.load(buf, weights_only=False)
    tok = torch.randn(2, 1, 24, dtype=F64)
    assert max_diff(m(tok, cache=cache).hidden_states, m(tok, cache=loaded).hidden_states) == 0.0


def test_every_parameter_receives_a_gradient():
    m = _module(13, projection_bias=True, output_gate_bias=True, output_bias=True)
    x = torch.randn(2, 7, 24, dtype=F64)
    mask = torch.ones(2, 7, dtype=torch.bool)
    mask[1, 5:] = False
    m(x, attention_mask=mask).hidden_states.square().sum().backward()
    for name, p in m.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all() and p.grad.abs().sum() > 0, name


def test_gradcheck_small_module():
    m = GatedMLA(GatedMLAConfig(d_model=4, num_heads=2, q_head_dim=2, v_head_dim=2, kv_latent_dim=3)).double()
    x = torch.randn(1, 3, 4, dtype=F64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda t: m(t).hidden_states, (x,))


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("backend", ["manual", "sdpa"])
def test_module_outputs_attentions_gradients_and_diagnostics_match_reference(backend):
    ref()
    from src.mla.config import GatedMLAConfig as RC
    from src.mla.gated_mla import GatedMLA as RM
    kw = dict(attention_backend=backend, projection_bias=True)
    ours = _module(14, **kw)
    theirs = RM(RC(**_cfg(**kw).to_dict())).double()
    theirs.load_state_dict(ours.state_dict())
    x = torch.randn(2, 9, 24, dtype=F64)
    mask = torch.ones(2, 9, dtype=torch.bool)
    mask[0, 7:] = False
    a = ours(x, attention_mask=mask, use_cache=True, output_attentions=True, output_diagnostics=True)
    b = theirs(x, attention_mask=mask, use_cache=True, output_attentions=True, output_diagnostics=True)
    assert max_diff(a.hidden_states, b.hidden_states) < 1e-12
    assert max_diff(a.attentions, b.attentions) < 1e-12
    assert max_diff(a.cache.latent_kv, b.cache.latent_kv) < 1e-13
    assert set(a.diagnostics) == set(b.diagnostics)
    for key in a.diagnostics:
        want = b.diagnostics[key].double()
        assert max_diff(a.diagnostics[key], want) < 1e-6 * (1.0 + want.abs().max().item()), key
    g = torch.randn_like(a.hidden_states)
    a.hidden_states.backward(g)
    b.hidden_states.backward(g)
    tg = dict(theirs.named_parameters())
    for name, p in ours.named_parameters():
        assert max_diff(p.grad, tg[name].grad) < 1e-10, name
