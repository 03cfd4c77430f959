"""Attention Residuals checks on CPU: config, site math, online softmax, block / full states, controllers.

Oracles: the depth-softmax equation of ``src/attention_residuals/site.py:16-43``
(``softmax_s(q . RMSNorm(src_s))``-weighted sum), the online-softmax merge rule of
``online_softmax.py:10-86``, the block bookkeeping of ``block_state.py:14-114`` and the reference
modules in float64.
"""
import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.attnres import (AttentionResidualConfig, AttentionResidualSite,
                                         BlockAttentionResidualController, BlockAttentionResidualState,
                                         DepthSiteMetadata, FullAttentionResidualController,
                                         FullAttentionResidualState, build_depth_attention_stats,
                                         depth_softmax_stats, merge_depth_softmax_stats,
                                         normalize_depth_softmax_stats, padded_weight_matrix, single_source_stats,
                                         stack_sources, weights_from_stats)

F64 = torch.float64


def _meta(i, block=None):
    return DepthSiteMetadata(i, i // 2, "attention" if i % 2 == 0 else "ffn", None, None, None, block, None)


def _site(i=0, d=8, seed=None, block=None):
    if seed is not None:
        torch.manual_seed(seed)
    s = AttentionResidualSite(d, metadata=_meta(i, block)).double()
    with torch.no_grad():
        s.pseudo_query.normal_()
        s.key_norm.weight.normal_(1.0, 0.3)
    return s


def _mix_by_definition(site, sources):
    keys = sources / torch.sqrt(sources.pow(2).mean(-1, keepdim=True) + site.key_norm.eps) * site.key_norm.weight
    w = torch.softmax(torch.einsum("d,btsd->bts", site.pseudo_query, keys), -1)
    return torch.einsum("bts,btsd->btd", w, sources), w


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("bad", [
    dict(d_model=0),
    dict(mode="sparse"),
    dict(rms_norm_eps=0.0),
    dict(query_init="normal"),
    dict(include_embedding_source=False),
    dict(add_final_output_mixer=False),
    dict(sublayers_per_depth_block=0),
    dict(transformer_layers_per_depth_block=3, sublayers_per_depth_block=4),
    dict(transformer_layers_per_depth_block=None, sublayers_per_depth_block=None),
    dict(mode="full", sublayers_per_depth_block=4),
    dict(mode="full", sublayers_per_depth_block=None, backend="two_phase"),
    dict(backend="fused"),
])
def test_config_rejects_invalid_values(bad):
    kw = dict(d_model=8)
    kw.update(bad)
    with pytest.raises(ValueError):
        AttentionResidualConfig(**kw)


def test_config_block_sizes_and_topology():
    c = AttentionResidualConfig(8, sublayers_per_depth_block=None, transformer_layers_per_depth_block=3)
    assert c.resolved_sublayers_per_depth_block == 6
    assert c.num_depth_blocks(5) == 2  # 10 sublayers in blocks of 6
    assert AttentionResidualConfig(8, sublayers_per_depth_block=4).num_depth_blocks(4) == 2
    assert AttentionResidualConfig(8, mode="full", sublayers_per_depth_block=None).num_depth_blocks(4) == 0
    with pytest.raises(ValueError):
        AttentionResidualConfig(8, mode="full", sublayers_per_depth_block=None).resolved_sublayers_per_depth_block
    with pytest.raises(ValueError):
        c.num_depth_blocks(0)
    t = AttentionResidualConfig(8, sublayers_per_depth_block=4, target_num_depth_blocks=3)
    t.validate_topology(6, every_layer_has_ffn=True)
    with pytest.raises(ValueError):
        t.validate_topology(4, every_layer_has_ffn=True)  # 8 sublayers make 2 blocks
    with pytest.raises(ValueError):
        t.validate_topology(6, every_layer_has_ffn=False)
    AttentionResidualConfig(8, mode="standard", sublayers_per_depth_block=None).validate_topology(
        3, every_layer_has_ffn=False)
    assert AttentionResidualConfig.from_dict(t.to_dict()) == t


@needs_reference
@pytest.mark.reference
def test_config_dict_matches_reference_schema():
    ref()
    from src.attention_residuals.config import AttentionResidualConfig as RC
    ours = AttentionResidualConfig(8, sublayers_per_depth_block=6, backend="two_phase").to_dict()
    theirs = RC(**ours)
    assert theirs.to_dict() == ours
    assert theirs.num_depth_blocks(7) == AttentionResidualConfig(**ours).num_depth_blocks(7)


# --------------------------------------------------------------------------- site math
@pytest.mark.parametrize("s", [1, 2, 5])
def test_site_mix_matches_definition(s):
    site = _site(seed=s)
    src = torch.randn(2, 3, s, 8, dtype=F64)
    out = site(src, return_weights=True, return_logits=True)
    want, w = _mix_by_definition(site, src)
    assert max_diff(out.mixed_state, want) < 1e-13
    assert max_diff(out.weights, w) < 1e-13
    assert max_diff(out.weights.sum(-1), torch.ones(2, 3, dtype=F64)) < 1e-13
    assert max_diff(torch.softmax(out.logits, -1), w) < 1e-13


def test_zero_query_mixes_uniformly_and_one_source_is_identity():
    site = AttentionResidualSite(8).double()
    src = torch.randn(2, 3, 4, 8, dtype=F64)
    out = site(src, return_weights=True)
    assert max_diff(out.weights, torch.full((2, 3, 4), 0.25, dtype=F64)) < 1e-15
    assert max_diff(out.mixed_state, src.mean(2)) < 1e-14
    one = _site(seed=1)(src[:, :, :1])
    assert max_diff(one.mixed_state, src[:, :, 0]) < 1e-15


def test_site_is_equivariant_to_a_common_source_scale():
    site = _site(seed=2)
    src = torch.randn(2, 3, 4, 8, dtype=F64)
    site.key_norm.eps = 1e-30  # the keys are exactly scale-free only without the eps
    a = site(src).mixed_state
    b = site(src * 7.5).mixed_state
    assert max_diff(b, 7.5 * a) < 1e-12


def test_site_validation_and_dtypes():
    site = _site(seed=3)
    with pytest.raises(ValueError):
        site(torch.randn(2, 3, 0, 8, dtype=F64))
    with pytest.raises(ValueError):
        site(torch.randn(2, 3, 8, dtype=F64))
    with pytest.raises(ValueError):
        AttentionResidualSite(8)(torch.randn(1, 1, 2, 8), return_stats=True)
    with pytest.raises(ValueError):
        stack_sources([])
    with pytest.raises(ValueError):
        stack_sources([torch.zeros(1, 2, 8), torch.zeros(1, 3, 8)])
    with pytest.raises(TypeError):
        stack_sources([torch.zeros(1, 2, 8), torch.zeros(1, 2, 8, dtype=F64)])
    bf = AttentionResidualSite(8)
    out = bf(torch.randn(1, 2, 3, 8).to(torch.bfloat16), return_logits=True, return_weights=True)
    assert out.mixed_state.dtype == torch.bfloat16 and out.logits.dtype == torch.float32
    assert out.weights.dtype == torch.float32


def test_site_gradcheck():
    site = _site(seed=4, d=4)
    src = torch.randn(1, 2, 3, 4, dtype=F64, requires_grad=True)
    assert torch.autograd.gradcheck(lambda x: site(x).mixed_state, (src,))
    assert torch.autograd.gradcheck(lambda q: _grad_wrt_query(site, src.detach(), q),
                                    (site.pseudo_query.detach().clone().requires_grad_(),))


def _grad_wrt_query(site, src, q):
    keys = site.key_norm(src)
    w = torch.softmax(torch.einsum("d,btsd->bts", q, keys), -1)
    return torch.einsum("bts,btsd->btd", w, src)


def test_depth_stats_summaries():
    site = _site(seed=5)
    src = torch.randn(2, 3, 4, 8, dtype=F64)
    out = site(src, return_weights=True, return_stats=True, mode="block", number_of_completed_blocks=2,
               has_current_partial=True)
    st = out.stats
    mw = out.weights.float().mean((0, 1))
    assert st.source_count == 4
    assert max_diff(st.mean_weights, mw) < 1e-6
    assert max_diff(st.embedding_weight, mw[0]) < 1e-6
    assert max_diff(st.completed_block_weight_total, mw[1:3].sum()) < 1e-6
    assert max_diff(st.current_partial_weight, mw[-1]) < 1e-6
    assert int(st.dominant_source_index) == int(mw.argmax())
    assert 0.0 <= float(st.normalized_entropy.detach()) <= 1.0 + 1e-6
    mat, mask = padded_weight_matrix([st, site(src[:, :, :2], return_weights=True, return_stats=True).stats])
    assert mat.shape == (2, 4) and mask.sum(1).tolist() == [4, 2]


@needs_reference
@pytest.mark.reference
def test_site_and_stats_match_reference():
    ref()
    from src.attention_residuals.metadata import DepthSiteMetadata as RMeta
    from src.attention_residuals.site import AttentionResidualSite as RSite
    ours = _site(3, seed=6)
    theirs = RSite(8, metadata=RMeta(*[getattr(ours.metadata, f) for f in ours.metadata.__dataclass_fields__]))
    theirs = theirs.double()
    theirs.load_state_dict(ours.state_dict())
    src = torch.randn(2, 5, 4, 8, dtype=F64)
    kw = dict(return_weights=True, return_logits=True, return_stats=True, mode="block",
              number_of_completed_blocks=2, has_current_partial=True)
    a, b = ours(src, **kw), theirs(src, **kw)
    for name in ("mixed_state", "weights", "logits"):
        assert max_diff(getattr(a, name), getattr(b, name)) < 1e-14, name
    for name in ("weight_entropy", "normalized_entropy", "max_weight", "embedding_weight", "mean_retrieval_distance",
                 "completed_block_weight_total", "current_partial_weight"):
        assert max_diff(getattr(a.stats, name), getattr(b.stats, name)) < 1e-6, name
    assert a.stats.source_count == b.stats.source_count


# --------------------------------------------------------------------------- online softmax
@pytest.mark.parametrize("split", [1, 2, 4])
def test_merged_partial_stats_equal_one_softmax(split):
    torch.manual_seed(7)
    logits = torch.randn(2, 3, 5, dtype=F64) * 4
    values = torch.randn(2, 3, 5, 6, dtype=F64)
    whole = depth_softmax_stats(logits, values)
    merged = depth_softmax_stats(logits[..., :split], values[:, :, :split])
    for j in range(split, 5):
        merged = merge_depth_softmax_stats(merged, single_source_stats(logits[..., j], values[:, :, j]))
    want = torch.einsum("bts,btsd->btd", torch.softmax(logits, -1), values)
    assert max_diff(normalize_depth_softmax_stats(merged, F64), want) < 1e-13
    assert max_diff(normalize_depth_softmax_stats(whole, F64), want) < 1e-13
    assert max_diff(weights_from_stats(merged), torch.softmax(logits, -1)) < 1e-13


def test_merge_is_order_independent_and_overflow_safe():
    logits = torch.tensor([[[800.0, -800.0, 799.0]]], dtype=F64)
    values = torch.randn(1, 1, 3, 4, dtype=F64)
    a = merge_depth_softmax_stats(depth_softmax_stats(logits[..., :1], values[:, :, :1]),
                                  depth_softmax_stats(logits[..., 1:], values[:, :, 1:]))
    b = merge_depth_softmax_stats(depth_softmax_stats(logits[..., 1:], values[:, :, 1:]),
                                  depth_softmax_stats(logits[..., :1], values[:, :, :1]))
    out_a, out_b = normalize_depth_softmax_stats(a, F64), normalize_depth_softmax_stats(b, F64)
    assert torch.isfinite(out_a).all() and max_diff(out_a, out_b) < 1e-13
    want = torch.einsum("bts,btsd->btd", torch.softmax(logits, -1), values)
    assert max_diff(out_a, want) < 1e-13


@needs_reference
@pytest.mark.reference
def test_online_softmax_matches_reference():
    ref()
    from src.attention_residuals import online_softmax as ro
    torch.manual_seed(8)
    logits = torch.randn(2, 3, 4, dtype=F64)
    values = torch.randn(2, 3, 4, 5, dtype=F64)
    a = merge_depth_softmax_stats(depth_softmax_stats(logits[..., :3], values[:, :, :3]),
                                  single_source_stats(logits[..., 3], values[:, :, 3]))
    b = ro.merge_depth_softmax_stats(ro.depth_softmax_stats(logits[..., :3], values[:, :, :3]),
                                     ro.single_source_stats(logits[..., 3], values[:, :, 3]))
    assert max_diff(normalize_depth_softmax_stats(a, F64), ro.normalize_depth_softmax_stats(b, F64)) < 1e-14
    assert max_diff(weights_from_stats(a), ro.weights_from_stats(b)) < 1e-14


# --------------------------------------------------------------------------- states and controllers
def test_block_state_bookkeeping():
    emb = torch.randn(1, 2, 8, dtype=F64)
    st = BlockAttentionResidualState(emb, 3)
    outs = [torch.randn(1, 2, 8, dtype=F64) for _ in range(7)]
    for i, o in enumerate(outs):
        st.prepare_for_site()
        st.append_output(o)
    st.finalize()
    assert st.block_sizes == [3, 3, 1]
    assert len(st.completed_blocks) == 3 and st.partial_block is None
    for blk, lo, hi in zip(st.completed_blocks, (0, 3, 6), (3, 6, 7)):
        assert max_diff(blk, sum(outs[lo:hi])) < 1e-14
    assert st.total_sublayer_outputs == 7 and st.current_depth_block_index == 3
    assert st.source_elements == 4 * emb.numel()
    c = st.clone(detach=True)
    assert c.completed_blocks[0] is not st.completed_blocks[0] and c.block_sizes == [3, 3, 1]
    with pytest.raises(ValueError):
        st.append_output(torch.randn(1, 3, 8, dtype=F64))
    full = BlockAttentionResidualState(emb, 1)
    full.append_output(outs[0])
    with pytest.raises(RuntimeError):
        full.append_output(outs[1])  # a full block must be closed first
    with pytest.raises(ValueError):
        BlockAttentionResidualState(emb, 0)
    with pytest.raises(ValueError):
        BlockAttentionResidualState(emb[0], 2)


def test_full_state_bookkeeping():
    emb = torch.randn(1, 2, 8, dtype=F64)
    st = FullAttentionResidualController().initialize(emb)
    for _ in range(3):
        st.append_output(torch.randn(1, 2, 8, dtype=F64))
    assert st.num_sublayer_outputs == 3 and len(st.source_list()) == 4
    assert st.available_sources().shape == (1, 2, 4, 8)
    c = st.clone()
    assert c.sources[1] is not st.sources[1]
    with pytest.raises(ValueError):
        FullAttentionResidualState([], 0)
    with pytest.raises(ValueError):
        FullAttentionResidualState([emb], 1)


def _run_controller(ctrl, sites, final, emb, outs_fn, per_block):
    """Drive a controller like a backbone: each site mixes, a 'sublayer' turns the mix into an output."""
    st = ctrl.initialize(emb)
    mixes = []
    for i, site in enumerate(sites):
        if i % per_block == 0:
            ctrl.prepare_depth_block(st, sites[i:i + per_block])
        m = ctrl.mix_for_site(site, st, return_weights=True).mixed_state
        mixes.append(m)
        ctrl.append_output(st, outs_fn(i, m))
    return mixes, ctrl.finalize(st, final).mixed_state


@pytest.mark.parametrize("per_block", [1, 2, 3, 8])
def test_two_phase_backend_equals_eager(per_block):
    torch.manual_seed(9)
    sites = [_site(i, seed=100 + i, block=i // per_block) for i in range(8)]
    final = _site(8, seed=200)
    emb = torch.randn(2, 3, 8, dtype=F64)
    weights = [torch.randn(8, 8, dtype=F64) * 0.3 for _ in range(8)]
    fn = lambda i, m: torch.tanh(m @ weights[i])  # noqa: E731
    a = _run_controller(BlockAttentionResidualController(per_block, "eager"), sites, final, emb, fn, per_block)
    b = _run_controller(BlockAttentionResidualController(per_block, "two_phase"), sites, final, emb, fn, per_block)
    for x, y in zip(a[0] + [a[1]], b[0] + [b[1]]):
        assert max_diff(x, y) < 1e-12


def test_block_size_one_equals_full_mode():
    torch.manual_seed(10)
    sites = [_site(i, seed=300 + i) for i in range(6)]
    final = _site(6, seed=400)
    emb = torch.randn(1, 4, 8, dtype=F64)
    fn = lambda i, m: torch.sin(m * (i + 1))  # noqa: E731
    a = _run_controller(BlockAttentionResidualController(1), sites, final, emb, fn, 1)
    b = _run_controller(FullAttentionResidualController(), sites, final, emb, fn, 1)
    for x, y in zip(a[0] + [a[1]], b[0] + [b[1]]):
        assert max_diff(x, y) < 1e-13


def test_two_phase_requires_a_prepared_block():
    site = _site(0, seed=11, block=0)
    ctrl = BlockAttentionResidualController(2, "two_phase")
    st = ctrl.initialize(torch.randn(1, 2, 8, dtype=F64))
    with pytest.raises(RuntimeError):
        ctrl.mix_for_site(site, st)
    with pytest.raises(ValueError):
        BlockAttentionResidualController(2, "fused")


def test_build_depth_stats_for_full_mode_has_no_block_fields():
    w = torch.softmax(torch.randn(1, 2, 3, dtype=F64), -1)
    st = build_depth_attention_stats(w, _meta(2), mode="full")
    assert st.completed_block_weight_total is None and st.number_of_completed_blocks is None
    assert st.source_count == 3
