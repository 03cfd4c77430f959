"""Hybrid backbone checks on CPU: config rules, layer pattern, standard and AttnRes forwards, caches,
padding, causality, gradients.

Oracles: the layer rules of ``src/hybrid_backbone/config.py`` and ``attention_layer.py:92-344`` (pre-norm
residual layers, or mix / attend / append / mix / FFN / append under AttnRes) and the reference backbone
in float64.
"""
import io

import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.attnres import AttentionResidualConfig
from kimi_k3_b200.models.backbone import HybridAttentionBackbone, HybridBackboneCache, HybridBackboneConfig
from kimi_k3_b200.models.kda import KDAConfig
from kimi_k3_b200.models.mla import GatedMLAConfig
from kimi_k3_b200.models.moe import StableLatentMoEConfig

F64 = torch.float64
D = 16


def _kda():
    return KDAConfig(d_model=D, num_heads=2, key_head_dim=4, value_head_dim=8, chunk_size=4, secondary_tile_size=4)


def _mla():
    return GatedMLAConfig(d_model=D, num_heads=2, q_head_dim=4, v_head_dim=8, kv_latent_dim=8)


def _moe():
    return StableLatentMoEConfig(d_model=D, latent_dim=8, num_shared_experts=1, num_routed_experts=4,
                                 routed_experts_per_token=2, shared_expert_hidden_dim=12,
                                 routed_expert_hidden_dim=12)


def _cfg(groups=1, attnres=None, moe=False, **kw):
    base = dict(d_model=D, num_hybrid_groups=groups, kda_config=_kda(), mla_config=_mla(), mlp_hidden_dim=24)
    if moe:
        base.update(channel_mixer_type="stable_latent_moe", use_dense_ffn=False, stable_latent_moe_config=_moe())
    if attnres is not None:
        base["attention_residual_config"] = attnres
    base.update(kw)
    return HybridBackboneConfig(**base)


def _block_attnres(per_block=4, backend="eager"):
    return AttentionResidualConfig(D, sublayers_per_depth_block=per_block, backend=backend)


def _model(seed=0, **kw):
    torch.manual_seed(seed)
    return HybridAttentionBackbone(_cfg(**kw)).double()


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("bad", [
    dict(attention_pattern=("kda", "gated_mla")),                         # canonical pattern enforced
    dict(attention_pattern=("kda", "lstm"), enforce_canonical_pattern=False),
    dict(add_final_gated_mla=False),
    dict(kda_config=None),
    dict(mla_config=None),
    dict(rms_norm_eps=0.0),
    dict(residual_dropout=1.0),
    dict(channel_mixer_type="conv"),
    dict(use_dense_ffn=False),
    dict(channel_mixer_type="stable_latent_moe"),                          # MoE with the dense FFN still on
    dict(stable_latent_moe_config=_moe()),                                 # MoE config without MoE mixing
    dict(activation="gelu"),
    dict(attention_residual_config=AttentionResidualConfig(8)),            # width mismatch
    dict(attention_residual_config=AttentionResidualConfig(D, sublayers_per_depth_block=4,
                                                           target_num_depth_blocks=7)),
])
def test_config_rejects_invalid_values(bad):
    with pytest.raises(ValueError):
        _cfg(**bad)


def test_config_counts_and_round_trip():
    c = _cfg(groups=3, attnres=_block_attnres())
    assert c.num_group_layers == 12 and c.num_attention_layers == 13
    assert c.num_kda_layers == 9 and c.num_mla_layers == 4
    assert c.depth_mixing == "block" and c.resolved_mlp_hidden_dim == 24
    assert _cfg(mlp_hidden_dim=None).resolved_mlp_hidden_dim == 4 * D
    assert HybridBackboneConfig.from_dict(c.to_dict()) == c
    free = _cfg(attention_pattern=("gated_mla", "kda"), enforce_canonical_pattern=False, add_final_gated_mla=False)
    assert free.num_attention_layers == 2 and free.num_mla_layers == 1


def test_layer_pattern_and_parameter_names():
    m = _model(groups=2)
    assert m.attention_types == ("kda", "kda", "kda", "gated_mla") * 2 + ("gated_mla_final",)
    assert len(m.layers) == 9
    mm = _model(groups=1, moe=True)
    assert all(layer.moe is not None for layer in mm.layers)


@needs_reference
@pytest.mark.reference
def test_config_dict_matches_reference_schema():
    ref()
    from src.hybrid_backbone.config import HybridBackboneConfig as RC
    ours = _cfg(groups=2, attnres=_block_attnres()).to_dict()
    theirs = RC.from_dict(ours)
    assert theirs.to_dict() == ours
    assert theirs.num_attention_layers == 9


# --------------------------------------------------------------------------- forwards
VARIANTS = {
    "standard": dict(),
    "standard_moe": dict(moe=True),
    "full_attnres": dict(attnres=AttentionResidualConfig(D, mode="full", sublayers_per_depth_block=None)),
    "block_attnres": dict(attnres=_block_attnres(4)),
    "block_two_phase": dict(attnres=_block_attnres(4, "two_phase")),
    "block_attnres_moe": dict(attnres=_block_attnres(6), moe=True),
}


@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_prefill_then_decode_equals_full_forward(variant):
    m = _model(1, groups=2, **VARIANTS[variant]).eval()
    x = torch.randn(2, 9, D, dtype=F64)
    full = m(x).last_hidden_state
    pre = m(x[:, :6], use_cache=True, mode="prefill")
    cache, outs = pre.cache, [pre.last_hidden_state]
    for i in range(6, 9):
        st = m(x[:, i:i + 1], cache=cache, use_cache=True, mode="decode")
        cache, _ = st.cache, outs.append(st.last_hidden_state)
    assert max_diff(torch.cat(outs, 1), full) < 1e-11
    assert cache.sequence_length == 9 and cache.sequence_lengths.tolist() == [9, 9]


@pytest.mark.parametrize("variant", ["standard", "block_attnres"])
def test_padded_rows_match_their_unpadded_runs(variant):
    m = _model(2, **VARIANTS[variant]).eval()
    x = torch.randn(2, 8, D, dtype=F64)
    mask = torch.ones(2, 8, dtype=torch.bool)
    mask[1, 5:] = False
    out = m(x, attention_mask=mask).last_hidden_state
    alone = m(x[1:, :5]).last_hidden_state
    assert max_diff(out[1, :5], alone[0]) < 1e-11
    assert max_diff(out[0], m(x[:1]).last_hidden_state[0]) < 1e-11


@pytest.mark.parametrize("variant", ["standard_moe", "full_attnres", "block_two_phase"])
def test_backbone_is_causal(variant):
    m = _model(3, **VARIANTS[variant]).eval()
    x = torch.randn(1, 10, D, dtype=F64)
    y = m(x).last_hidden_state
    x2 = x.clone()
    x2[:, 7:] = torch.randn(1, 3, D, dtype=F64)
    assert max_diff(m(x2).last_hidden_state[:, :7], y[:, :7]) < 1e-12


def test_standard_layer_is_pre_norm_residual():
    m = _model(4).eval()
    layer = m.layers[0]
    x = torch.randn(1, 5, D, dtype=F64)
    out = layer(x, None).hidden_states
    h = x + layer.attention(layer.attention_norm(x)).hidden_states
    want = h + layer.ffn(layer.ffn_norm(h))
    assert max_diff(out, want) < 1e-13


def test_hidden_states_and_depth_outputs():
    m = _model(5, groups=2, attnres=_block_attnres(4)).eval()
    x = torch.randn(2, 4, D, dtype=F64)
    out = m(x, output_hidden_states=True, output_depth_weights=True)
    n = len(m.layers)
    assert max_diff(out.hidden_states[0], x) == 0.0
    tr = out.hidden_state_trace
    assert max_diff(tr.embedding, x) == 0.0
    assert len(tr.pre_attention) == len(tr.attention_outputs) == len(tr.pre_ffn) == len(tr.ffn_outputs) == n
    # the final mixer reads the same sources the last site saw plus the last FFN output
    assert max_diff(m.final_norm(tr.final_mixed), out.last_hidden_state) < 1e-13
    d = out.depth_outputs
    assert d.mode == "block" and len(d.site_stats) == 2 * len(m.layers)
    assert d.num_depth_blocks == m.config.attention_residual_config.num_depth_blocks(len(m.layers))
    assert d.averaged_weight_matrix.shape[0] == 2 * len(m.layers) + 1
    s = m(x).last_hidden_state
    assert max_diff(out.last_hidden_state, s) < 1e-13


def test_cache_clone_reorder_and_accounting():
    m = _model(6, groups=2).eval()
    x = torch.randn(3, 5, D, dtype=F64)
    cache = m(x, use_cache=True, mode="prefill").cache
    assert isinstance(cache, HybridBackboneCache) and len(cache.layer_caches) == len(m.layers)
    kda = m.config.kda_config
    per_kda = 3 * (kda.num_heads * kda.key_head_dim * kda.value_head_dim
                   + (kda.short_conv_kernel_size - 1) * (2 * kda.key_width + kda.value_width))
    assert cache.kda_elements == 6 * per_kda
    assert cache.mla_elements == 3 * 3 * 5 * m.config.mla_config.kv_latent_dim
    assert cache.total_elements == cache.kda_elements + cache.mla_elements
    idx = torch.tensor([2, 0])
    r = cache.reorder(idx)
    tok = torch.randn(3, 1, D, dtype=F64)
    a = m(tok, cache=cache.clone(), mode="decode").last_hidden_state
    b = m(tok[idx], cache=r, mode="decode").last_hidden_state
    assert max_diff(b, a[idx]) < 1e-12
    buf = io.BytesIO()
    torch.save(cache, buf)
    buf.seek(0)
    loaded = torch.load(buf, weights_only=False)
    assert max_diff(m(tok, cache=loaded, mode="decode").last_hidden_state, a) == 0.0


def test_input_validation():
    m = _model(7)
    x = torch.randn(2, 3, D, dtype=F64)
    with pytest.raises(ValueError):
        m(x, mode="decode")
    with pytest.raises(ValueError):
        m(x, mode="stream")
    with pytest.raises(ValueError):
        m(x[:, :0])
    with pytest.raises(ValueError):
        m(torch.randn(2, 3, D + 1, dtype=F64))
    with pytest.raises(ValueError):
        m(x, attention_mask=torch.ones(2, 2, dtype=torch.bool))


@pytest.mark.parametrize("variant", ["standard_moe", "block_attnres"])
def test_every_parameter_receives_a_gradient(variant):
    m = _model(8, **VARIANTS[variant])
    x = torch.randn(2, 6, D, dtype=F64)
    m(x).last_hidden_state.square().sum().backward()
    for name, p in m.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("variant", sorted(VARIANTS))
def test_forward_and_gradients_match_reference(variant):
    ref()
    from _oracle import expand_expert_grads
    from src.hybrid_backbone.backbone import HybridAttentionBackbone as RB
    from src.hybrid_backbone.config import HybridBackboneConfig as RC
    ours = _model(9, groups=2, **VARIANTS[variant])
    theirs = RB(RC.from_dict(ours.config.to_dict())).double()
    missing, unexpected = theirs.load_state_dict(ours.state_dict(), strict=False)
    assert not missing and not unexpected
    x = torch.randn(2, 7, D, dtype=F64)
    mask = torch.ones(2, 7, dtype=torch.bool)
    mask[0, 5:] = False
    a = ours(x, attention_mask=mask).last_hidden_state
    b = theirs(x, attention_mask=mask).last_hidden_state
    assert max_diff(a, b) < 1e-11
    g = torch.randn_like(a)
    a.backward(g)
    b.backward(g)
    og = expand_expert_grads((n, p.grad) for n, p in ours.named_parameters())
    for n, p in theirs.named_parameters():
        if p.grad is not None:
            assert max_diff(og[n], p.grad) < 1e-10, n
