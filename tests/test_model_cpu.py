"""KimiK3 orchestrator and MTP head checks on CPU: config builders, tying, masks, MTP alignment and
fusion, causality, drafts, parameter accounting.

Oracles: the MTP target rule ``h[t] (+) x[t+1] -> x[t+2]`` of ``src/mtp/alignment.py:43-103``, the fusion
``proj(RMSNorm(h) || RMSNorm(E[x]))`` of ``src/mtp/fusion.py:11-47``, the tied head of
``src/kimi_k3_mini.py:183`` and the reference config builders.
"""
import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.models.kimi_k3 import KimiK3Config, kimi_k3_canonical_config, resolve_execution_mode
from kimi_k3_b200.models.mtp import (KimiMTPFusion, build_mtp_feature_mask, build_mtp_training_view,
                                     mtp_parameter_counts)

F64 = torch.float64


def _model(seed=0, **kw):
    torch.manual_seed(seed)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False, **kw)).double()


# --------------------------------------------------------------------------- configs
def test_config_round_trip_and_validation():
    c = kimi_k3_cpu_tiny_config()
    assert KimiK3Config.from_dict(c.to_dict()) == c
    d = c.to_dict()
    with pytest.raises(ValueError):
        KimiK3Config.from_dict({**d, "vocab_size": 0})
    with pytest.raises(ValueError):
        KimiK3Config.from_dict({**d, "pad_token_id": 500})
    with pytest.raises(ValueError):
        KimiK3Config.from_dict({**d, "eos_token_id": 1})          # duplicates bos
    with pytest.raises(ValueError):
        KimiK3Config.from_dict({**d, "vision_token_integration": "concat"})
    with pytest.raises(ValueError):
        KimiK3Config.from_dict({**d, "image_token_id": None})      # vision enabled without a placeholder id
    with pytest.raises(ValueError):
        KimiK3Config.from_dict({**d, "vision_type": "convnext"})


def test_canonical_config_dimensions():
    c = kimi_k3_canonical_config()
    assert (c.d_model, c.vocab_size) == (7168, 160000)
    assert c.backbone.num_pattern_repeats == 23
    assert c.backbone.stable_latent_moe_config.num_routed_experts == 896
    assert c.backbone.attention_residual_config.target_num_depth_blocks == 8


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("builder", ["kimi_k3_cpu_tiny_config", "kimi_k3_canonical_config"])
def test_config_builders_match_reference(builder):
    ref()
    import src.kimi_k3.config as rc
    import kimi_k3_b200.models.kimi_k3 as oc
    ours, theirs = getattr(oc, builder)().to_dict(), getattr(rc, builder)().to_dict()
    assert ours == theirs


# --------------------------------------------------------------------------- orchestrator
def test_lm_head_is_tied_and_padding_row_is_zero():
    m = _model()
    assert m.lm_head.weight is m.embed_tokens.weight
    assert m.embed_tokens.weight[0].abs().max().item() == 0.0
    assert m.mtp.lm_head is m.lm_head and m.mtp.input_embeddings is m.embed_tokens
    ids = {id(p) for p in m.parameters()}
    assert len(ids) == len(list(m.parameters()))  # every shared tensor is registered once
    new = torch.nn.Embedding(128, 16, padding_idx=0).double()
    m.set_input_embeddings(new)
    m.tie_weights()
    assert m.lm_head.weight is new.weight and m.mtp.input_embeddings is new
    with pytest.raises(ValueError):
        m.set_input_embeddings(torch.nn.Embedding(127, 16))


def test_padding_is_derived_from_the_pad_id_and_rows_are_independent():
    m = _model(1).eval()
    ids = torch.randint(5, 128, (2, 10))
    ids[1, 6:] = 0
    with torch.no_grad():
        out = m(input_ids=ids).logits
        alone = m(input_ids=ids[1:, :6]).logits
    assert max_diff(out[1, :6], alone[0]) < 1e-11


def test_execution_mode_resolution_and_argument_checks():
    assert resolve_execution_mode(None, False, 5) == "full"
    assert resolve_execution_mode(None, True, 5) == "prefill"
    m = _model(2)
    ids = torch.randint(5, 128, (2, 6))
    with pytest.raises(ValueError):
        m(input_ids=ids, position_ids=torch.arange(6)[None])
    with pytest.raises(ValueError):
        m(input_ids=ids, training_phase="sft", labels=ids)
    with pytest.raises(ValueError):
        m(input_ids=ids, labels=ids[:, :5])
    with pytest.raises(ValueError):
        m(input_ids=ids, use_cache=True, use_mtp=True)
    with pytest.raises(ValueError):
        m(input_ids=ids, compute_logits=False)
    with pytest.raises(ValueError):
        m.decode_step(ids[:, :1], None)
    with pytest.raises(ValueError):
        _model(3, enable_mtp=False)(input_ids=ids, use_mtp=True)


def test_loss_without_logits_equals_loss_with_logits():
    m = _model(4)
    ids = torch.randint(5, 128, (2, 12))
    a = m(input_ids=ids, labels=ids, use_mtp=True)
    b = m(input_ids=ids, labels=ids, use_mtp=True, compute_logits=False)
    assert b.logits is None
    assert abs(a.loss.item() - b.loss.item()) < 1e-12
    assert abs(a.ntp_loss.loss.item() - b.ntp_loss.loss.item()) < 1e-12
    assert abs(a.mtp_loss.loss.item() - b.mtp_loss.loss.item()) < 1e-12


def test_loss_normalizers_count_the_trained_tokens():
    m = _model(5)
    ids = torch.randint(5, 128, (2, 10))
    ids[1, 7:] = 0
    ntp_n, mtp_n = m.loss_normalizers(ids)
    # double shift: logits[t] vs labels[t+1] over valid pairs -> (T-1) + (7-1)
    assert ntp_n == 9 + 6
    assert mtp_n == 8 + 5


def test_embeddings_input_equals_id_input():
    m = _model(6).eval()
    ids = torch.randint(5, 128, (2, 7))
    with torch.no_grad():
        a = m(input_ids=ids).logits
        b = m(inputs_embeds=m.embed_tokens(ids), attention_mask=torch.ones(2, 7, dtype=torch.bool)).logits
    assert max_diff(a, b) < 1e-13


def test_parameter_report_counts_shared_tensors_once():
    m = _model(7)
    rep = m.parameter_report()
    assert m.num_parameters() == sum(p.numel() for p in m.parameters())
    counts = mtp_parameter_counts(m.mtp)
    assert counts and all(isinstance(v, int) and v >= 0 for v in counts.values())
    assert rep is not None


# --------------------------------------------------------------------------- MTP
def test_mtp_training_view_alignment_and_masks():
    h = torch.randn(2, 8, 4, dtype=F64)
    ids = torch.arange(16).reshape(2, 8)
    mask = torch.ones(2, 8, dtype=torch.bool)
    mask[1, 6:] = False
    labels = ids + 100
    labels[0, 5] = -100
    v = build_mtp_training_view(h, ids, mask, labels)
    assert max_diff(v.source_hidden, h[:, :-2]) == 0.0
    assert torch.equal(v.future_input_ids, ids[:, 1:-1])
    assert torch.equal(v.target_ids, labels[:, 2:])
    want = torch.ones(2, 6, dtype=torch.bool)
    want[0, 3] = False          # labels[0,5] ignored
    want[1, 4:] = False         # targets at 6, 7 are padding
    assert torch.equal(v.valid_mask, want)
    seg = torch.tensor([[0, 0, 0, 1, 1, 1, 1, 1], [0] * 8])
    vs = build_mtp_training_view(h, ids, None, None, seg)
    assert vs.valid_mask[0].tolist() == [True, False, False, True, True, True]
    assert torch.equal(build_mtp_feature_mask(mask, ids), mask[:, :-2] & mask[:, 1:-1] & mask[:, 2:])
    with pytest.raises(ValueError):
        build_mtp_training_view(h[0], ids, mask)
    with pytest.raises(ValueError):
        build_mtp_training_view(h, ids.float(), mask)


def test_mtp_fusion_equation_and_validation():
    torch.manual_seed(8)
    f = KimiMTPFusion(4).double()
    with torch.no_grad():
        f.hidden_norm.weight.normal_()
        f.future_embedding_norm.weight.normal_()
    h, e = torch.randn(2, 3, 4, dtype=F64), torch.randn(2, 3, 4, dtype=F64)
    rms = lambda x, w: x / torch.sqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w  # noqa: E731
    want = torch.cat((rms(h, f.hidden_norm.weight), rms(e, f.future_embedding_norm.weight)), -1) @ f.projection.weight.T
    assert max_diff(f(h, e), want) < 1e-13
    with pytest.raises(ValueError):
        f(h, e[:, :2])
    with pytest.raises(TypeError):
        f(h, e.float())


def test_mtp_logits_are_causal_in_the_inputs():
    m = _model(9).eval()
    ids = torch.randint(5, 128, (1, 12))
    with torch.no_grad():
        a = m(input_ids=ids, use_mtp=True).mtp_logits
        ids2 = ids.clone()
        ids2[:, 9:] = torch.randint(5, 128, (1, 3))
        b = m(input_ids=ids2, use_mtp=True).mtp_logits
    # position t reads h[t] and x[t+1]: rows t <= 7 only see tokens <= 8
    assert max_diff(a[:, :8], b[:, :8]) < 1e-12
    assert a.shape == (1, 10, 128)


def test_mtp_draft_matches_the_training_branch_for_one_position():
    m = _model(10).eval()
    ids = torch.randint(5, 128, (2, 2))
    with torch.no_grad():
        h = m(input_ids=ids[:, :1]).last_hidden_state
        draft = m.mtp.draft_one_step(h, ids[:, 1:2])
        full = m.mtp(torch.cat((h, h, h), 1), torch.cat((ids, ids[:, :1]), 1), compute_loss=False,
                     return_logits=True)
    assert draft.logits.shape == (2, 1, 128)
    assert max_diff(draft.logits, full.logits[:, :1]) < 1e-11
    m.train()
    with pytest.raises(RuntimeError):
        m.mtp.draft_one_step(h, ids[:, 1:2])


def test_mtp_gradients_reach_shared_embeddings_and_backbone():
    m = _model(11)
    ids = torch.randint(5, 128, (2, 9))
    out = m(input_ids=ids, use_mtp=True)
    out.mtp_logits.square().mean().backward()
    assert m.embed_tokens.weight.grad is not None and m.embed_tokens.weight.grad.abs().sum() > 0
    for name, p in m.mtp.named_parameters():
        assert p.grad is not None, name
    assert any(p.grad is not None and p.grad.abs().sum() > 0 for p in m.backbone.parameters())
    det = _model(11, enable_mtp=True)
    det.mtp.config = type(det.mtp.config).from_dict({**det.mtp.config.to_dict(), "detach_backbone_hidden": True})
    det(input_ids=ids, use_mtp=True).mtp_logits.square().mean().backward()
    assert all(p.grad is None or p.grad.abs().sum() == 0 for p in det.backbone.parameters())


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("vision,mtp", [(True, True), (False, True), (False, False)])
def test_parameter_report_and_backbone_counts_match_reference(vision, mtp):
    ref()
    import dataclasses
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as rcfg
    from src.kimi_k3_mini import KimiK3 as RK
    from kimi_k3_b200.models.diagnostics import parameter_counts
    torch.manual_seed(0)
    ours = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=vision, enable_mtp=mtp))
    theirs = RK(rcfg(enable_vision=vision, enable_mtp=mtp))
    assert dataclasses.asdict(ours.parameter_report()) == dataclasses.asdict(theirs.parameter_report())
    assert ours.num_parameters() == theirs.num_parameters()
    assert ours.num_parameters(only_trainable=True) == theirs.num_parameters(only_trainable=True)
    rb = theirs.backbone
    from src.hybrid_backbone.diagnostics import parameter_counts as rcounts
    inner = rb.backbone if hasattr(rb, "backbone") else rb
    want = rcounts(inner.groups, inner.final_global_layer, inner.final_norm,
                   getattr(inner, "final_output_attnres", None))
    got = parameter_counts(ours.backbone.backbone if hasattr(ours.backbone, "backbone") else ours.backbone)
    for key, value in want.items():
        assert got[key] == value, key
