"""Pretraining losses on CPU: next-token CE under both alignments and every mask, token weights, label
smoothing, zero-valid policies, the hidden-state (fused-head) form, multi-token prediction with depth
weights, and the composite objective.

Oracles: the alignment rule of ``src/loss/common/validation.py:71-127`` (``causal_shift`` pairs
``logits[:, :-1]`` with ``labels[:, 1:]``), the token-weighted reduction of ``common/reduction.py:10-51``
and the reference loss modules in float64.
"""
import pytest
import torch
import torch.nn.functional as F

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.losses import (KimiPretrainingLoss, MultiTokenPredictionLoss, NextTokenCrossEntropyLoss,
                                        align_token_inputs)

F64 = torch.float64
V = 11


def _inputs(b=2, t=7, seed=0):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(b, t, V, generator=g, dtype=F64) * 2
    labels = torch.randint(0, V, (b, t), generator=g)
    return logits, labels


def _ce_by_definition(logits, labels, valid, weights=None, smoothing=0.0):
    per = F.cross_entropy(logits.reshape(-1, V), labels.masked_fill(~valid, 0).reshape(-1), reduction="none",
                          label_smoothing=smoothing).reshape(labels.shape)
    w = torch.ones_like(per) if weights is None else weights.to(per.dtype)
    w = w * valid
    return (per * w).sum() / w.sum()


# --------------------------------------------------------------------------- next-token CE
def test_causal_shift_pairs_each_position_with_the_next_label():
    logits, labels = _inputs()
    out = NextTokenCrossEntropyLoss()(logits, labels)
    valid = torch.ones(2, 6, dtype=torch.bool)
    assert max_diff(out.loss, _ce_by_definition(logits[:, :-1], labels[:, 1:], valid)) < 2e-6  # CE runs in fp32
    assert out.normalizer.item() == 12 and out.num_valid_tokens.item() == 12


def test_already_aligned_equals_a_manual_shift():
    logits, labels = _inputs(seed=1)
    shifted = NextTokenCrossEntropyLoss()(logits, labels).loss
    aligned = NextTokenCrossEntropyLoss(label_alignment="already_aligned")(logits[:, :-1], labels[:, 1:]).loss
    alias = NextTokenCrossEntropyLoss(alignment="already_aligned")
    assert alias.alignment == "already_aligned"
    assert max_diff(shifted, aligned) < 1e-14
    assert max_diff(alias(logits[:, :-1], labels[:, 1:]).loss, aligned) == 0.0
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss(label_alignment="shift_twice")
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss(label_alignment="causal_shift", alignment="bogus")
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss(label_smoothing=1.0)


def test_masks_combine_as_the_alignment_rule_says():
    logits, labels = _inputs(t=8, seed=2)
    attn = torch.ones(2, 8, dtype=torch.bool)
    attn[1, 6:] = False
    loss_mask = torch.ones(2, 8, dtype=torch.bool)
    loss_mask[0, 3] = False
    boundary = torch.ones(2, 8, dtype=torch.bool)
    boundary[0, 5] = False
    labels[1, 2] = -100
    out = NextTokenCrossEntropyLoss()(logits, labels, attention_mask=attn, loss_mask=loss_mask,
                                      boundary_mask=boundary)
    # a target at t+1 counts when both t and t+1 are attended, t+1 is in the loss mask, is not a
    # document boundary and is not ignore_index
    valid = attn[:, :-1] & attn[:, 1:] & loss_mask[:, 1:] & boundary[:, 1:] & labels[:, 1:].ne(-100)
    assert max_diff(out.loss, _ce_by_definition(logits[:, :-1], labels[:, 1:], valid)) < 2e-6  # CE runs in fp32
    assert out.normalizer.item() == valid.sum().item()
    _, al, v2, _ = align_token_inputs(logits, labels, alignment="causal_shift", attention_mask=attn,
                                      loss_mask=loss_mask, boundary_mask=boundary, token_weights=None,
                                      ignore_index=-100)
    assert torch.equal(v2, valid) and torch.equal(al, labels[:, 1:])


def test_token_weights_and_label_smoothing():
    logits, labels = _inputs(seed=3)
    w = torch.rand(2, 7, dtype=F64) + 0.1
    out = NextTokenCrossEntropyLoss(label_smoothing=0.1)(logits, labels, token_weights=w)
    valid = torch.ones(2, 6, dtype=torch.bool)
    want = _ce_by_definition(logits[:, :-1], labels[:, 1:], valid, w[:, 1:], smoothing=0.1)
    assert max_diff(out.loss, want) < 1e-6  # weights are reduced in fp32
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss()(logits, labels, token_weights=-w)
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss()(logits, labels, token_weights=w[:, :3])


def test_zero_valid_policies():
    logits, labels = _inputs(seed=4)
    logits.requires_grad_(True)
    labels[:] = -100
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss()(logits, labels)
    out = NextTokenCrossEntropyLoss(zero_valid_policy="connected_zero")(logits, labels)
    assert out.loss.item() == 0.0
    out.loss.backward()
    assert logits.grad is not None and logits.grad.abs().max().item() == 0.0
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss(zero_valid_policy="ignore")


def test_invalid_inputs_are_rejected():
    logits, labels = _inputs(seed=5)
    bad = labels.clone()
    bad[0, 3] = V
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss()(logits, bad)
    with pytest.raises(TypeError):
        NextTokenCrossEntropyLoss()(logits, labels.float())
    nan = logits.clone()
    nan[0, 2, 0] = float("nan")
    with pytest.raises(FloatingPointError):
        NextTokenCrossEntropyLoss()(nan, labels)
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss()(logits, labels[:, :5])
    with pytest.raises(ValueError):
        NextTokenCrossEntropyLoss()(logits, labels, attention_mask=torch.ones(2, 6, dtype=torch.bool))


@pytest.mark.parametrize("weighted", [False, True])
def test_hidden_state_form_equals_the_logit_form(weighted):
    torch.manual_seed(6)
    h = torch.randn(2, 7, 5, dtype=F64, requires_grad=True)
    wt = torch.randn(V, 5, dtype=F64, requires_grad=True)
    labels = torch.randint(0, V, (2, 7))
    attn = torch.ones(2, 7, dtype=torch.bool)
    attn[1, 5:] = False
    tw = torch.rand(2, 7, dtype=F64) + 0.5 if weighted else None
    loss = NextTokenCrossEntropyLoss()
    a = loss(h @ wt.T, labels, attention_mask=attn, token_weights=tw).loss
    b = loss.forward_hidden(h, wt, labels, attention_mask=attn, token_weights=tw).loss
    assert max_diff(a, b) < 1e-6
    ga = torch.autograd.grad(a, (h, wt))
    gb = torch.autograd.grad(b, (h, wt))
    for x, y in zip(ga, gb):
        assert max_diff(x, y) < 1e-6


# --------------------------------------------------------------------------- MTP and composite
def test_mtp_loss_per_depth_and_depth_weights():
    g = torch.Generator().manual_seed(7)
    logits = torch.randn(2, 3, 5, V, generator=g, dtype=F64)
    labels = torch.randint(0, V, (2, 3, 5), generator=g)
    mask = torch.rand(2, 3, 5, generator=g) > 0.3
    labels[0, 1, 2] = -100
    dw = (1.0, 0.5, 0.25)
    out = MultiTokenPredictionLoss(depth_weights=dw)(logits, labels, mtp_loss_mask=mask, return_per_depth=True)
    valid = mask & labels.ne(-100)
    per = F.cross_entropy(logits.reshape(-1, V), labels.clamp_min(0).reshape(-1), reduction="none").reshape(2, 3, 5)
    w = valid.double() * torch.tensor(dw, dtype=F64).view(1, 3, 1)
    assert max_diff(out.loss, (per * w).sum() / w.sum()) < 1e-6
    assert out.future_offsets == (2, 3, 4)
    for d in range(3):
        assert max_diff(out.per_depth_loss_sum[d], (per[:, d] * w[:, d]).sum()) < 1e-5
    one = MultiTokenPredictionLoss()(logits[:, 0], labels[:, 0], mtp_loss_mask=mask[:, 0], future_offsets=(2,))
    want = (per[:, 0] * valid[:, 0]).sum() / valid[:, 0].sum()
    assert max_diff(one.loss, want) < 1e-6
    with pytest.raises(ValueError):
        MultiTokenPredictionLoss(depth_weights=(1.0, -1.0))
    with pytest.raises(ValueError):
        MultiTokenPredictionLoss(depth_weights=(1.0,))(logits, labels)
    with pytest.raises(ValueError):
        MultiTokenPredictionLoss()(logits, labels, future_offsets=(2, 3))


def test_composite_is_ntp_plus_weighted_mtp():
    logits, labels = _inputs(seed=8)
    g = torch.Generator().manual_seed(9)
    mlog = torch.randn(2, 5, V, generator=g, dtype=F64)
    mlab = torch.randint(0, V, (2, 5), generator=g)
    loss = KimiPretrainingLoss(lambda_mtp=0.3)
    out = loss(logits=logits, labels=labels, mtp_logits=mlog, mtp_labels=mlab)
    ntp = NextTokenCrossEntropyLoss()(logits, labels).loss
    mtp = MultiTokenPredictionLoss()(mlog, mlab).loss
    assert max_diff(out.loss, ntp + 0.3 * mtp) < 1e-6
    assert loss(logits=logits, labels=labels).mtp is None
    with pytest.raises(ValueError):
        loss(logits=logits, labels=labels, mtp_logits=mlog)
    with pytest.raises(ValueError):
        KimiPretrainingLoss(lambda_mtp=-1.0)


# --------------------------------------------------------------------------- reference parity
@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("alignment", ["causal_shift", "already_aligned"])
@pytest.mark.parametrize("smoothing", [0.0, 0.2])
def test_ntp_matches_reference(alignment, smoothing):
    ref()
    from src.loss.next_token_loss import NextTokenCrossEntropyLoss as RNTP
    logits, labels = _inputs(t=9, seed=10)
    attn = torch.ones(2, 9, dtype=torch.bool)
    attn[0, 7:] = False
    lm = torch.rand(2, 9) > 0.2
    bnd = torch.rand(2, 9) > 0.1
    tw = torch.rand(2, 9, dtype=F64)
    kw = dict(attention_mask=attn, loss_mask=lm, boundary_mask=bnd, token_weights=tw, return_per_token=True)
    a = NextTokenCrossEntropyLoss(alignment=alignment, label_smoothing=smoothing)(logits, labels, **kw)
    b = RNTP(alignment=alignment, label_smoothing=smoothing)(logits, labels, **kw)
    for name in ("loss", "loss_sum", "normalizer", "num_valid_tokens", "per_token_nll", "per_sample_loss_sum",
                 "per_sample_num_tokens"):
        x, y = getattr(a, name), getattr(b, name)
        assert max_diff(x, y) < 1e-10, name


@needs_reference
@pytest.mark.reference
def test_mtp_and_composite_match_reference():
    ref()
    from src.loss.multi_token_prediction_loss import MultiTokenPredictionLoss as RMTP
    from src.loss.pretraining.composite import KimiPretrainingLoss as RComp
    g = torch.Generator().manual_seed(11)
    mlog = torch.randn(2, 2, 6, V, generator=g, dtype=F64)
    mlab = torch.randint(0, V, (2, 2, 6), generator=g)
    mask = torch.rand(2, 2, 6, generator=g) > 0.25
    a = MultiTokenPredictionLoss(depth_weights=(1.0, 0.5))(mlog, mlab, mtp_loss_mask=mask, return_per_depth=True)
    b = RMTP(depth_weights=(1.0, 0.5))(mlog, mlab, mtp_loss_mask=mask, return_per_depth=True)
    assert max_diff(a.loss, b.loss) < 1e-10 and max_diff(a.per_depth_loss_sum, b.per_depth_loss_sum) < 1e-10
    logits, labels = _inputs(seed=12)
    kw = dict(logits=logits, labels=labels, mtp_logits=mlog[:, 0, :5], mtp_labels=mlab[:, 0, :5])
    x, y = KimiPretrainingLoss(lambda_mtp=0.7)(**kw), RComp(lambda_mtp=0.7)(**kw)
    assert max_diff(x.loss, y.loss) < 1e-10
