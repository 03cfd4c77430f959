"""Progressive Context Curriculum checks on CPU: stage rules, the token-driven state machine, resume
compatibility, context truncation, dynamic collation and loader rebuilds.

Oracles: the stage rules of ``training/context_curriculum/config.py``, the transition rule of
``curriculum.py`` (stage = first stage whose ``until_tokens`` is not yet reached; never backward) and the
reference modules run on the same inputs.
"""
import pytest
import torch

from _oracle import needs_reference, ref
from kimi_k3_b200.train.curriculum import (ContextCurriculumConfig, ContextStage, ProgressiveContextCollator,
                                           ProgressiveContextCurriculum, build_context_loader, default_stages,
                                           dynamic_collate, pad_batch_to, truncate_batch_to_context)

STAGES = (ContextStage(8, 100), ContextStage(16, 250), ContextStage(32, 600), ContextStage(64, None))


def _cur(enabled=True, **kw):
    base = dict(training_max_seq_len=64, mtp_min_seq_len=3)
    base.update(kw)
    return ProgressiveContextCurriculum(ContextCurriculumConfig(enabled=enabled, stages=STAGES), **base)


# --------------------------------------------------------------------------- config
@pytest.mark.parametrize("stages", [
    (),
    (ContextStage(16, 10), ContextStage(16, None)),                     # lengths must increase
    (ContextStage(8, 10), ContextStage(16, 20)),                        # last stage must be open-ended
    (ContextStage(8, None), ContextStage(16, None)),                    # only the last may be open-ended
    (ContextStage(8, 30), ContextStage(16, 20), ContextStage(32, None)),  # token bounds must increase
])
def test_config_rejects_bad_stages(stages):
    with pytest.raises(ValueError):
        ContextCurriculumConfig(enabled=True, stages=stages)


@pytest.mark.parametrize("kw", [dict(transition_unit="steps"), dict(preserve_optimizer_state=False),
                                dict(preserve_scheduler_state=False)])
def test_config_rejects_unsupported_policies(kw):
    with pytest.raises(ValueError):
        ContextCurriculumConfig(enabled=True, **kw)


def test_stage_validation_and_defaults():
    with pytest.raises(ValueError):
        ContextStage(0, 5)
    with pytest.raises(ValueError):
        ContextStage(8, 0)
    d = default_stages()
    assert [s.max_seq_len for s in d] == [512, 1024, 2048, 4096, 8192] and d[-1].until_tokens is None
    c = ContextCurriculumConfig(enabled=True, stages=[{"max_seq_len": 4, "until_tokens": 9},
                                                      {"max_seq_len": 8, "until_tokens": None}])
    assert c.stages == (ContextStage(4, 9), ContextStage(8, None))
    assert ContextCurriculumConfig.from_dict(c.to_dict()) == c


# --------------------------------------------------------------------------- state machine
@pytest.mark.parametrize("tokens,stage", [(0, 0), (99, 0), (100, 1), (249, 1), (250, 2), (599, 2), (600, 3),
                                          (10 ** 9, 3)])
def test_stage_for_tokens(tokens, stage):
    assert _cur().stage_for_tokens(tokens) == stage


def test_updates_move_forward_only_and_can_skip_stages():
    cur = _cur()
    assert cur.current_max_seq_len() == 8 and cur.enabled
    assert not cur.update(40)
    assert cur.update(700)          # jumps from stage 0 straight to stage 3
    t = cur.last_transition
    assert (t.old_stage_index, t.new_stage_index, t.old_max_seq_len, t.new_max_seq_len) == (0, 3, 8, 64)
    assert t.tokens_seen_at_transition == 700 and t.to_dict()["new_max_seq_len"] == 64
    assert cur.state.transition_count == 1
    assert not cur.update(800) and cur.last_transition is None
    with pytest.raises(ValueError):
        cur.update(10)
    m = cur.metrics()
    assert m["context/stage_index"] == 3.0 and m["context/max_seq_len"] == 64.0 and m["context/tokens_seen"] == 800


def test_disabled_curriculum_uses_the_full_context():
    cur = _cur(enabled=False, model_max_seq_len=48)
    assert cur.current_max_seq_len() == 48 and not cur.update(10 ** 6) and cur.stage_index == 0


def test_limits_and_length_checks():
    with pytest.raises(ValueError):
        _cur(training_max_seq_len=32)               # last stage (64) exceeds the training length
    with pytest.raises(ValueError):
        _cur(model_max_seq_len=32)
    with pytest.raises(ValueError):
        _cur(mtp_min_seq_len=9)                     # first stage (8) too short for MTP
    with pytest.raises(ValueError):
        _cur(training_max_seq_len=0)
    cur = _cur()
    cur.validate_sequence_length(8)
    with pytest.raises(ValueError):
        cur.validate_sequence_length(9)
    cur.validate_valid_tokens(torch.tensor([3, 8]))
    with pytest.raises(ValueError):
        cur.validate_valid_tokens(torch.tensor([2, 8]))


@pytest.mark.parametrize("tokens", [0, 150, 300, 900])
def test_state_dict_round_trip(tokens):
    cur = _cur()
    cur.update(tokens)
    fresh = _cur()
    fresh.load_state_dict(cur.state_dict())
    assert fresh.state == cur.state


@pytest.mark.parametrize("change", [
    dict(stage_index=1, max_seq_len=16),                       # stage does not match its token count
    dict(max_seq_len=16),                                      # inconsistent active length
    dict(stages=[{"max_seq_len": 8, "until_tokens": None}]),   # different stage definition
    dict(training_max_seq_len=128),                            # different training limit
    dict(mtp_min_seq_len=1),
    dict(stage_index=7),
    dict(tokens_seen=-1),
])
def test_incompatible_checkpoints_are_rejected(change):
    cur = _cur()
    cur.update(300)
    st = cur.state_dict()
    st.update(change)
    with pytest.raises(ValueError):
        _cur().load_state_dict(st)


def test_resume_cannot_move_backward():
    early = _cur()
    early.update(120)
    late = _cur()
    late.update(700)
    with pytest.raises(ValueError):
        late.load_state_dict(early.state_dict())


@needs_reference
@pytest.mark.reference
def test_state_machine_matches_reference():
    ref()
    from training.context_curriculum.config import ContextCurriculumConfig as RCfg
    from training.context_curriculum.config import ContextStage as RStage
    from training.context_curriculum.curriculum import ProgressiveContextCurriculum as RCur
    rstages = tuple(RStage(s.max_seq_len, s.until_tokens) for s in STAGES)
    theirs = RCur(RCfg(enabled=True, stages=rstages), training_max_seq_len=64, mtp_min_seq_len=3)
    ours = _cur()
    for tokens in (0, 50, 100, 180, 250, 251, 640, 10 ** 5):
        assert ours.update(tokens) == theirs.update(tokens)
        assert ours.current_max_seq_len() == theirs.current_max_seq_len()
        assert ours.stage_index == theirs.stage_index
    assert ours.state_dict() == theirs.state_dict()


# --------------------------------------------------------------------------- batching
def _batch(lengths, width, *, with_segments=False):
    b = len(lengths)
    ids = torch.zeros(b, width, dtype=torch.long)
    mask = torch.zeros(b, width, dtype=torch.bool)
    for i, n in enumerate(lengths):
        ids[i, :n] = torch.arange(5, 5 + n)
        mask[i, :n] = True
    labels = ids.masked_fill(~mask, -100)
    out = {"input_ids": ids, "labels": labels, "attention_mask": mask, "sample_id": torch.arange(b)}
    if with_segments:
        out["segment_ids"] = torch.zeros(b, width, dtype=torch.long)
    return out


def test_truncation_clips_to_context_then_to_the_longest_row():
    batch = _batch([20, 6], 24)
    out, stats = truncate_batch_to_context(batch, 16)
    assert out["input_ids"].shape == (2, 16) and out["labels"].shape == (2, 16)
    assert torch.equal(out["input_ids"][0], torch.arange(5, 21))
    assert stats["sequence_length"] == 16.0 and stats["valid_tokens"] == 22.0
    assert stats["padding_fraction"] == pytest.approx(1 - 22 / 32)
    short, st = truncate_batch_to_context(_batch([6, 3], 24), 16)
    assert short["input_ids"].shape == (2, 6) and st["sequence_length"] == 6.0
    assert torch.equal(short["sample_id"], torch.arange(2))      # non-sequence fields pass through
    bucket, _ = truncate_batch_to_context(_batch([6, 3], 24), 16, length_multiple=4)
    assert bucket["input_ids"].shape == (2, 8)


def test_truncation_rejects_bad_batches():
    with pytest.raises(ValueError):
        truncate_batch_to_context(_batch([4], 8), 0)
    with pytest.raises(ValueError):
        truncate_batch_to_context({"input_ids": [1, 2]}, 4)
    bad = _batch([4, 4], 8)
    bad["attention_mask"] = bad["attention_mask"].long()
    with pytest.raises(TypeError):
        truncate_batch_to_context(bad, 8)
    left = _batch([4, 4], 8)
    left["attention_mask"] = left["attention_mask"].flip(1)      # left padding
    with pytest.raises(ValueError):
        truncate_batch_to_context(left, 8)
    empty = _batch([4, 4], 8)
    empty["attention_mask"][1] = False
    with pytest.raises(ValueError):
        truncate_batch_to_context(empty, 8)
    packed = _batch([6, 6], 8, with_segments=True)
    packed["segment_ids"][0, 3:] = 1
    with pytest.raises(ValueError):
        truncate_batch_to_context(packed, 8)
    misaligned = _batch([4, 4], 8)
    misaligned["labels"] = misaligned["labels"][:, :6]
    with pytest.raises(ValueError):
        truncate_batch_to_context(misaligned, 8)


def test_truncation_keeps_visual_placeholders_attached():
    batch = _batch([10, 10], 10)
    batch["input_ids"][0, 8] = 3
    batch["pixel_values"] = torch.zeros(1, 3, 4, 4)
    with pytest.raises(ValueError):
        truncate_batch_to_context(batch, 6, image_token_id=3)
    out, _ = truncate_batch_to_context(batch, 9, image_token_id=3)
    assert out["input_ids"].shape == (2, 9)


def test_single_segment_rows_get_a_boundary_mask():
    out, _ = truncate_batch_to_context(_batch([5, 3], 6, with_segments=True), 6)
    assert torch.equal(out["boundary_mask"], out["attention_mask"])


def test_dynamic_collate_pads_each_field_with_its_own_value():
    samples = [{"input_ids": torch.arange(1, 6), "labels": torch.arange(1, 6), "loss_mask": torch.ones(5, dtype=torch.bool),
                "token_weights": torch.ones(5), "idx": 0},
               {"input_ids": torch.arange(1, 3), "labels": torch.arange(1, 3), "loss_mask": torch.ones(2, dtype=torch.bool),
                "token_weights": torch.ones(2), "idx": 1}]
    out = dynamic_collate(samples, pad_token_id=0, ignore_index=-100)
    assert out["input_ids"][1].tolist() == [1, 2, 0, 0, 0]
    assert out["labels"][1].tolist() == [1, 2, -100, -100, -100]
    assert out["loss_mask"][1].tolist() == [True, True, False, False, False]
    assert out["token_weights"][1].tolist() == [1.0, 1.0, 0.0, 0.0, 0.0]
    assert out["attention_mask"].sum(1).tolist() == [5, 2]
    assert out["idx"].tolist() == [0, 1]
    with pytest.raises(ValueError):
        dynamic_collate([], 0, -100)
    wide = pad_batch_to(out, 8, 0, -100)
    assert wide["input_ids"].shape == (2, 8) and wide["labels"][0, 5:].tolist() == [-100] * 3
    assert pad_batch_to(out, 3, 0, -100)["input_ids"].shape == (2, 5)


def test_collator_clips_samples_before_collating():
    samples = [{"input_ids": torch.arange(1, 31), "labels": torch.arange(1, 31)},
               {"input_ids": torch.arange(1, 5), "labels": torch.arange(1, 5)}]
    b = ProgressiveContextCollator(12, pad_token_id=0)(samples)
    assert b["input_ids"].shape == (2, 12) and b["attention_mask"].sum(1).tolist() == [12, 4]
    base_calls = []

    def base(xs):
        base_calls.append([x["input_ids"].shape[0] for x in xs])
        return dynamic_collate(xs, 0, -100)
    ProgressiveContextCollator(8, base_collator=base)(samples)
    assert base_calls == [[8, 4]]
    vis = [{"input_ids": torch.tensor([5, 6, 7, 3]), "pixel_values": torch.zeros(3, 4, 4)}]
    with pytest.raises(ValueError):
        ProgressiveContextCollator(3, image_token_id=3)(vis)


def test_loader_factory_receives_the_active_length():
    assert build_context_loader(lambda max_seq_len: ("kw", max_seq_len), 64) == ("kw", 64)
    assert build_context_loader(lambda n: ("pos", n), 32) == ("pos", 32)
    assert build_context_loader(lambda **kw: kw, 16) == {"max_seq_len": 16}
    with pytest.raises(ValueError):
        build_context_loader(None, 8)
    with pytest.raises(TypeError):
        build_context_loader(lambda: None, 8)


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("lengths,width,limit", [([20, 6], 24, 16), ([6, 3], 24, 16), ([9, 9, 1], 9, 32)])
def test_truncation_and_collation_match_reference(lengths, width, limit):
    ref()
    from training.context_curriculum.batching import ProgressiveContextCollator as RCol
    from training.context_curriculum.batching import truncate_batch_to_context as rt
    batch = _batch(lengths, width)
    a, sa = truncate_batch_to_context(batch, limit)
    b, sb = rt(batch, limit)
    assert set(a) == set(b) and sa == sb
    for key in a:
        assert torch.equal(a[key], b[key]), key
    samples = [{"input_ids": torch.arange(1, n + 1), "labels": torch.arange(1, n + 1)} for n in lengths]
    ca, cb = ProgressiveContextCollator(limit)(samples), RCol(limit)(samples)
    assert set(ca) == set(cb)
    for key in ca:
        assert torch.equal(ca[key], cb[key]), key
