"""Inference on CPU: cached greedy generation equals full-forward greedy, ragged prompts,
sampling helpers against the reference, audit, checkpoint loading from YAML."""
import pytest
import torch

from _oracle import needs_reference, ref
from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.infer import (GenerationConfig, apply_repetition_penalty, compare_full_vs_cached_logits,
                                generate_tokens, inference_autoregressive, sample_next_token, top_k_filter,
                                top_p_filter)


def _model():
    torch.manual_seed(0)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double().eval()


def test_cached_greedy_equals_full_forward_greedy():
    m = _model()
    ids = torch.randint(5, 128, (2, 9))
    out = generate_tokens(m, ids, generation_config=GenerationConfig(max_new_tokens=6))
    seq = ids
    with torch.no_grad():
        for _ in range(6):
            nxt = m(input_ids=seq).logits[:, -1].argmax(-1, keepdim=True)
            seq = torch.cat((seq, nxt), 1)
    assert torch.equal(out.sequences, seq) and out.generated_tokens == 6 and out.finish_reason == "length"
    assert out.cache_stats["sequence_lengths"] == [15, 15]


def test_ragged_prompts_match_individual_generation():
    m = _model()
    a, b = torch.randint(5, 128, (1, 9)), torch.randint(5, 128, (1, 5))
    ids = torch.zeros(2, 9, dtype=torch.long)
    ids[0], ids[1, :5] = a[0], b[0]
    mask = torch.zeros(2, 9, dtype=torch.bool)
    mask[0], mask[1, :5] = True, True
    cfg = GenerationConfig(max_new_tokens=4)
    batched = generate_tokens(m, ids, generation_config=cfg, attention_mask=mask)
    ra = generate_tokens(m, a, generation_config=cfg)
    rb = generate_tokens(m, b, generation_config=cfg)
    assert torch.equal(batched.generated_ids[0], ra.generated_ids[0])
    assert torch.equal(batched.generated_ids[1], rb.generated_ids[0])


def test_eos_stops_and_pads():
    m = _model()
    ids = torch.randint(5, 128, (1, 6))
    first = generate_tokens(m, ids, generation_config=GenerationConfig(max_new_tokens=1)).generated_ids[0, 0].item()
    out = generate_tokens(m, ids, generation_config=GenerationConfig(max_new_tokens=5, eos_token_id=first))
    assert out.finish_reason == "eos" and out.generated_tokens == 1


def test_audit_and_autoregressive_api():
    m = _model()
    rep = compare_full_vs_cached_logits(m, torch.randint(5, 128, (2, 10)), atol=1e-9, rtol=1e-9)
    assert rep["allclose"], rep["max_abs_diff"]
    out = inference_autoregressive(m, [5, 6, 7], max_new_tokens=3)
    assert out.sequences.shape == (1, 6) and int(out.sequences[0, 0]) == 5  # id lists get no extra <bos>


def test_sampling_is_seeded_and_filtered():
    torch.manual_seed(0)
    logits = torch.randn(3, 50)
    cfg = GenerationConfig(do_sample=True, top_k=5, top_p=0.9, temperature=0.7)
    g1 = torch.Generator().manual_seed(3)
    g2 = torch.Generator().manual_seed(3)
    a = sample_next_token(logits, cfg, generator=g1)
    b = sample_next_token(logits, cfg, generator=g2)
    assert torch.equal(a, b)
    top5 = torch.topk(logits, 5, -1).indices
    assert all(int(a[i]) in top5[i].tolist() for i in range(3))
    nan = logits.clone()
    nan[0, 3] = float("nan")
    assert sample_next_token(nan, cfg, generator=g1).shape == (3, 1)


@needs_reference
@pytest.mark.reference
def test_sampling_helpers_match_reference():
    ref()
    from inference.sampling import apply_repetition_penalty as rrp, top_k_filter as rtk, top_p_filter as rtp
    torch.manual_seed(1)
    logits = torch.randn(4, 30)
    prev = torch.randint(0, 30, (4, 7))
    assert torch.equal(apply_repetition_penalty(logits, prev, 1.3), rrp(logits, prev, 1.3))
    assert torch.equal(top_k_filter(logits, 4), rtk(logits, 4))
    assert torch.equal(top_p_filter(logits, 0.8), rtp(logits, 0.8))


# ------------------------------------------------------------------ serving decoder (eager on CPU)
def test_graph_decoder_matches_generate_tokens():
    from kimi_k3_b200.infer import GraphDecoder
    m = _model()
    ids = torch.randint(5, 128, (2, 9))
    for cfg in (GenerationConfig(max_new_tokens=6),
                GenerationConfig(max_new_tokens=5, do_sample=True, top_k=20, top_p=0.9, temperature=0.8,
                                 repetition_penalty=1.3, seed=7)):
        ref_out = generate_tokens(m, ids, generation_config=cfg)
        out = GraphDecoder(m, max_length=32, generation_config=cfg).generate(ids)
        assert torch.equal(out.sequences, ref_out.sequences), (out.sequences, ref_out.sequences)
        assert out.cache_stats["sequence_lengths"] == [9 + cfg.max_new_tokens - 1] * 2


def test_graph_decoder_ragged_prompts_and_eos():
    from kimi_k3_b200.infer import GraphDecoder
    m = _model()
    ids = torch.randint(5, 128, (2, 9))
    mask = torch.ones(2, 9, dtype=torch.bool)
    mask[1, 5:] = False
    cfg = GenerationConfig(max_new_tokens=4)
    ref_out = generate_tokens(m, ids, generation_config=cfg, attention_mask=mask)
    out = GraphDecoder(m, max_length=16, generation_config=cfg).generate(ids, mask)
    assert torch.equal(out.generated_ids, ref_out.generated_ids)
    first = int(ref_out.generated_ids[0, 0])
    cfg = GenerationConfig(max_new_tokens=6, eos_token_id=first, pad_token_id=0)
    ref_out = generate_tokens(m, ids[:1], generation_config=cfg)
    out = GraphDecoder(m, max_length=16, generation_config=cfg).generate(ids[:1])
    assert out.finish_reason == ref_out.finish_reason == "eos"
    assert torch.equal(out.generated_ids, ref_out.generated_ids)


def test_static_mla_cache_appends_in_place():
    from kimi_k3_b200.models.mla import MLACache, StaticMLACache
    lat = torch.randn(2, 3, 4)
    mask = torch.tensor([[True, True, True], [True, True, False]])
    c = MLACache(lat, mask, mask.sum(1))
    s = StaticMLACache.from_cache(c, 6)
    buf = s.latent_kv
    new = torch.randn(2, 1, 4)
    assert s.append(new) is s and s.latent_kv is buf
    assert s.sequence_offset.tolist() == [4, 3]
    assert torch.equal(buf[0, 3], new[0, 0]) and torch.equal(buf[1, 2], new[1, 0])
    assert s.valid_mask().tolist() == [[True] * 4 + [False] * 2, [True] * 3 + [False] * 3]
