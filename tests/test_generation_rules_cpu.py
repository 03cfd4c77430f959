"""Generation contract on CPU: generation-config checks, sampling rules (repetition penalty, top-k, top-p,
temperature, NaN safety, seeding), and the generate loop (length limits, EOS with pad fill, ragged
prompts, token accounting, scores, train/eval mode restore).

Oracles: the rules stated in ``inference/sampling.py:10-91`` (penalty divides positive and multiplies
negative logits of seen tokens; top-p keeps the shortest prefix reaching p and always the top token) and
``inference/generation.py:54-194`` (one prefill, then one decode step per token; finished rows emit the
pad id).
"""
import pytest
import torch

from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.infer import GenerationConfig, generate_tokens
from kimi_k3_b200.infer.sampling import (apply_repetition_penalty, safe_argmax, sample_next_token, top_k_filter,
                                         top_p_filter)

NEG = float("-inf")


@pytest.mark.parametrize("bad", [dict(max_new_tokens=-1), dict(temperature=0.0), dict(top_k=0), dict(top_p=0.0),
                                 dict(top_p=1.5), dict(repetition_penalty=0.0), dict(eos_token_id=-1),
                                 dict(device=""), dict(max_total_tokens=0), dict(eos_check_every=0)])
def test_generation_config_rejects_invalid_values(bad):
    with pytest.raises(ValueError):
        GenerationConfig(**bad)


# --------------------------------------------------------------------------- sampling rules
def test_repetition_penalty_rule():
    logits = torch.tensor([[2.0, -2.0, 1.0, -1.0]])
    out = apply_repetition_penalty(logits, torch.tensor([[0, 1, 1]]), 2.0)
    assert out.tolist() == [[1.0, -4.0, 1.0, -1.0]]
    assert apply_repetition_penalty(logits, torch.tensor([[0]]), None) is logits
    assert apply_repetition_penalty(logits, torch.tensor([[0]]), 1.0) is logits
    with pytest.raises(ValueError):
        apply_repetition_penalty(logits, torch.tensor([[0]]), -1.0)


def test_top_k_keeps_the_k_largest_and_their_ties():
    logits = torch.tensor([[1.0, 5.0, 3.0, 4.0, 2.0], [1.0, 2.0, 2.0, 2.0, 0.0]])
    out = top_k_filter(logits, 2)
    assert out[0].tolist() == [NEG, 5.0, NEG, 4.0, NEG]
    assert out[1].tolist() == [NEG, 2.0, 2.0, 2.0, NEG]         # ties with the k-th value survive
    assert top_k_filter(logits, None) is logits and top_k_filter(logits, 9) is logits


def test_top_p_keeps_tokens_whose_mass_ahead_is_within_p():
    # a token survives when the probability mass strictly ahead of it is at most p
    p = torch.tensor([[0.5, 0.3, 0.15, 0.05]])
    logits = p.log()
    assert top_p_filter(logits, 0.45)[0].isfinite().tolist() == [True, False, False, False]
    assert top_p_filter(logits, 0.6)[0].isfinite().tolist() == [True, True, False, False]
    assert top_p_filter(logits, 0.79)[0].isfinite().tolist() == [True, True, False, False]
    assert top_p_filter(logits, 0.81)[0].isfinite().tolist() == [True, True, True, False]
    assert top_p_filter(logits, 1e-6)[0].isfinite().tolist() == [True, False, False, False]  # top always kept
    assert top_p_filter(logits, 1.0) is logits
    shuffled = logits[:, [2, 0, 3, 1]]
    assert top_p_filter(shuffled, 0.6)[0].isfinite().tolist() == [False, True, False, True]


def test_greedy_sampling_is_nan_safe_and_ignores_temperature():
    logits = torch.tensor([[0.1, float("nan"), 0.3], [float("inf"), 0.0, 1.0]])
    assert safe_argmax(logits).tolist() == [[2], [0]]
    cfg = GenerationConfig(temperature=0.01)
    assert torch.equal(sample_next_token(logits, cfg), safe_argmax(logits))
    with pytest.raises(ValueError):
        sample_next_token(logits[0], cfg)


def test_sampling_is_seeded_restricted_and_falls_back_on_invalid_rows():
    torch.manual_seed(0)
    logits = torch.randn(4, 50)
    cfg = GenerationConfig(do_sample=True, top_k=5, temperature=0.7)
    a = sample_next_token(logits, cfg, generator=torch.Generator().manual_seed(3))
    b = sample_next_token(logits, cfg, generator=torch.Generator().manual_seed(3))
    assert torch.equal(a, b)
    top5 = logits.topk(5, -1).indices
    draws = torch.cat([sample_next_token(logits, cfg, generator=torch.Generator().manual_seed(s)) for s in range(40)], 1)
    for r in range(4):
        assert set(draws[r].tolist()) <= set(top5[r].tolist())
    bad = logits.clone()
    bad[1] = float("nan")
    out = sample_next_token(bad, GenerationConfig(do_sample=True), generator=torch.Generator().manual_seed(1))
    assert out.shape == (4, 1) and 0 <= int(out[1]) < 50


def test_low_temperature_sampling_concentrates_on_the_argmax():
    torch.manual_seed(1)
    logits = torch.randn(3, 20)
    cfg = GenerationConfig(do_sample=True, temperature=1e-4)
    for s in range(10):
        assert torch.equal(sample_next_token(logits, cfg, generator=torch.Generator().manual_seed(s)),
                           logits.argmax(-1, keepdim=True))


# --------------------------------------------------------------------------- generate loop
@pytest.fixture(scope="module")
def model():
    torch.manual_seed(0)
    return KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double()


def test_length_limits_and_accounting(model):
    ids = torch.randint(5, 128, (2, 6))
    out = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=4))
    assert out.generated_ids.shape == (2, 4) and out.sequences.shape == (2, 10)
    assert torch.equal(out.sequences[:, :6], ids) and out.finish_reason == "length"
    assert out.prompt_tokens == 6 and out.generated_tokens == 4
    assert out.batch_tokens_per_second == pytest.approx(2 * out.tokens_per_second)
    capped = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=10, max_total_tokens=8))
    assert capped.generated_tokens == 2 and capped.finish_reason == "max_total_tokens"
    none = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=0))
    assert none.generated_ids.shape == (2, 0)
    with pytest.raises(ValueError):
        generate_tokens(model, ids[:, :0])


def test_eos_finishes_rows_and_pads_them(model):
    ids = torch.randint(5, 128, (2, 5))
    greedy = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=6))
    eos = int(greedy.generated_ids[0, 1])                  # row 0 emits this token at step 2
    out = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=6, eos_token_id=eos,
                                                                          pad_token_id=0))
    row0 = out.generated_ids[0].tolist()
    k = row0.index(eos)
    assert all(t == 0 for t in row0[k + 1:])
    assert out.generated_ids[:, :k + 1].tolist()[0] == greedy.generated_ids[0, :k + 1].tolist()
    # the other row keeps generating exactly as without an EOS (the reference's loop raises here,
    # once one row has finished before the others)
    if eos not in greedy.generated_ids[1].tolist():
        assert torch.equal(out.generated_ids[1], greedy.generated_ids[1]) and out.finish_reason == "length"


def test_scores_cache_and_mode_restore(model):
    ids = torch.randint(5, 128, (1, 4))
    model.train()
    out = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=3, return_scores=True,
                                                                          return_cache=False))
    assert model.training                                   # restored after generation
    model.eval()
    assert len(out.scores) == 3 and out.scores[0].shape == (1, 128)
    assert torch.equal(out.scores[0].argmax(-1), out.generated_ids[:, 0])
    assert out.cache is None and out.cache_stats
    assert set(out.to_dict()) >= {"sequences", "generated_ids", "finish_reason", "tokens_per_second"}


def test_left_to_right_ragged_prompts_use_each_rows_last_valid_token(model):
    torch.manual_seed(2)
    a = torch.randint(5, 128, (1, 7))
    b = torch.randint(5, 128, (1, 4))
    padded = torch.cat((a, torch.cat((b, torch.zeros(1, 3, dtype=torch.long)), 1)), 0)
    mask = padded.ne(0)
    out = generate_tokens(model, padded, attention_mask=mask, generation_config=GenerationConfig(max_new_tokens=3))
    alone = generate_tokens(model, b, generation_config=GenerationConfig(max_new_tokens=3))
    assert torch.equal(out.generated_ids[1], alone.generated_ids[0])
    with pytest.raises(TypeError):
        generate_tokens(model, padded, attention_mask=mask.long())


def test_image_prompt_generation_matches_the_full_multimodal_forward():
    torch.manual_seed(0)
    cfg = kimi_k3_cpu_tiny_config()
    m = KimiK3(cfg).double().eval()
    ids = torch.randint(5, 128, (1, 10))
    ids[0, 2:6] = cfg.image_token_id              # a 16x16 image gives 4 tokens after the 2x2 shuffle
    img = torch.randn(1, 3, 16, 16, dtype=torch.float64)
    out = generate_tokens(m, ids, generation_config=GenerationConfig(max_new_tokens=4),
                          prefill_kwargs={"pixel_values": img})
    with torch.no_grad():
        full = m(input_ids=torch.cat((ids, out.generated_ids[:, :3]), 1), pixel_values=img).logits
    assert torch.equal(full[:, -4:].argmax(-1), out.generated_ids)


def test_graph_decoder_and_generate_agree_when_one_row_finishes_first(model):
    from kimi_k3_b200.infer import GraphDecoder
    torch.manual_seed(5)
    ids = torch.randint(5, 128, (2, 7))
    greedy = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=5))
    eos = int(greedy.generated_ids[0, 0])
    if eos in greedy.generated_ids[1].tolist():
        pytest.skip("both rows emit the chosen token")
    cfg = GenerationConfig(max_new_tokens=5, eos_token_id=eos, pad_token_id=0)
    a = generate_tokens(model, ids, generation_config=cfg)
    b = GraphDecoder(model, max_length=16, generation_config=cfg).generate(ids)
    assert torch.equal(a.generated_ids, b.generated_ids)
    assert a.generated_ids[0].tolist() == [eos] + [0] * 4
    assert torch.equal(a.generated_ids[1], greedy.generated_ids[1])


def test_a_generated_placeholder_id_decodes_as_an_ordinary_token():
    """A vision model may emit its image or video placeholder id; the next decode step embeds it as a
    token (the visual inputs were consumed by the prefill) instead of failing the placeholder check."""
    torch.manual_seed(0)
    cfg = kimi_k3_cpu_tiny_config()
    m = KimiK3(cfg).double().eval()
    ids = torch.randint(5, 128, (2, 6))
    with torch.no_grad():
        pre = m.prefill(ids)
        for placeholder in (cfg.image_token_id, cfg.video_token_id):
            st = m.decode_step(torch.full((2, 1), placeholder), pre.cache.clone())
            assert torch.isfinite(st.logits).all()
        with pytest.raises(ValueError):   # in a prompt, a placeholder still needs its image
            m.prefill(torch.tensor([[5, cfg.image_token_id, 6]]))


def test_graph_decoder_serves_image_prompts():
    from kimi_k3_b200.infer import GraphDecoder
    torch.manual_seed(0)
    cfg = kimi_k3_cpu_tiny_config()
    m = KimiK3(cfg).double().eval()
    ids = torch.randint(5, 128, (1, 10))
    ids[0, 2:6] = cfg.image_token_id
    img = torch.randn(1, 3, 16, 16, dtype=torch.float64)
    gcfg = GenerationConfig(max_new_tokens=4)
    eager = generate_tokens(m, ids, generation_config=gcfg, prefill_kwargs={"pixel_values": img})
    served = GraphDecoder(m, max_length=16, generation_config=gcfg).generate(ids, prefill_kwargs={"pixel_values": img})
    assert torch.equal(eager.generated_ids, served.generated_ids)
    with pytest.raises(ValueError):     # the placeholders need their image
        GraphDecoder(m, max_length=16, generation_config=gcfg).generate(ids)
