"""Inference session pieces on CPU: the prompt codec and cache report against the reference's
helpers, the nucleus / top-k filters on tie-free logits, and the streamed audit."""
import pytest
import torch

from _oracle import needs_reference, ref
from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.infer import (CacheReport, InferenceSession, TextCodec, cache_summary, decode_token_ids,
                                encode_prompt, generate_tokens, top_k_filter, top_p_filter)
from kimi_k3_b200.infer.config import GenerationConfig


class _Tok:
    """A toy tokenizer: characters to ids 10.., with the usual special-id attributes."""
    bos_token_id, eos_token_id, pad_token_id = 1, 2, 0
    vocab_size = 200

    def encode(self, text):
        return [10 + (ord(c) % 150) for c in text]

    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(((i - 10) % 150)) if i >= 10 else f"<{i}>" for i in ids)


@needs_reference
def test_codec_matches_reference_helpers():
    ref()
    import importlib
    r = importlib.import_module("inference.tokenization")
    tok = _Tok()
    for prompt in ("hello world", [5, 6, 7], torch.tensor([3, 4, 5])):
        ours = encode_prompt(prompt, tokenizer=tok)
        theirs = r.encode_prompt(prompt, tokenizer=tok)
        assert torch.equal(ours, theirs)
    ids = torch.tensor([[1, 20, 21, 2, 0], [1, 30, 31, 32, 2]])
    assert decode_token_ids(ids, tokenizer=tok) == r.decode_token_ids(ids, tokenizer=tok)
    assert decode_token_ids(ids[:1], tokenizer=tok) == r.decode_token_ids(ids[:1], tokenizer=tok)
    assert TextCodec(tok).special_id("<eos>") == r.tokenizer_token_id(tok, "<eos>")


@needs_reference
@pytest.mark.parametrize("k,p", [(1, 0.3), (5, 0.9), (50, 0.5), (None, 0.999)])
def test_filters_match_reference_without_ties(k, p):
    ref()
    import importlib
    r = importlib.import_module("inference.sampling")
    torch.manual_seed(k or 0)
    logits = torch.randn(4, 97, dtype=torch.float64) * 3
    assert torch.equal(top_k_filter(logits, k), r.top_k_filter(logits, k))
    assert torch.equal(top_p_filter(logits, p), r.top_p_filter(logits, p))


def test_cache_report_counts_shared_buffers_once():
    torch.manual_seed(0)
    m = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double().eval()
    out = generate_tokens(m, torch.randint(5, 128, (2, 7)), generation_config=GenerationConfig(max_new_tokens=2))
    rep = CacheReport.of(out.cache)
    assert rep.as_dict() == cache_summary(out.cache)
    assert rep.num_kda_layers + rep.num_mla_layers == rep.num_layers
    assert rep.sequence_lengths == [9, 9]
    assert rep.memory_bytes > 0
    twice = cache_summary({"a": out.cache, "b": out.cache}["a"])
    assert twice["memory_bytes"] == rep.memory_bytes


def test_session_audit_streams_pieces():
    torch.manual_seed(1)
    m = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double().eval()
    rep = InferenceSession(m).audit(torch.randint(5, 128, (1, 8)), split=3, atol=1e-9, rtol=1e-9)
    assert rep["allclose"] and rep["max_abs_diff"] < 1e-9
    assert rep["cache_stats"]["sequence_lengths"] == [8]
