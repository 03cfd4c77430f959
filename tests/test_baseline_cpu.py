"""Baseline causal Transformer (RoPE, MHA with KV cache, SwiGLU) against the reference."""
import pytest
import torch

from _oracle import max_diff, needs_reference, ref
from kimi_k3_b200.models.baseline import BaselineCausalLM, BaselineCausalLMConfig


@needs_reference
@pytest.mark.reference
def test_baseline_lm_matches_reference():
    ref()
    from src.causal_lm import BaselineCausalLM as R, BaselineCausalLMConfig as RC
    torch.manual_seed(0)
    theirs = R(RC(vocab_size=50, d_model=32, n_layers=2, n_heads=4)).double()
    ours = BaselineCausalLM(BaselineCausalLMConfig(vocab_size=50, d_model=32, n_layers=2, n_heads=4)).double()
    ours.load_state_dict(theirs.state_dict())
    ids = torch.randint(0, 50, (3, 17))
    a, b = theirs(ids, labels=ids), ours(ids, labels=ids)
    # the rotary tables are built in float32 in both implementations (rounding differs slightly)
    assert max_diff(a.logits, b.logits) < 1e-7 and abs(a.loss.item() - b.loss.item()) < 1e-6
    a.loss.backward()
    b.loss.backward()
    g = dict(theirs.named_parameters())
    assert max(max_diff(g[n].grad, p.grad) for n, p in ours.named_parameters()) < 1e-7


def test_kv_cache_decode_equals_full():
    torch.manual_seed(1)
    m = BaselineCausalLM(BaselineCausalLMConfig(vocab_size=40, d_model=32, n_layers=2, n_heads=4)).double().eval()
    ids = torch.randint(0, 40, (2, 12))
    full = m(ids).logits
    pre = m(ids[:, :7], use_cache=True)
    outs, cache = [pre.logits], pre.cache
    for i in range(7, 12):
        st = m(ids[:, i:i + 1], cache=cache, use_cache=True)
        outs.append(st.logits)
        cache = st.cache
    assert max_diff(torch.cat(outs, 1), full) < 1e-12
