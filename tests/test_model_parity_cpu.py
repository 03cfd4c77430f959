"""Whole-model oracle: KimiK3 (cpu tiny profile, float64) against the reference implementation.

Same weights (the reference state dict loads unchanged), same inputs: logits, losses, MTP logits
and every parameter gradient agree to float64 round-off; cached prefill + decode equals the full
forward; one hybrid-optimizer step moves every parameter identically.
"""
import pytest
import torch

from _oracle import expand_expert_grads, max_diff, needs_reference, ref
from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config

pytestmark = [needs_reference, pytest.mark.reference]


def _pair(seed=0):
    ref()
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as ref_cfg
    from src.kimi_k3_mini import KimiK3 as RefK3
    torch.manual_seed(seed)
    theirs = RefK3(ref_cfg()).double()
    ours = KimiK3(kimi_k3_cpu_tiny_config()).double()
    missing, unexpected = ours.load_state_dict(theirs.state_dict(), strict=True)
    assert not missing and not unexpected
    return ours, theirs


def test_state_dict_keys_identical():
    ours, theirs = _pair()
    assert set(ours.state_dict().keys()) == set(theirs.state_dict().keys())
    assert sum(p.numel() for p in ours.parameters()) == sum(p.numel() for p in theirs.parameters())


def test_forward_losses_and_gradients_match():
    ours, theirs = _pair()
    ids = torch.randint(5, 128, (3, 70))
    mask = torch.ones(3, 70, dtype=torch.bool)
    mask[1, 50:] = False
    o1 = theirs(input_ids=ids, attention_mask=mask, labels=ids, use_mtp=True)
    o2 = ours(input_ids=ids, attention_mask=mask, labels=ids, use_mtp=True)
    assert max_diff(o1.logits, o2.logits) < 1e-12
    assert max_diff(o1.mtp_logits, o2.mtp_logits) < 1e-12
    assert abs(o1.loss.item() - o2.loss.item()) < 1e-12
    o1.loss.backward()
    o2.loss.backward()
    g1 = {n: p.grad for n, p in theirs.named_parameters() if p.grad is not None}
    g2 = expand_expert_grads((n, p.grad) for n, p in ours.named_parameters())
    assert set(g1) <= set(g2)
    worst = max(max_diff(g1[n], g2[n]) for n in g1)
    assert worst < 1e-12


def test_prefill_decode_equals_full_forward():
    ours, theirs = _pair(1)
    ours.eval()
    theirs.eval()
    ids = torch.randint(5, 128, (2, 12))
    with torch.no_grad():
        full = ours(input_ids=ids).logits
        assert max_diff(full, theirs(input_ids=ids).logits) < 1e-12
        pre = ours.prefill(ids[:, :8])
        cache, outs = pre.cache, [pre.logits]
        for t in range(8, 12):
            st = ours.decode_step(ids[:, t:t + 1], cache)
            cache = st.cache
            outs.append(st.logits)
    assert max_diff(torch.cat(outs, 1), full) < 1e-11


def test_hybrid_optimizer_step_matches_reference():
    ref()
    from training.optimizer.config import KimiOptimizerConfig as RefCfg
    from training.optimizer.hybrid import build_kimi_optimizer as ref_build
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    ours, theirs = _pair(2)
    kw = dict(adamw_lr=1e-3, muon_lr=2e-2, weight_decay=0.1, qk_clip_threshold=5.0)
    opt1, _ = ref_build(theirs, RefCfg(**kw))
    opt2, _ = build_kimi_optimizer(ours, KimiOptimizerConfig(**kw))
    for step in range(2):
        ids = torch.randint(5, 128, (2, 33))
        for model, opt in ((theirs, opt1), (ours, opt2)):
            opt.zero_grad()
            model(input_ids=ids, labels=ids, use_mtp=True).loss.backward()
            opt.step()
        p1 = dict(theirs.named_parameters())
        p2 = expand_expert_grads((n, p.detach()) for n, p in ours.named_parameters())
        worst = max(max_diff(p1[n], p2[n]) for n in p1)
        # Newton-Schulz runs in float32 in both implementations
        assert worst < 1e-5, (step, worst)


@pytest.mark.parametrize("mode,backend", [("full", "eager"), ("block", "two_phase"), ("block", "eager")])
def test_attention_residual_variants_match_reference(mode, backend):
    """Full AttnRes, Block AttnRes eager and two-phase: whole-model logits and gradients."""
    import dataclasses
    ref()
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as ref_cfg
    from src.kimi_k3_mini import KimiK3 as RefK3

    def variant(cfg):
        ar = cfg.backbone.attention_residual_config
        kw = dict(mode=mode, backend=backend)
        if mode == "full":
            kw.update(sublayers_per_depth_block=None, transformer_layers_per_depth_block=None,
                      target_num_depth_blocks=None)
        return dataclasses.replace(cfg, enable_vision=False,
                                   backbone=dataclasses.replace(cfg.backbone,
                                                                attention_residual_config=dataclasses.replace(ar, **kw)))

    torch.manual_seed(4)
    theirs = RefK3(variant(ref_cfg())).double()
    ours = KimiK3(variant(kimi_k3_cpu_tiny_config())).double()
    ours.load_state_dict(theirs.state_dict())
    with torch.no_grad():  # non-zero pseudo-queries so the depth softmax is not uniform
        for (n1, p1), (n2, p2) in zip(sorted(theirs.named_parameters()), sorted(ours.named_parameters())):
            if "pseudo_query" in n1:
                p1.normal_()
                dict(ours.named_parameters())[n1].copy_(p1)
    ids = torch.randint(5, 128, (2, 21))
    o1 = theirs(input_ids=ids, labels=ids, use_mtp=True)
    o2 = ours(input_ids=ids, labels=ids, use_mtp=True)
    assert max_diff(o1.logits, o2.logits) < 1e-12
    o1.loss.backward()
    o2.loss.backward()
    g1 = {n: p.grad for n, p in theirs.named_parameters() if p.grad is not None}
    g2 = expand_expert_grads((n, p.grad) for n, p in ours.named_parameters())
    assert max(max_diff(g1[n], g2[n]) for n in g1) < 1e-12
