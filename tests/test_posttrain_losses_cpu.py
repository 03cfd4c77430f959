"""Post-training objectives (SFT, Kimi policy loss, MOPD, reward shaping, phase dispatch) against
the reference implementation as an fp64 oracle, on random inputs and on the contract's cases."""
import importlib

import pytest
import torch

from _oracle import needs_reference, ref
from kimi_k3_b200.models import posttrain as ours
from kimi_k3_b200.models.losses import RewardWeights

pytestmark = needs_reference


def _theirs():
    ref()
    return importlib.import_module("src.loss")


def _close(a, b, tol=1e-10):
    if a is None or b is None:
        assert a is None and b is None
        return
    a, b = torch.as_tensor(a).double(), torch.as_tensor(b).double()
    assert torch.allclose(a, b, atol=tol, rtol=tol), (a, b)


@pytest.mark.parametrize("reduction", ["token_mean", "sequence_mean"])
def test_sft_matches_reference(reduction):
    R = _theirs()
    torch.manual_seed(3)
    b, t, v = 3, 9, 13
    logits = torch.randn(b, t, v, dtype=torch.float64)
    labels = torch.randint(0, v, (b, t))
    assistant = torch.rand(b, t) > 0.3
    comp = torch.randint(0, 5, (b, t))
    weights = {1: 2.0, 2: 0.5, 3: 1.0, 4: 1.5}
    samples = torch.tensor([1.0, 0.5, 2.0], dtype=torch.float64)
    outs, grads = [], []
    for mod in (ours.SFTTrajectoryCrossEntropyLoss(reduction=reduction),
                R.SFTTrajectoryCrossEntropyLoss(reduction=reduction)):
        x = logits.clone().requires_grad_()
        o = mod(x, labels, assistant_mask=assistant, component_ids=comp, component_weights=weights,
                sample_weights=samples, return_per_component=True)
        o.loss.backward()
        outs.append(o)
        grads.append(x.grad)
    a, r = outs
    for name in ("loss", "loss_sum", "normalizer", "num_valid_tokens"):
        _close(getattr(a, name), getattr(r, name))
    assert a.per_component_loss_sum.keys() == r.per_component_loss_sum.keys()
    for k in a.per_component_loss_sum:
        _close(a.per_component_loss_sum[k], r.per_component_loss_sum[k])
        _close(a.per_component_num_tokens[k], r.per_component_num_tokens[k])
    _close(grads[0], grads[1])


def test_sft_without_targets_raises():
    logits = torch.randn(1, 4, 5)
    with pytest.raises(ValueError, match="no assistant"):
        ours.SFTTrajectoryCrossEntropyLoss()(logits, torch.zeros(1, 4, dtype=torch.long),
                                             assistant_mask=torch.zeros(1, 4, dtype=torch.bool))


@pytest.mark.parametrize("normalize", [False, True])
@pytest.mark.parametrize("explicit", [False, True])
def test_policy_loss_matches_reference(normalize, explicit):
    R = _theirs()
    torch.manual_seed(5)
    b, t = 6, 7
    cur = torch.randn(b, t, dtype=torch.float64) * 0.3 - 1
    old = cur.detach() + torch.randn(b, t, dtype=torch.float64) * 0.4
    mask = torch.rand(b, t) > 0.25
    kw = dict(advantages=torch.randn(b, dtype=torch.float64)) if explicit else dict(
        rewards=torch.randn(b, dtype=torch.float64), prompt_group_ids=torch.tensor([0, 0, 1, 1, 2, 2]),
        expected_group_size=2)
    cfg = dict(ratio_clip_min=0.8, ratio_clip_max=1.25, log_ratio_l2_coef=0.05, normalize_advantages=normalize)
    outs, grads = [], []
    for mod in (ours.KimiPolicyOptimizationLoss(**cfg), R.KimiPolicyOptimizationLoss(**cfg)):
        x = cur.clone().requires_grad_()
        o = mod(current_logprobs=x, old_logprobs=old, action_mask=mask,
                sample_weights=torch.tensor([1., 2., 1., .5, 1., 1.], dtype=torch.float64), **kw)
        o.loss.backward()
        outs.append(o)
        grads.append(x.grad)
    a, r = outs
    for name in ("loss", "loss_sum", "normalizer", "num_valid_tokens", "policy_objective_sum", "regularization_sum",
                 "mean_advantage", "mean_log_ratio", "max_abs_log_ratio", "clipped_fraction", "mean_reward",
                 "reward_std"):
        _close(getattr(a, name), getattr(r, name))
    _close(grads[0], grads[1])


def test_policy_loss_contract_errors():
    mod = ours.KimiPolicyOptimizationLoss(ratio_clip_min=0.8, ratio_clip_max=1.2, log_ratio_l2_coef=0.1)
    x = torch.zeros(4, 3)
    with pytest.raises(ValueError, match="incomplete"):
        mod(current_logprobs=x, old_logprobs=x, action_mask=torch.ones(4, 3, dtype=torch.bool),
            rewards=torch.ones(4), prompt_group_ids=torch.tensor([0, 0, 0, 1]), expected_group_size=2)
    with pytest.raises(ValueError, match="no action"):
        mod(current_logprobs=x, old_logprobs=x, action_mask=torch.zeros(4, 3, dtype=torch.bool),
            advantages=torch.ones(4))


@pytest.mark.parametrize("mode", ["sampled_token_pg", "kimi_rl_regularized", "topk_reverse_kl"])
@pytest.mark.parametrize("stored", [False, True])
def test_mopd_matches_reference(mode, stored):
    R = _theirs()
    torch.manual_seed(7)
    b, t, k = 4, 6, 5
    student = torch.randn(b, t, dtype=torch.float64) - 1
    teacher = torch.randn(b, t, dtype=torch.float64) - 1
    mask = torch.rand(b, t) > 0.2
    ids = torch.stack([torch.randperm(50)[:k] for _ in range(b * t)]).reshape(b, t, k)
    t_top = torch.log_softmax(torch.randn(b, t, k, dtype=torch.float64), -1)
    s_top = torch.log_softmax(torch.randn(b, t, k, dtype=torch.float64), -1)
    extra = dict(student_logprobs_for_reward=student - 0.2) if stored else {}
    results = []
    for lib in (ours, R):
        pol = lib.KimiPolicyOptimizationLoss(ratio_clip_min=0.8, ratio_clip_max=1.25, log_ratio_l2_coef=0.05)
        mod = lib.MultiTeacherOnPolicyDistillationLoss(reward_clip_max=0.7, mode=mode, policy_loss=pol)
        x = student.clone().requires_grad_()
        st = s_top.clone().requires_grad_()
        o = mod(current_student_logprobs=x, teacher_sampled_token_logprobs=teacher, action_mask=mask,
                teacher_ids=torch.tensor([[0, 1], [2, 2], [1, 0], [0, 0]]), old_student_logprobs=student + 0.1,
                teacher_topk_token_ids=ids, teacher_topk_logprobs=t_top, student_topk_logprobs=st, **extra)
        o.loss.backward()
        results.append((o, x.grad, st.grad))
    (a, ga, sa), (r, gr, sr) = results
    for name in ("loss", "loss_sum", "normalizer", "num_valid_tokens", "mean_token_reward", "reward_clip_fraction",
                 "mean_teacher_logprob", "mean_student_logprob", "mean_teacher_student_gap", "teacher_token_count"):
        _close(getattr(a, name), getattr(r, name), 1e-6)  # fp32 loss arithmetic, summed in another order
    assert a.mode == r.mode and a.reward_reference == r.reward_reference
    _close(ga, gr, 1e-6)
    _close(sa, sr, 1e-6)


def test_mopd_contract_errors():
    mod = ours.MultiTeacherOnPolicyDistillationLoss(reward_clip_max=1.0)
    s = torch.zeros(2, 3)
    with pytest.raises(ValueError, match="teacher IDs"):
        mod(current_student_logprobs=s, teacher_sampled_token_logprobs=s, action_mask=torch.ones(2, 3, dtype=torch.bool),
            teacher_ids=torch.tensor([0, 9]))
    with pytest.raises(ValueError, match="tokenization"):
        mod(current_student_logprobs=s, teacher_sampled_token_logprobs=s, action_mask=torch.ones(2, 3, dtype=torch.bool),
            teacher_ids=torch.tensor([0, 1]), sampled_token_ids=torch.zeros(2, 3, dtype=torch.long),
            teacher_sampled_token_ids=torch.ones(2, 3, dtype=torch.long))


def test_reward_shaping_cases():
    reward = torch.tensor([1.0, 2.0], requires_grad=True)
    with pytest.raises(ValueError, match="explicit"):
        ours.KimiRewardComposer()(verifier_reward=reward, generative_reward=None, task_specific_reward=None,
                                  weights=RewardWeights())
    out = ours.KimiRewardComposer()(verifier_reward=reward, generative_reward=torch.tensor([2.0, 4.0]),
                                    task_specific_reward=None, weights=RewardWeights(verifier=2.0, generative=-0.5))
    assert torch.allclose(out, torch.tensor([1.0, 2.0])) and not out.requires_grad
    r = ours.apply_reasoning_budget_override(torch.tensor([0.5, 0.8]), torch.tensor([10, 21]), torch.tensor([10, 10]),
                                             2.0)
    assert torch.allclose(r, torch.tensor([0.5, -1.0]))
    w = ours.apply_verbosity_binary_rule(torch.tensor([True, True]), torch.tensor([10, 11]), torch.tensor([5, 5]), 2.0)
    assert w.tolist() == [True, False]


def test_objective_dispatch():
    obj = ours.KimiTrainingObjective(ours.KimiLossConfig())
    with pytest.raises(ValueError, match="another phase"):
        obj("sft", logits=torch.randn(1, 3, 4), labels=torch.zeros(1, 3, dtype=torch.long),
            assistant_mask=torch.ones(1, 3, dtype=torch.bool), rewards=torch.ones(1))
    with pytest.raises(ValueError, match="explicitly"):
        obj("rl", current_logprobs=torch.zeros(1, 2), old_logprobs=torch.zeros(1, 2),
            action_mask=torch.ones(1, 2, dtype=torch.bool), advantages=torch.ones(1))
    full = ours.KimiTrainingObjective(ours.KimiLossConfig(rl_ratio_clip_min=0.8, rl_ratio_clip_max=1.2,
                                                          rl_log_ratio_l2_coef=0.1, mopd_reward_clip_max=1.0))
    out = full("rl", current_logprobs=torch.zeros(1, 2, requires_grad=True), old_logprobs=torch.zeros(1, 2),
               action_mask=torch.ones(1, 2, dtype=torch.bool), advantages=torch.ones(1))
    assert out.phase.value == "rl" and torch.isfinite(out.loss)


def test_sft_phase_trains_the_model_through_the_objective():
    """Three optimizer steps on the SFT objective (assistant tokens only) lower its loss; the RL phase
    refuses to run until its unpublished coefficients are configured."""
    from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
    from kimi_k3_b200.models.posttrain import KimiLossConfig, KimiTrainingObjective
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    torch.manual_seed(0)
    m = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False))
    opt, _ = build_kimi_optimizer(m, KimiOptimizerConfig(muon_lr=0.01))
    objective = KimiTrainingObjective(KimiLossConfig())
    ids = torch.randint(5, 128, (2, 12))
    assistant = torch.zeros(2, 12, dtype=torch.bool)
    assistant[:, 6:] = True
    losses = []
    for _ in range(3):
        bundle = objective("sft", logits=m(input_ids=ids).logits, labels=ids, assistant_mask=assistant)
        opt.zero_grad()
        bundle.loss.backward()
        opt.step()
        losses.append(bundle.loss.item())
    assert losses[2] < losses[0]
    with pytest.raises(ValueError):
        objective("rl", current_logprobs=torch.zeros(2, 4), old_logprobs=torch.zeros(2, 4),
                  action_mask=torch.ones(2, 4, dtype=torch.bool), rewards=torch.ones(2))
    with pytest.raises(ValueError):
        objective("sft", logits=m(input_ids=ids).logits, labels=ids, rewards=torch.ones(2))
