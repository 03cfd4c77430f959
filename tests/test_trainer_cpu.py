"""Token-exact accumulation windows against the reference trainer (float64, CPU)."""
import dataclasses

import pytest
import torch

from _oracle import expand_expert_grads, max_diff, needs_reference, ref
from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.train.engine import MoEController
from kimi_k3_b200.train.loop import eval_one_epoch, next_token_preview, train_one_epoch
from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer


def _batches(n=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for i in range(n):
        ids = torch.randint(5, 128, (2, 26), generator=g)
        mask = torch.ones(2, 26, dtype=torch.bool)
        mask[1, 18 + i:] = False  # ragged valid counts: window normalisers matter
        out.append({"input_ids": ids, "labels": ids.clone(), "attention_mask": mask})
    return out


@needs_reference
@pytest.mark.reference
def test_streaming_windows_match_reference_trainer():
    ref()
    from src.kimi_k3.config import kimi_k3_cpu_tiny_config as ref_cfg
    from src.kimi_k3_mini import KimiK3 as RefK3
    from training.moe_control import MoEController as RefMoE
    from training.optimizer.config import KimiOptimizerConfig as RefCfg
    from training.optimizer.hybrid import build_kimi_optimizer as ref_build
    from training.train_one_epoch import train_one_epoch as ref_train
    torch.manual_seed(0)
    theirs = RefK3(dataclasses.replace(ref_cfg(), enable_vision=False)).double()
    ours = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False)).double()
    ours.load_state_dict(theirs.state_dict())
    kw = dict(adamw_lr=1e-3, muon_lr=1e-2)
    o1, _ = ref_build(theirs, RefCfg(**kw))
    o2, _ = build_kimi_optimizer(ours, KimiOptimizerConfig(**kw))
    data = _batches()
    r1 = ref_train(theirs, data, o1, grad_accum_steps=3, grad_clip=1.0, use_mtp=True, moe_controller=RefMoE(theirs))
    r2 = train_one_epoch(ours, data, o2, grad_accum_steps=3, grad_clip=1.0, use_mtp=True,
                         moe_controller=MoEController(ours))
    assert r2["optimizer_steps"] == r1["optimizer_steps"] == 2
    assert abs(r1["loss"] - r2["loss"]) < 1e-9 and r1["ntp_tokens"] == r2["ntp_tokens"]
    p1 = dict(theirs.named_parameters())
    p2 = expand_expert_grads((n, p.detach()) for n, p in ours.named_parameters())
    # fp32 Newton-Schulz (batched here, per matrix there) rounds differently: ~1e-6 per step
    assert max(max_diff(p1[n], p2[n]) for n in p1) < 2e-5


def test_eval_and_preview():
    torch.manual_seed(1)
    m = KimiK3(kimi_k3_cpu_tiny_config(enable_vision=False))
    data = _batches(3)
    stats = eval_one_epoch(m, data, use_mtp=True)
    assert stats["num_batches"] == 3 and stats["perplexity"] > 1 and m.training
    prev = next_token_preview(m, data[0], sample_index=1, max_tokens=8)
    assert prev["position"] == 17 and len(prev["predicted_ids"]) == 8


def test_yaml_trainer_end_to_end_and_resume(tmp_path):
    """The cpu_smoke pipeline trains through ``train_kimi_from_yaml``, checkpoints, and resumes."""
    import yaml
    from kimi_k3_b200.config.model_yaml import build_model_from_yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    from kimi_k3_b200.data import build_dataloaders_from_yaml
    from kimi_k3_b200.train.trainer import train_kimi_from_yaml
    d = write_pipeline("cpu_smoke", tmp_path / "prof")
    tr = yaml.safe_load((d / "training.yaml").read_text())
    tr["checkpoint"]["output_dir"] = str(tmp_path / "ckpt")
    tr["training"]["epochs"] = 2
    tr["runtime"]["verbose"] = False
    tr["runtime"]["use_ema"] = True
    (d / "training.yaml").write_text(yaml.safe_dump(tr))
    data = build_dataloaders_from_yaml(d / "data.yaml")
    torch.manual_seed(0)
    model = build_model_from_yaml(d / "model.yaml", data_bundle=data)
    res = train_kimi_from_yaml(d / "training.yaml", model=model, data=data)
    assert res["state"].optimizer_step == 16 and res["state"].epoch == 2
    assert len(res["history"]["validation"]) == 2 and res["last_checkpoint"].is_file()
    assert (tmp_path / "ckpt" / "latest").is_file()
    # resume from the epoch-0 checkpoint and finish epoch 1 again: same final weights
    tr["checkpoint"]["resume_from"] = str(tmp_path / "ckpt" / "kimi_k3_cpu_smoke_epoch_0000.pt")
    tr["checkpoint"]["output_dir"] = str(tmp_path / "ckpt2")
    (d / "training.yaml").write_text(yaml.safe_dump(tr))
    data2 = build_dataloaders_from_yaml(d / "data.yaml")
    model2 = build_model_from_yaml(d / "model.yaml", data_bundle=data2)
    res2 = train_kimi_from_yaml(d / "training.yaml", model=model2, data=data2)
    assert res2["state"].optimizer_step == 16
    # equal up to the order of multi-threaded CPU reductions (a missed RNG, optimizer or
    # scheduler state would differ by far more)
    for (n, p), (_, q) in zip(res["model"].named_parameters(), res2["model"].named_parameters()):
        torch.testing.assert_close(p, q, rtol=1e-5, atol=1e-6, msg=n)


def test_yaml_trainer_with_context_curriculum_transitions_and_resumes(tmp_path):
    """A two-stage curriculum (16 then 32 tokens) through ``train_kimi_from_yaml``: the run moves to the
    second stage, the curriculum state rides in the checkpoint, and a run resumed from the first
    epoch's checkpoint ends in the same curriculum state with the same token count."""
    import yaml
    from kimi_k3_b200.config.model_yaml import build_model_from_yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    from kimi_k3_b200.data import build_dataloaders_from_yaml
    from kimi_k3_b200.train.checkpoints import list_checkpoints
    from kimi_k3_b200.train.trainer import train_kimi_from_yaml
    d = write_pipeline("cpu_smoke", tmp_path / "prof")
    tr = yaml.safe_load((d / "training.yaml").read_text())
    tr["checkpoint"]["output_dir"] = str(tmp_path / "ckpt")
    tr["training"]["epochs"] = 2
    tr["runtime"]["verbose"] = False
    tr["context_curriculum"] = {"enabled": True, "stages": [{"max_seq_len": 16, "until_tokens": 200},
                                                            {"max_seq_len": 32, "until_tokens": None}]}
    (d / "training.yaml").write_text(yaml.safe_dump(tr))
    data = build_dataloaders_from_yaml(d / "data.yaml")
    torch.manual_seed(0)
    model = build_model_from_yaml(d / "model.yaml", data_bundle=data)
    res = train_kimi_from_yaml(d / "training.yaml", model=model, data=data)
    cur = res["curriculum"] if "curriculum" in res else None
    ckpts = list_checkpoints(tmp_path / "ckpt")
    assert ckpts
    payload = torch.load(ckpts[-1], weights_only=False)
    state = payload["context_curriculum"]
    assert state is not None and state["stage_index"] == 1 and state["max_seq_len"] == 32
    assert state["transition_count"] >= 1 and state["tokens_seen"] >= 200
    if cur is not None:
        assert cur.current_max_seq_len() == 32
    assert res["state"].optimizer_step > 0
    first = [p for p in ckpts if p.name.endswith("epoch_0000.pt")][0]
    tr["checkpoint"]["resume_from"] = str(first)
    tr["checkpoint"]["output_dir"] = str(tmp_path / "ckpt2")
    (d / "training.yaml").write_text(yaml.safe_dump(tr))
    data2 = build_dataloaders_from_yaml(d / "data.yaml")
    model2 = build_model_from_yaml(d / "model.yaml", data_bundle=data2)
    res2 = train_kimi_from_yaml(d / "training.yaml", model=model2, data=data2)
    again = torch.load(list_checkpoints(tmp_path / "ckpt2")[-1], weights_only=False)["context_curriculum"]
    for key in ("stage_index", "max_seq_len", "tokens_seen"):
        assert again[key] == state[key], key
    assert res2["state"].optimizer_step == res["state"].optimizer_step


def test_single_threaded_resume_is_bit_identical(tmp_path):
    """With one CPU thread (a fixed reduction order) a run resumed from its first epoch's checkpoint
    ends with exactly the weights of the uninterrupted run: model, optimizer, scheduler, RNG and
    sampler state all round-trip."""
    import yaml
    from kimi_k3_b200.config.model_yaml import build_model_from_yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    from kimi_k3_b200.data import build_dataloaders_from_yaml
    from kimi_k3_b200.train.trainer import train_kimi_from_yaml
    threads = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        d = write_pipeline("cpu_smoke", tmp_path / "prof")
        tr = yaml.safe_load((d / "training.yaml").read_text())
        tr["checkpoint"]["output_dir"] = str(tmp_path / "ckpt")
        tr["training"]["epochs"] = 2
        tr["runtime"]["verbose"] = False
        (d / "training.yaml").write_text(yaml.safe_dump(tr))
        data = build_dataloaders_from_yaml(d / "data.yaml")
        torch.manual_seed(0)
        res = train_kimi_from_yaml(d / "training.yaml", model=build_model_from_yaml(d / "model.yaml", data_bundle=data),
                                   data=data)
        tr["checkpoint"]["resume_from"] = str(tmp_path / "ckpt" / "kimi_k3_cpu_smoke_epoch_0000.pt")
        tr["checkpoint"]["output_dir"] = str(tmp_path / "ckpt2")
        (d / "training.yaml").write_text(yaml.safe_dump(tr))
        data2 = build_dataloaders_from_yaml(d / "data.yaml")
        res2 = train_kimi_from_yaml(d / "training.yaml",
                                    model=build_model_from_yaml(d / "model.yaml", data_bundle=data2), data=data2)
    finally:
        torch.set_num_threads(threads)
    for (n, p), (_, q) in zip(res["model"].named_parameters(), res2["model"].named_parameters()):
        assert torch.equal(p, q), n
    for (n, b), (_, c) in zip(res["model"].named_buffers(), res2["model"].named_buffers()):
        assert torch.equal(b, c), n
