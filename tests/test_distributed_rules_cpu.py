"""Distributed runtime rules on CPU: mesh rank arithmetic and axis groups, configuration checks, the
torchrun environment contract, metric reduction, the resumable sampler, size-1 collectives, failure
detection between gloo ranks, and a four-rank TP x EP layout against one process.

Reference behaviour: ``training/distributed/{mesh,config,environment,metrics,sampler,collectives}.py`` and
the four-rank TP x EP smoke of ``tests/training/distributed/test_tp_ep_smoke.py``.
"""
import os
import time

import pytest
import torch

from _dist_harness import run_ranks
from _oracle import needs_reference, ref
from kimi_k3_b200.parallel.collectives import (all_gather_variable, all_ranks_true, all_reduce_max, all_reduce_mean,
                                               all_reduce_sum)
from kimi_k3_b200.parallel.config import distributed_config_from_dict
from kimi_k3_b200.parallel.environment import (axis_rank_lists, coordinates_from_rank, initialize_distributed,
                                               rank_from_coordinates)
from kimi_k3_b200.parallel.metrics import reduce_scalar_metrics, reduction_for
from kimi_k3_b200.parallel.sampler import StatefulDistributedSampler


# --------------------------------------------------------------------------- mesh
@pytest.mark.parametrize("dp,tp,ep", [(1, 1, 1), (2, 1, 1), (1, 2, 2), (2, 2, 2), (4, 2, 1), (1, 1, 8)])
def test_rank_coordinates_round_trip_and_groups_partition_the_world(dp, tp, ep):
    world = dp * tp * ep
    seen = set()
    for r in range(world):
        d, t, e = coordinates_from_rank(r, tp_size=tp, ep_size=ep)
        assert rank_from_coordinates(d, t, e, tp_size=tp, ep_size=ep) == r
        seen.add((d, t, e))
    assert len(seen) == world
    for axis, size in zip(axis_rank_lists(dp, tp, ep), (dp, tp, ep)):
        assert sorted(r for g in axis for r in g) == list(range(world))
        assert all(len(g) == size for g in axis)
    # a rank's TP peers share its DP and EP coordinates
    _, tp_groups, _ = axis_rank_lists(dp, tp, ep)
    for g in tp_groups:
        coords = [coordinates_from_rank(r, tp_size=tp, ep_size=ep) for r in g]
        assert len({(c[0], c[2]) for c in coords}) == 1


def test_expert_parallel_overlaid_on_tensor_parallel_shares_the_tp_groups():
    dp_groups, tp_groups, ep_groups = axis_rank_lists(2, 4, 4, overlay=True)
    assert tp_groups == ep_groups == [[0, 1, 2, 3], [4, 5, 6, 7]]
    assert dp_groups == [[0, 4], [1, 5], [2, 6], [3, 7]]


@needs_reference
@pytest.mark.reference
@pytest.mark.parametrize("dp,tp,ep", [(2, 2, 2), (1, 4, 2), (3, 1, 2)])
def test_axis_groups_match_reference(dp, tp, ep):
    ref()
    from training.distributed.mesh import _all_axis_groups
    assert tuple(axis_rank_lists(dp, tp, ep)) == tuple(_all_axis_groups(dp, tp, ep))


# --------------------------------------------------------------------------- configuration
@pytest.mark.parametrize("bad", [
    {"data_parallel": {"mode": "zero3", "size": 2}},
    {"data_parallel": {"size": 0}},
    {"tensor_parallel": {"enabled": True, "size": 0}},
    {"expert_parallel": {"enabled": True, "size": -2}},
    {"pipeline_parallel": {"enabled": True, "size": 2}},
    {"context_parallel": {"enabled": True, "size": 2}},
    {"backend": "mpi"},
    {"timeout_seconds": 0},
    {"not_a_section": {}},
])
def test_distributed_config_rejects_invalid_values(bad):
    with pytest.raises((ValueError, TypeError)):
        distributed_config_from_dict({"enabled": True, **bad})


def test_logical_world_size_and_overlay():
    c = distributed_config_from_dict({"enabled": True, "data_parallel": {"mode": "ddp", "size": 2},
                                      "tensor_parallel": {"enabled": True, "size": 4},
                                      "expert_parallel": {"enabled": True, "size": 2}})
    assert c.logical_world_size == 16
    o = distributed_config_from_dict({"enabled": True, "tensor_parallel": {"enabled": True, "size": 8},
                                      "expert_parallel": {"enabled": True, "size": 8,
                                                          "overlay_tensor_parallel": True}})
    assert o.logical_world_size == 8
    assert distributed_config_from_dict(None).logical_world_size == 1


def test_environment_contract_is_checked_before_any_process_group():
    disabled = distributed_config_from_dict({"enabled": False})
    with pytest.raises(RuntimeError):
        initialize_distributed(disabled, environment={"WORLD_SIZE": "2", "RANK": "0", "LOCAL_RANK": "0"})
    ctx = initialize_distributed(disabled, environment={"WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"})
    assert not ctx.initialized and ctx.world_size == 1
    two = distributed_config_from_dict({"enabled": True, "backend": "gloo", "data_parallel": {"mode": "ddp",
                                                                                             "size": 2}})
    with pytest.raises(RuntimeError):
        initialize_distributed(two, environment={"WORLD_SIZE": "4", "RANK": "0", "LOCAL_RANK": "0"})


# --------------------------------------------------------------------------- metrics, collectives, sampler
@pytest.mark.parametrize("name,kind", [("train/loss", "mean"), ("memory/peak_gb", "max"), ("grad/max_norm", "max"),
                                       ("kda/alpha_min", "min"), ("throughput/tokens", "mean")])
def test_metric_reduction_rule(name, kind):
    assert reduction_for(name) == kind


def test_size_one_helpers_are_identities_without_a_process_group():
    t = torch.tensor([1.0, -2.0])
    assert torch.equal(all_reduce_sum(t.clone()), t) and torch.equal(all_reduce_mean(t.clone()), t)
    assert torch.equal(all_reduce_max(t.clone()), t)
    assert all_ranks_true(True) and not all_ranks_true(False)
    assert torch.equal(all_gather_variable(t), t)
    assert reduce_scalar_metrics({"a": 1.0}) == {"a": 1.0}


@pytest.mark.parametrize("n,replicas,drop_last", [(10, 3, False), (10, 3, True), (8, 4, False), (5, 8, False)])
def test_sampler_shards_cover_the_dataset(n, replicas, drop_last):
    data = list(range(n))
    shards = [list(StatefulDistributedSampler(data, replicas, r, shuffle=True, seed=3, drop_last=drop_last))
              for r in range(replicas)]
    sizes = {len(s) for s in shards}
    assert len(sizes) == 1
    flat = [i for s in shards for i in s]
    if drop_last:
        assert len(set(flat)) == len(flat) == (n // replicas) * replicas
    else:
        assert set(flat) == set(data)


def test_sampler_resumes_mid_epoch_and_reshuffles_per_epoch():
    data = list(range(20))
    s = StatefulDistributedSampler(data, 2, 1, seed=5)
    it = iter(s)
    first = [next(it) for _ in range(4)]
    state = s.state_dict()
    resumed = StatefulDistributedSampler(data, 2, 1, seed=5)
    resumed.load_state_dict(state)
    assert first + list(resumed) == list(StatefulDistributedSampler(data, 2, 1, seed=5))
    assert len(resumed) == 0
    e0 = list(StatefulDistributedSampler(data, 2, 1, seed=5))
    s1 = StatefulDistributedSampler(data, 2, 1, seed=5)
    s1.set_epoch(1)
    assert list(s1) != e0
    with pytest.raises(ValueError):
        StatefulDistributedSampler(data, 4, 1, seed=5).load_state_dict(state)
    with pytest.raises(ValueError):
        StatefulDistributedSampler(data, 2, 2)


# --------------------------------------------------------------------------- multi-process
def _metrics_rank(rank, world):
    from kimi_k3_b200.parallel.environment import setup_distributed
    ctx = setup_distributed(distributed_config_from_dict({"enabled": True, "backend": "gloo",
                                                          "data_parallel": {"mode": "ddp", "size": world}}))
    out = reduce_scalar_metrics({"train/loss": float(rank + 1), "memory/peak_gb": float(10 * rank),
                                 "kda/alpha_min": float(rank - 5), "label": "x"}, context=ctx)
    ragged = all_gather_variable(torch.arange(rank + 1, dtype=torch.float32), group=None)
    ctx.close()
    return out, ragged


def _uneven_metrics_rank(rank, world):
    from kimi_k3_b200.parallel.environment import setup_distributed
    ctx = setup_distributed(distributed_config_from_dict({"enabled": True, "backend": "gloo",
                                                          "data_parallel": {"mode": "ddp", "size": world}}))
    mine = {"train/loss": float(rank + 1)}
    if rank == 1:   # optional metrics that only this rank logged
        mine.update({"diag/rms": 4.0, "memory/peak_gb": 7.0, "kda/alpha_min": -1.0})
    out = reduce_scalar_metrics(mine, context=ctx)
    ctx.close()
    return out


def test_metric_reduction_tolerates_ranks_that_log_different_metrics():
    for out in run_ranks(_uneven_metrics_rank, 2):
        assert out["train/loss"] == pytest.approx(1.5)
        assert out["diag/rms"] == 4.0 and out["memory/peak_gb"] == 7.0 and out["kda/alpha_min"] == -1.0


def test_metrics_and_ragged_gather_over_gloo_ranks():
    res = run_ranks(_metrics_rank, 3)
    for out, ragged in res:
        assert out["train/loss"] == pytest.approx(2.0) and out["memory/peak_gb"] == 20.0
        assert out["kda/alpha_min"] == -5.0 and out["label"] == "x"
        assert ragged.tolist() == [0.0, 0.0, 1.0, 0.0, 1.0, 2.0]


def _failing_rank(rank, world, marker):
    from kimi_k3_b200.parallel.environment import setup_distributed
    ctx = setup_distributed(distributed_config_from_dict({"enabled": True, "backend": "gloo", "timeout_seconds": 20,
                                                          "data_parallel": {"mode": "ddp", "size": world}}))
    t = torch.ones(1)
    torch.distributed.all_reduce(t)               # both ranks reach the first collective
    if rank == 1:
        os._exit(3)                               # this rank dies between steps
    start = time.monotonic()
    try:
        torch.distributed.all_reduce(t)           # the survivor learns of it from its next collective
        outcome = "completed"
    except Exception as exc:                       # noqa: BLE001 - any transport error is the signal
        outcome = type(exc).__name__
    with open(marker, "w") as f:
        f.write(f"{outcome} {time.monotonic() - start:.1f}")
    os._exit(0)


def test_a_dead_rank_surfaces_as_an_error_on_the_survivor(tmp_path):
    import torch.multiprocessing as mp
    from _dist_harness import _entry, free_port
    marker = str(tmp_path / "survivor.txt")
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=_entry, args=(r, 2, port, _failing_rank, str(tmp_path), (marker,)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
        if p.is_alive():
            p.kill()
    assert procs[1].exitcode == 3
    outcome, seconds = open(marker).read().split()
    assert outcome != "completed" and float(seconds) < 60.0


def _tp_ep_rank(rank, world, kind):
    from test_distributed_cpu import _global_batch, _model, _train
    from kimi_k3_b200.parallel.environment import setup_distributed
    from kimi_k3_b200.parallel.parallelize import parallelize_kimi_model
    dcfg = distributed_config_from_dict({"enabled": True, "backend": "gloo", "timeout_seconds": 120,
                                         "tensor_parallel": {"enabled": True, "size": 2},
                                         "expert_parallel": {"enabled": True, "size": 2}})
    ctx = setup_distributed(dcfg)
    model = _model()
    plan = parallelize_kimi_model(model, dcfg, ctx)
    plan.broadcast_parameters()
    full = _global_batch(2)                         # two data replicas (the EP ranks) of two rows each
    batch = {k: v[2 * ctx.ep_rank: 2 * ctx.ep_rank + 2] for k, v in full.items()}
    res = _train(model, batch, kind, context=ctx, plan=plan, steps=2)
    shared = {n: p.detach().clone() for n, p in model.named_parameters()
              if not getattr(p, "_kimi_tp_shard", False) and not getattr(p, "_kimi_local_expert", False)}
    ctx.close()
    return res["loss"], shared, (ctx.tp_rank, ctx.ep_rank)


@pytest.mark.slow
def test_four_rank_tp_ep_layout_matches_single_process():
    from test_distributed_cpu import _compare, _single
    ref_loss, ref_params = _single(2, "adamw")
    results = run_ranks(_tp_ep_rank, 4, "adamw")
    assert sorted(r[2] for r in results) == [(0, 0), (0, 1), (1, 0), (1, 1)]
    for loss, params, _ in results:
        assert abs(loss - ref_loss) < 1e-6
        assert _compare(ref_params, params, 1e-7) < 1e-7


def _fsdp_ckpt_rank(rank, world, path):
    from test_distributed_cpu import _global_batch, _model, _train
    from kimi_k3_b200.parallel.checkpoint import (export_rank0_full_checkpoint, load_distributed_checkpoint,
                                                  save_distributed_checkpoint)
    from kimi_k3_b200.parallel.environment import setup_distributed
    from kimi_k3_b200.parallel.fsdp import shard_kimi_model
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    dcfg = distributed_config_from_dict({"enabled": True, "backend": "gloo", "timeout_seconds": 120,
                                         "data_parallel": {"mode": "fsdp", "size": world}})
    ctx = setup_distributed(dcfg)
    full = _global_batch(world)
    batch = {k: v[2 * rank: 2 * rank + 2] for k, v in full.items()}

    def build():
        m = _model()
        shard_kimi_model(m, dcfg, ctx)
        m._test_params = [p for p in m.parameters() if p.requires_grad]   # the shards, as the trainer keeps
        opt, _ = build_kimi_optimizer(m, KimiOptimizerConfig(kind="adamw", adamw_lr=1e-3, adamw_eps=1e-2))
        return m, opt

    def step(m, opt):
        from kimi_k3_b200.train.loop import train_one_epoch
        from kimi_k3_b200.parallel.fsdp import sharded_grad_norm
        train_one_epoch(m, [batch], opt, grad_clip=0.5, use_mtp=True, distributed_context=ctx,
                        grad_norm_fn=lambda: sharded_grad_norm(m._test_params))

    a, oa = build()
    step(a, oa)                                            # optimizer state exists before the save
    a.eval()
    with torch.no_grad():
        ref = a(input_ids=full["input_ids"][:2], attention_mask=full["attention_mask"][:2]).logits
    a.train()
    save_distributed_checkpoint(os.path.join(path, "step_1"), model=a, context=ctx, step=1, optimizer=oa)
    export_rank0_full_checkpoint(os.path.join(path, "full.pt"), model=a, context=ctx)
    b, ob = build()
    load_distributed_checkpoint(os.path.join(path, "step_1"), model=b, context=ctx, optimizer=ob)
    b.eval()
    with torch.no_grad():
        got = b(input_ids=full["input_ids"][:2], attention_mask=full["attention_mask"][:2]).logits
    b.train()
    step(a, oa)                                            # one more step on both: same parameters
    step(b, ob)
    worst = max((pa.full_tensor() - pb.full_tensor()).abs().max().item()
                for pa, pb in zip(a.parameters(), b.parameters()))
    ctx.close()
    return (ref - got).abs().max().item(), worst, ref


def test_fully_sharded_checkpoint_round_trip_and_full_export(tmp_path):
    from test_distributed_cpu import _model
    from kimi_k3_b200.train.checkpoints import load_checkpoint
    res = run_ranks(_fsdp_ckpt_rank, 2, str(tmp_path))
    for logits_diff, param_diff, _ in res:
        assert logits_diff == 0.0 and param_diff == 0.0
    single = _model()
    info = load_checkpoint(tmp_path / "full.pt", single)
    assert not info["missing_keys"] and not info["unexpected_keys"]
    single.eval()
    from test_distributed_cpu import _global_batch
    b = _global_batch(2)
    with torch.no_grad():
        out = single(input_ids=b["input_ids"][:2], attention_mask=b["attention_mask"][:2]).logits
    assert (out - res[0][2]).abs().max().item() < 1e-12


def test_expert_parallel_with_histogram_balancing_matches_single_process():
    """EP reduces the Quantile-Balancing histograms over the expert group (one all-reduce of the
    counts); the routing biases and parameters then follow the single-process run."""
    from test_distributed_cpu import _compare, _rank, _single
    ref_loss, ref_params = _single(2, "adamw", qb="histogram")
    results = run_ranks(_rank, 2, "ep", "adamw", "histogram")
    for loss, params, _ in results:
        assert abs(loss - ref_loss) < 1e-6
        assert _compare(ref_params, params, 1e-7) < 1e-7


def _dp_accum_rank(rank, world, micro):
    from test_distributed_cpu import _model
    from kimi_k3_b200.parallel.environment import setup_distributed
    from kimi_k3_b200.parallel.parallelize import parallelize_kimi_model
    from kimi_k3_b200.train.engine import MoEController
    from kimi_k3_b200.train.loop import train_one_epoch
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    dcfg = distributed_config_from_dict({"enabled": True, "backend": "gloo", "timeout_seconds": 120,
                                         "data_parallel": {"mode": "ddp", "size": world}})
    ctx = setup_distributed(dcfg)
    model = _model()
    plan = parallelize_kimi_model(model, dcfg, ctx)
    plan.broadcast_parameters()
    opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(kind="adamw", adamw_lr=1e-3, adamw_eps=1e-2))
    mine = micro[rank::world]
    res = train_one_epoch(model, mine, opt, grad_accum_steps=len(mine), grad_clip=0.5, use_mtp=True,
                          moe_controller=MoEController(model, reducer=plan.qb_reducer()), distributed_context=ctx,
                          grad_reducer=plan.sync_gradients, grad_norm_fn=plan.grad_norm)
    out = {n: p.detach().clone() for n, p in model.named_parameters()}
    ctx.close()
    return res["loss"], out


def _uneven_micro_batches(n=4):
    g = torch.Generator().manual_seed(11)
    out = []
    for i in range(n):
        ids = torch.randint(5, 128, (2, 16), generator=g)
        mask = torch.ones(2, 16, dtype=torch.bool)
        mask[1, 4 + 3 * i:] = False                     # each micro-batch has a different token count
        out.append({"input_ids": ids, "labels": ids.clone(), "attention_mask": mask})
    return out


def test_data_parallel_accumulation_windows_are_token_exact():
    from test_distributed_cpu import _compare, _model
    from kimi_k3_b200.train.engine import MoEController
    from kimi_k3_b200.train.loop import train_one_epoch
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    micro = _uneven_micro_batches(4)
    single = _model()
    opt, _ = build_kimi_optimizer(single, KimiOptimizerConfig(kind="adamw", adamw_lr=1e-3, adamw_eps=1e-2))
    ref_res = train_one_epoch(single, micro, opt, grad_accum_steps=4, grad_clip=0.5, use_mtp=True,
                              moe_controller=MoEController(single))
    ref_params = {n: p.detach().clone() for n, p in single.named_parameters()}
    for loss, params in run_ranks(_dp_accum_rank, 2, micro):
        assert abs(loss - ref_res["loss"]) < 1e-6
        assert _compare(ref_params, params, 1e-7) < 1e-7


def _fsdp_trainer_rank(rank, world, root, resume, overrides=None):
    import yaml
    from pathlib import Path
    from kimi_k3_b200.config.model_yaml import build_model_from_yaml
    from kimi_k3_b200.data import build_dataloaders_from_yaml
    from kimi_k3_b200.parallel.config import distributed_config_from_dict
    from kimi_k3_b200.parallel.environment import setup_distributed
    from kimi_k3_b200.train.trainer import train_kimi_from_yaml
    d = Path(root) / "prof"
    tr = yaml.safe_load((d / "training.yaml").read_text())
    for section, values in (overrides or {}).items():
        tr[section] = {**tr.get(section, {}), **values} if isinstance(values, dict) else values
    tr["checkpoint"]["output_dir"] = str(Path(root) / ("resumed" if resume else "ckpt"))
    if resume:
        tr["checkpoint"]["resume_from"] = str(Path(root) / "ckpt" / "kimi_k3_cpu_smoke_epoch_0000")
    path = d / f"training_{rank}_{int(resume)}.yaml"
    path.write_text(yaml.safe_dump(tr))
    ctx = setup_distributed(distributed_config_from_dict(tr["distributed"]))
    data = build_dataloaders_from_yaml(d / "data.yaml", distributed_context=ctx)
    torch.manual_seed(0)
    model = build_model_from_yaml(d / "model.yaml", data_bundle=data)
    res = train_kimi_from_yaml(path, model=model, data=data, distributed_context=ctx)
    from kimi_k3_b200.parallel.checkpoint import full_state_dict
    full = {k: v.clone() for k, v in full_state_dict(res["model"], ctx).items()}
    steps = res["state"].optimizer_step
    ctx.close()
    return steps, full


YAML_LAYOUTS = {
    "fsdp": {"data_parallel": {"mode": "fsdp", "size": 2}},
    "ddp": {"data_parallel": {"mode": "ddp", "size": 2}},
    "tp": {"tensor_parallel": {"enabled": True, "size": 2}},
    "ep": {"expert_parallel": {"enabled": True, "size": 2}},
    "tp_ep_overlay": {"tensor_parallel": {"enabled": True, "size": 2},
                      "expert_parallel": {"enabled": True, "size": 2, "overlay_tensor_parallel": True}},
}


@pytest.mark.slow
@pytest.mark.parametrize("layout", sorted(YAML_LAYOUTS))
def test_distributed_yaml_trainer_checkpoints_every_epoch_and_resumes(tmp_path, layout):
    """The YAML trainer on two gloo ranks for every parallel layout: diagnostics, an evaluation pass and a
    distributed checkpoint after each epoch, then a run resumed from the first epoch's checkpoint ends
    with the weights of the uninterrupted run."""
    import yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    d = write_pipeline("cpu_smoke", tmp_path / "prof")
    tr = yaml.safe_load((d / "training.yaml").read_text())
    tr["training"]["epochs"] = 2
    tr["training"]["max_batches_per_epoch"] = 1
    tr["runtime"]["verbose"] = False
    tr["diagnostics"]["standard_every_steps"] = 1   # every diagnostics tier runs (ranks may degrade apart)
    tr["diagnostics"]["deep_every_steps"] = 2
    tr["distributed"] = {"enabled": True, "backend": "gloo", "timeout_seconds": 120, **YAML_LAYOUTS[layout]}
    (d / "training.yaml").write_text(yaml.safe_dump(tr))
    first = run_ranks(_fsdp_trainer_rank, 2, str(tmp_path), False)
    assert (tmp_path / "ckpt" / "kimi_k3_cpu_smoke_epoch_0001" / "SUCCESS").is_file()
    assert (tmp_path / "ckpt" / "kimi_k3_cpu_smoke_epoch_0000" / "rank_00001.pt").is_file()
    again = run_ranks(_fsdp_trainer_rank, 2, str(tmp_path), True)
    assert first[0][0] == again[0][0] == 2
    for k, v in first[0][1].items():
        torch.testing.assert_close(again[0][1][k], v, rtol=1e-5, atol=1e-6, msg=k)


@pytest.mark.slow
def test_data_parallel_trainer_with_curriculum_ema_and_accumulation_resumes(tmp_path):
    """DDP over two gloo ranks with a two-stage context curriculum (loader rebuilt on the transition
    with its distributed sampler), EMA and two-micro-batch windows: checkpoints and resumes."""
    import yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    d = write_pipeline("cpu_smoke", tmp_path / "prof")
    tr = yaml.safe_load((d / "training.yaml").read_text())
    tr["training"]["epochs"] = 2
    tr["training"]["gradient_accumulation_steps"] = 2
    tr["runtime"]["verbose"] = False
    tr["runtime"]["use_ema"] = True
    tr["context_curriculum"] = {"enabled": True, "stages": [{"max_seq_len": 16, "until_tokens": 300},
                                                            {"max_seq_len": 32, "until_tokens": None}]}
    tr["distributed"] = {"enabled": True, "backend": "gloo", "timeout_seconds": 120,
                         "data_parallel": {"mode": "ddp", "size": 2}}
    (d / "training.yaml").write_text(yaml.safe_dump(tr))
    first = run_ranks(_fsdp_trainer_rank, 2, str(tmp_path), False)
    again = run_ranks(_fsdp_trainer_rank, 2, str(tmp_path), True)
    assert first[0][0] == again[0][0] > 0
    for k, v in first[0][1].items():
        torch.testing.assert_close(again[0][1][k], v, rtol=1e-5, atol=1e-6, msg=k)


def _budget_rank(rank, world):
    from test_distributed_cpu import _model
    from kimi_k3_b200.parallel.environment import setup_distributed
    from kimi_k3_b200.train.diagnostics import DiagnosticsConfig, KimiDiagnosticCollector
    from kimi_k3_b200.train.loop import train_one_epoch
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    ctx = setup_distributed(distributed_config_from_dict({"enabled": True, "backend": "gloo",
                                                          "data_parallel": {"mode": "ddp", "size": world}}))
    model = _model()
    opt, registry = build_kimi_optimizer(model, KimiOptimizerConfig(kind="adamw"))
    # only rank 0 has a budget it is sure to exceed
    cfg = DiagnosticsConfig(standard_every_steps=1, deep_every_steps=4,
                            max_diagnostic_time_fraction=1e-9 if rank == 0 else 1.0)
    collector = KimiDiagnosticCollector(model, cfg, parameter_specs=registry.specs)
    collector.budget_device = ctx.device
    ids = torch.randint(5, 128, (2, 12), generator=torch.Generator().manual_seed(rank))
    batch = {"input_ids": ids, "labels": ids.clone(), "attention_mask": torch.ones(2, 12, dtype=torch.bool)}
    train_one_epoch(model, [batch], opt, use_mtp=True, diagnostics=collector, distributed_context=ctx)
    ctx.close()
    return collector.degrade_until_step, [collector.level_for_step(s) for s in range(2, 5)]


def test_diagnostics_degrade_on_the_same_steps_on_every_rank():
    a, b = run_ranks(_budget_rank, 2)
    assert a == b and a[0] > 0 and a[1][0] == "cheap"


@pytest.mark.slow
def test_tp_ep_overlay_trainer_with_bf16_accumulation_curriculum_and_all_diagnostics(tmp_path):
    """The most composed layout (EP on the TP ranks) under bf16 autocast, two-micro-batch windows, a
    two-stage context curriculum and every diagnostics tier trains through the YAML trainer."""
    import yaml
    from kimi_k3_b200.config.profiles import write_pipeline
    d = write_pipeline("cpu_smoke", tmp_path / "prof")
    tr = yaml.safe_load((d / "training.yaml").read_text())
    tr["training"].update(epochs=1, max_batches_per_epoch=4, gradient_accumulation_steps=2, precision="bf16")
    tr["runtime"]["verbose"] = False
    tr["diagnostics"].update(standard_every_steps=1, deep_every_steps=2)
    tr["context_curriculum"] = {"enabled": True, "stages": [{"max_seq_len": 16, "until_tokens": 200},
                                                            {"max_seq_len": 32, "until_tokens": None}]}
    tr["distributed"] = {"enabled": True, "backend": "gloo", "timeout_seconds": 120,
                         **YAML_LAYOUTS["tp_ep_overlay"]}
    (d / "training.yaml").write_text(yaml.safe_dump(tr))
    res = run_ranks(_fsdp_trainer_rank, 2, str(tmp_path), False)
    assert res[0][0] == res[1][0] == 2
    for k, v in res[0][1].items():
        assert torch.isfinite(v).all(), k
        assert torch.equal(v, res[1][1][k]), k      # both ranks export the same full weights
