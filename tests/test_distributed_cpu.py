"""Multi-process CPU (gloo) tests of the distributed runtime against single-process runs.

Each parallel layout trains one optimizer step on a global batch split over ranks and must
land on the same parameters as one process training on the whole batch (float64).
"""
import dataclasses

import pytest
import torch

from _dist_harness import run_ranks

CFG_KW = dict(enable_vision=False)


def _global_batch(world):
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(5, 128, (2 * world, 24), generator=g)
    mask = torch.ones_like(ids, dtype=torch.bool)
    mask[1, 17:] = False
    return {"input_ids": ids, "labels": ids.clone(), "attention_mask": mask}


def _model(qb="exact"):
    from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
    cfg = kimi_k3_cpu_tiny_config(**CFG_KW)
    moe = dataclasses.replace(cfg.backbone.stable_latent_moe_config, quantile_backend=qb)
    cfg = dataclasses.replace(cfg, backbone=dataclasses.replace(cfg.backbone, stable_latent_moe_config=moe),
                              mtp=dataclasses.replace(cfg.mtp, stable_latent_moe_config=moe))
    torch.manual_seed(0)
    return KimiK3(cfg).double()


def _train(model, batch, kind, *, context=None, plan=None, steps=1, zero=False):
    from kimi_k3_b200.train.engine import MoEController
    from kimi_k3_b200.train.loop import train_one_epoch
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    # a large AdamW epsilon keeps the update linear in tiny gradients, whose float32 rounding
    # (the vocabulary-parallel logits) would otherwise be amplified to full-size updates
    opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(kind=kind, adamw_lr=1e-3, muon_lr=1e-2, adamw_eps=1e-2))
    if zero:  # fully sharded: gradients were reduce-scattered in backward
        from kimi_k3_b200.parallel.data_parallel import QBReducer
        from kimi_k3_b200.parallel.fsdp import sharded_grad_norm
        params = [p for p in model.parameters() if p.requires_grad]
        ctl = MoEController(model, reducer=QBReducer(context.dp_group))
        if getattr(opt, "qk_clip", None) is not None:
            opt.qk_clip.replica_group = context.dp_group
        sync, norm = None, (lambda: sharded_grad_norm(params))
    else:
        ctl = MoEController(model, reducer=None if plan is None else plan.qb_reducer())
        sync = None if plan is None else plan.sync_gradients
        norm = None if plan is None else plan.grad_norm
    res = None
    for _ in range(steps):
        res = train_one_epoch(model, [batch], opt, grad_clip=0.5, use_mtp=True, moe_controller=ctl,
                              distributed_context=context, grad_reducer=sync, grad_norm_fn=norm)
    return res


def _single(world, kind, qb="exact"):
    m = _model(qb)
    res = _train(m, _global_batch(world), kind, steps=2)
    return res["loss"], {n: p.detach().clone() for n, p in m.named_parameters()}


def _rank(rank, world, layout, kind, qb):
    from kimi_k3_b200.parallel.config import distributed_config_from_dict
    from kimi_k3_b200.parallel.environment import setup_distributed
    from kimi_k3_b200.parallel.parallelize import parallelize_kimi_model
    cfg = {"enabled": True, "backend": "gloo", "timeout_seconds": 120}
    if layout == "dp":
        cfg["data_parallel"] = {"mode": "ddp", "size": world}
    elif layout == "fsdp":
        cfg["data_parallel"] = {"mode": "fsdp", "size": world}
    elif layout == "tp":
        cfg["tensor_parallel"] = {"enabled": True, "size": world}
    elif layout == "tp_fused_output":  # the fused output projection (CPU ranks take its all-reduce path)
        cfg["tensor_parallel"] = {"enabled": True, "size": world, "fused_output_reduce": True}
    elif layout == "ep":
        cfg["expert_parallel"] = {"enabled": True, "size": world}
    elif layout == "tp_ep_overlay":
        cfg["tensor_parallel"] = {"enabled": True, "size": world}
        cfg["expert_parallel"] = {"enabled": True, "size": world, "overlay_tensor_parallel": True}
    dcfg = distributed_config_from_dict(cfg)
    ctx = setup_distributed(dcfg)
    model = _model(qb)
    plan = None
    shard_bytes = None
    if layout != "fsdp":
        plan = parallelize_kimi_model(model, dcfg, ctx)
        plan.broadcast_parameters()
    else:
        from kimi_k3_b200.parallel.fsdp import local_shard_bytes, shard_kimi_model
        full_bytes = sum(p.numel() * p.element_size() for p in model.parameters())
        shard_kimi_model(model, dcfg, ctx)
        shard_bytes = local_shard_bytes(model) / full_bytes
    full = _global_batch(world)
    data_replicas = world if layout in ("dp", "ep", "fsdp") else 1
    if data_replicas > 1:
        batch = {k: v[2 * ctx.global_rank: 2 * ctx.global_rank + 2] for k, v in full.items()}
    else:
        batch = full
    res = _train(model, batch, kind, context=ctx, plan=plan, steps=2, zero=layout == "fsdp")
    out = {n: (p.full_tensor() if hasattr(p, "full_tensor") else p).detach().clone()
           for n, p in model.named_parameters()
           if not getattr(p, "_kimi_tp_shard", False) and not getattr(p, "_kimi_local_expert", False)}
    if shard_bytes is not None:
        out["__shard_fraction__"] = torch.tensor(shard_bytes)
    experts = {n: p.detach().clone() for n, p in model.named_parameters() if getattr(p, "_kimi_local_expert", False)}
    # tensor-parallel shards with the dimension they split (compared against slices of the full matrices)
    shards = {n: (p._kimi_tp_dim, ctx.tp_rank, p.detach().clone()) for n, p in model.named_parameters()
              if getattr(p, "_kimi_tp_dim", None) is not None}
    experts["__tp_shards__"] = shards
    ctx.close()
    return res["loss"], out, experts


def _compare(ref_params, got, tol):
    worst = 0.0
    for n, v in got.items():
        key = n.replace(".inner.", ".")
        if key in ref_params and ref_params[key].shape == v.shape:
            worst = max(worst, (ref_params[key] - v).abs().max().item())
    return worst


@pytest.mark.parametrize("layout,kind", [("dp", "per_head_muon_adamw"), ("tp", "adamw"), ("tp", "per_head_muon_adamw"),
                                         ("tp_fused_output", "adamw"),
                                         ("ep", "per_head_muon_adamw"),
                                         ("tp_ep_overlay", "adamw"), ("fsdp", "per_head_muon_adamw")])
def test_parallel_layout_matches_single_process(layout, kind):
    world = 2
    # Muon's Newton-Schulz runs in float32: float64 summation-order differences between the
    # layouts surface at float32 rounding after the first update.
    tol = 1e-7 if kind == "adamw" else 2e-6
    ref_loss, ref_params = _single(world, kind)
    results = run_ranks(_rank, world, layout, kind, "exact")
    for loss, params, experts in results:
        # the single-process CPU loss is reduced in float32 (its logits are float32)
        assert abs(loss - ref_loss) < max(tol, 1e-6), (layout, loss, ref_loss)
        if layout == "fsdp":  # each rank holds about 1/world of the parameters
            frac = float(params.pop("__shard_fraction__"))
            assert frac < 0.6, frac
        assert _compare(ref_params, params, tol) < tol, layout
    for _, _, experts in results:
        # every tensor-parallel shard equals its slice of the single-process matrix (Muon orthogonalises
        # the gathered whole matrix, so sharded and unsharded runs take the same step)
        for n, (dim, tp_rank, v) in experts.pop("__tp_shards__").items():
            full = ref_params[n.replace(".inner.", ".")]
            want = full.chunk(world, dim)[tp_rank]
            assert (want - v).abs().max().item() < tol, (layout, n)
    if layout in ("ep", "tp_ep_overlay"):
        # each rank's local experts equal the matching slice of the single-process experts
        for rank, (_, _, experts) in enumerate(results):
            for n, v in experts.items():
                per = v.shape[0]
                assert (ref_params[n][rank * per:(rank + 1) * per] - v).abs().max().item() < tol, n


def _ckpt_rank(rank, world, path):
    import os
    from kimi_k3_b200.parallel.checkpoint import (export_rank0_full_checkpoint, load_distributed_checkpoint,
                                                  save_distributed_checkpoint)
    from kimi_k3_b200.parallel.config import distributed_config_from_dict
    from kimi_k3_b200.parallel.environment import setup_distributed
    from kimi_k3_b200.parallel.parallelize import parallelize_kimi_model
    dcfg = distributed_config_from_dict({"enabled": True, "backend": "gloo",
                                         "tensor_parallel": {"enabled": True, "size": world},
                                         "expert_parallel": {"enabled": True, "size": world,
                                                             "overlay_tensor_parallel": True}})
    ctx = setup_distributed(dcfg)
    b = _global_batch(world)
    m = _model()
    parallelize_kimi_model(m, dcfg, ctx)
    with torch.no_grad():
        for p in m.parameters():  # make the state differ from the seeded init
            p.add_(0.01 * torch.randn_like(p))
    m.eval()
    ref = m(input_ids=b["input_ids"], attention_mask=b["attention_mask"]).logits
    save_distributed_checkpoint(os.path.join(path, "step_1"), model=m, context=ctx, step=1)
    m2 = _model()
    parallelize_kimi_model(m2, dcfg, ctx)
    load_distributed_checkpoint(os.path.join(path, "step_1"), model=m2, context=ctx)
    m2.eval()
    got = m2(input_ids=b["input_ids"], attention_mask=b["attention_mask"]).logits
    export_rank0_full_checkpoint(os.path.join(path, "full.pt"), model=m, context=ctx)
    ctx.close()
    return (ref - got).abs().max().item(), ref


def test_distributed_checkpoint_roundtrip_and_full_export(tmp_path):
    from kimi_k3_b200.train.checkpoints import load_checkpoint
    res = run_ranks(_ckpt_rank, 2, str(tmp_path))
    assert all(r[0] == 0.0 for r in res)
    assert (tmp_path / "step_1" / "SUCCESS").is_file() and (tmp_path / "step_1" / "rank_00001.pt").is_file()
    single = _model()
    info = load_checkpoint(tmp_path / "full.pt", single)
    assert not info["missing_keys"] and not info["unexpected_keys"]
    single.eval()
    b = _global_batch(2)
    logits = single(input_ids=b["input_ids"], attention_mask=b["attention_mask"]).logits
    assert (logits - res[0][1]).abs().max().item() < 1e-6  # the export reassembles the sharded model
