"""Two-GPU runs of the sharded training and inference paths (NCCL, one process per GPU).

* fully sharded data parallelism: a few bf16 training steps of the tiny model, each rank holding
  half of every parameter, against the same steps with plain data parallelism (bucketed
  all-reduce) from the same initial weights;
* tensor-parallel and expert-parallel decode: the serving decoder's captured decode step (CUDA
  graph with NCCL collectives, or the device-initiated expert exchange) against eager cached
  generation on the same ranks.

Each case runs under torchrun on 127.0.0.1 with a hard timeout, NVLS off.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HERE = os.path.abspath(__file__)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _torchrun(mode: str, timeout: int = 300) -> str:
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""), NCCL_NVLS_ENABLE="0")
    args = ["timeout", "-k", "30", str(timeout - 30), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
            "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}", HERE, mode]
    r = subprocess.run(args, env=env, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    return r.stdout


def test_fsdp_training_two_gpus():
    assert "fsdp ok" in _torchrun("fsdp")


def test_sharded_graph_decode_two_gpus():
    assert "decode ok" in _torchrun("decode")


# ----------------------------------------------------------------------------- rank side
def _tiny(seed=0):
    """A small model whose shapes take the CUDA kernels (head dims 64, MoE latent 64)."""
    from kimi_k3_b200.config.model_yaml import build_model_config_from_mapping
    from kimi_k3_b200.config.profiles import profile_model_mapping
    from kimi_k3_b200.models import KimiK3
    m = profile_model_mapping("t4_wikitext")
    m["model"].update(d_model=128, num_heads=2, num_hybrid_groups=1, vocab_size=1000)
    m["model"]["moe"].update(latent_dim=64, shared_expert_hidden_dim=96, routed_expert_hidden_dim=128)
    m["model"]["mla"]["kv_latent_dim"] = 128
    torch.manual_seed(seed)
    return KimiK3(build_model_config_from_mapping(m))


def _dist(cfg):
    from kimi_k3_b200.parallel.config import distributed_config_from_dict
    from kimi_k3_b200.parallel.environment import setup_distributed
    base = {"enabled": True, "backend": "nccl", "timeout_seconds": 60}
    base.update(cfg)
    dcfg = distributed_config_from_dict(base)
    return dcfg, setup_distributed(dcfg)


def _fsdp_rank():
    import torch.distributed as dist
    from kimi_k3_b200.parallel.fsdp import local_shard_bytes, shard_kimi_model, sharded_grad_norm
    from kimi_k3_b200.parallel.parallelize import parallelize_kimi_model
    from kimi_k3_b200.train.engine import MoEController
    from kimi_k3_b200.train.loop import train_one_epoch
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    from kimi_k3_b200.parallel.data_parallel import QBReducer
    losses = {}
    for mode in ("ddp", "fsdp"):
        dcfg, ctx = _dist({"data_parallel": {"mode": mode, "size": 2}})
        model = _tiny().to(ctx.device)
        full = sum(p.numel() * p.element_size() for p in model.parameters())
        g = torch.Generator().manual_seed(11 + ctx.global_rank)
        ids = torch.randint(5, 1000, (2, 128), generator=g).to(ctx.device)
        batch = {"input_ids": ids, "labels": ids.clone(), "attention_mask": torch.ones_like(ids, dtype=torch.bool)}
        opt_cfg = KimiOptimizerConfig(kind="per_head_muon_adamw", adamw_lr=1e-3, muon_lr=1e-2)
        if mode == "fsdp":
            shard_kimi_model(model, dcfg, ctx)
            frac = local_shard_bytes(model) / full
            assert frac < 0.6, frac
            params = [p for p in model.parameters() if p.requires_grad]
            opt, _ = build_kimi_optimizer(model, opt_cfg)
            if getattr(opt, "qk_clip", None) is not None:
                opt.qk_clip.replica_group = ctx.dp_group
            kw = dict(moe_controller=MoEController(model, reducer=QBReducer(ctx.dp_group)),
                      grad_norm_fn=lambda: sharded_grad_norm(params))
        else:
            plan = parallelize_kimi_model(model, dcfg, ctx)
            plan.broadcast_parameters()
            opt, _ = build_kimi_optimizer(model, opt_cfg)
            kw = dict(moe_controller=MoEController(model, reducer=plan.qb_reducer()),
                      grad_reducer=plan.sync_gradients, grad_norm_fn=plan.grad_norm)
        out = []
        for _ in range(3):
            res = train_one_epoch(model, [batch], opt, device=ctx.device, grad_clip=1.0, use_mtp=True,
                                  amp_enabled=True, amp_dtype="bf16", distributed_context=ctx, **kw)
            out.append(float(res["loss"]))
        losses[mode] = out
        dist.barrier()
    dist.destroy_process_group()
    a, b = losses["ddp"], losses["fsdp"]
    assert all(abs(x - y) < 2e-2 * max(1.0, abs(x)) for x, y in zip(a, b)), (a, b)
    assert b[-1] < b[0], b
    print("fsdp ok", a, b)


def _decode_rank():
    from kimi_k3_b200.infer import GenerationConfig, GraphDecoder, generate_tokens
    from kimi_k3_b200.infer.distributed import graph_capturable, prepare_distributed_model
    layouts = [{"tensor_parallel": {"enabled": True, "size": 2}},
               {"expert_parallel": {"enabled": True, "size": 2, "dispatch": "nvlink_fused"}},
               {"tensor_parallel": {"enabled": True, "size": 2},
                "expert_parallel": {"enabled": True, "size": 2, "overlay_tensor_parallel": True,
                                    "dispatch": "nvlink_fused"}}]
    for layout in layouts:
        dcfg, ctx = _dist(layout)
        model = prepare_distributed_model(_tiny().to(ctx.device), dcfg, ctx)
        assert graph_capturable(model)
        ids = torch.randint(5, 1000, (4, 16), generator=torch.Generator().manual_seed(5)).to(ctx.device)
        cfg = GenerationConfig(max_new_tokens=12, do_sample=False, device=str(ctx.device))
        eager = generate_tokens(model, ids, generation_config=cfg).sequences
        dec = GraphDecoder(model, max_length=ids.shape[1] + 12, generation_config=cfg, autocast_dtype=None)
        graph = dec.generate(ids).sequences
        assert dec.replays == 11, dec.replays
        dec.release()
        assert torch.equal(eager, graph), (layout, eager, graph)
    import torch.distributed as dist
    dist.barrier()
    dist.destroy_process_group()
    print("decode ok")


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    {"fsdp": _fsdp_rank, "decode": _decode_rank}[sys.argv[1]]()
