"""Command-line entry points: ``python -m kimi_k3_b200 {train,infer,validate,smoke,profiles}``.

Parity: ``scripts/{train_kimi,infer_kimi,validate_*,cpu_smoke}.py`` (reference): train from a
profile directory (or three explicit YAMLs) with ``--validate-only``, infer from a model YAML
and a checkpoint, validate data / model / distributed configurations (the latter prints the
``torchrun`` command), and a CPU smoke run that trains the tiny model and decodes tokens.
A profile name of the built-in set (``cpu_smoke``, ``t4_wikitext``, ...) may be used instead
of a directory: it is materialised under ``configs/kimi_full_pipeline``.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def _profile_paths(profile: str):
    from .config.profiles import PIPELINES, write_pipeline
    from .config.yaml_utils import resolve_kimi_pipeline_profile
    p = Path(profile)
    if not p.is_dir() and profile in PIPELINES:
        p = Path("configs/kimi_full_pipeline") / profile
        if not (p / "model.yaml").is_file():
            write_pipeline(profile, p)
    return resolve_kimi_pipeline_profile(p)


def _paths(args):
    explicit = (args.data_config, args.model_config, args.training_config)
    if args.profile:
        if any(explicit):
            raise SystemExit("--profile cannot be combined with individual YAML paths")
        pp = _profile_paths(args.profile)
        return pp.data, pp.model, pp.training
    if not all(explicit):
        raise SystemExit("pass --profile or all of --data-config --model-config --training-config")
    return tuple(Path(x) for x in explicit)


def cmd_train(args) -> int:
    from .config.model_yaml import build_model_from_yaml, load_model_config
    from .data import build_dataloaders_from_yaml, load_data_config
    from .parallel.environment import setup_distributed
    from .train.config import load_training_config, validate_pipeline_compatibility
    from .train.trainer import train_kimi_from_yaml
    data_p, model_p, train_p = _paths(args)
    tcfg = load_training_config(train_p)
    dcfg = load_data_config(data_p)
    mcfg = load_model_config(model_p)
    validate_pipeline_compatibility(tcfg, model_config=mcfg, data_config=dcfg)
    if args.validate_only:
        summary = {"data": dcfg.name, "model_d_model": mcfg.d_model, "vocab": mcfg.vocab_size,
                   "training_steps_epochs": tcfg.training.epochs, "precision": tcfg.training.precision,
                   "distributed_world": tcfg.distributed.logical_world_size}
        print(json.dumps(summary, indent=2))
        return 0
    ctx = setup_distributed(tcfg.distributed)
    data = build_dataloaders_from_yaml(data_p, distributed_context=ctx if tcfg.distributed.enabled else None)
    model = build_model_from_yaml(model_p, data_bundle=data)
    result = train_kimi_from_yaml(train_p, model=model, data=data, distributed_context=ctx)
    if ctx.is_global_zero:
        print(f"finished: {result['state'].optimizer_step} optimizer steps, last checkpoint {result['last_checkpoint']}")
    ctx.close()
    return 0


def cmd_infer(args) -> int:
    """Generate from a checkpoint.  An inference YAML with ``distributed.enabled`` shards the model
    over the torchrun ranks (TP / EP) before generating; every rank generates, rank 0 prints."""
    from dataclasses import replace
    from .infer import GenerationConfig, load_inference_yaml_config
    from .infer.distributed import run_distributed_generation
    from .infer.yaml_config import InferenceYamlConfig
    from .parallel.config import DistributedConfig
    model_p = Path(args.model_config) if args.model_config else _profile_paths(args.profile).model
    tok = None
    if args.data_config or args.profile:
        from .data import load_tokenizer_from_data_yaml
        try:
            tok = load_tokenizer_from_data_yaml(Path(args.data_config) if args.data_config
                                                else _profile_paths(args.profile).data)
        except FileNotFoundError:
            tok = None
    if args.inference_config:
        iy = load_inference_yaml_config(args.inference_config)
    else:
        iy = InferenceYamlConfig(GenerationConfig(max_new_tokens=32), DistributedConfig(), None)
    if args.max_new_tokens is not None:
        iy = replace(iy, generation=replace(iy.generation, max_new_tokens=args.max_new_tokens))
    prompt = args.prompt
    if tok is None:
        prompt = [int(x) for x in prompt.split()]
    out, ctx = run_distributed_generation(model_p, args.checkpoint, prompt, iy, tokenizer=tok,
                                          precision=args.precision, use_graph=args.graph)
    try:
        if ctx.is_global_zero:
            print(out.text if out.text is not None else out.sequences.tolist())
            print(json.dumps({"prefill_seconds": out.prefill_seconds, "decode_seconds": out.decode_seconds,
                              "tokens_per_second": out.tokens_per_second, "finish_reason": out.finish_reason,
                              "world_size": ctx.world_size}))
    finally:
        ctx.close()
    return 0


def cmd_validate(args) -> int:
    from .config.model_yaml import load_model_config
    from .data import load_data_config
    from .train.config import load_training_config
    out = {}
    if args.data_config:
        d = load_data_config(args.data_config)
        out["data"] = {"name": d.name, "kind": d.kind, "block_size": d.max_seq_len, "batch_size": d.loader.batch_size}
    if args.model_config:
        m = load_model_config(args.model_config)
        out["model"] = {"d_model": m.d_model, "vocab_size": m.vocab_size}
    if args.training_config:
        t = load_training_config(args.training_config)
        dist = t.distributed
        out["distributed"] = {"enabled": dist.enabled, "world_size": dist.logical_world_size,
                              "dp": dist.data_parallel.size, "tp": dist.tensor_parallel.size,
                              "ep": dist.expert_parallel.size,
                              "ep_overlays_tp": dist.expert_parallel.overlay_tensor_parallel}
        if dist.enabled:
            out["launch"] = (f"torchrun --standalone --nproc-per-node {dist.logical_world_size} -m kimi_k3_b200 "
                             f"train --training-config {args.training_config} ...")
    print(json.dumps(out, indent=2))
    return 0


def cmd_smoke(args) -> int:
    """CPU smoke: a few training steps of the tiny profile, then 8 decoded tokens."""
    import torch
    from . import KimiK3, kimi_k3_cpu_tiny_config
    from .data import SyntheticRetrievalConfig, create_synthetic_retrieval_dataloaders
    from .infer import GenerationConfig, generate_tokens
    from .train.engine import MoEController
    from .train.loop import train_one_epoch
    from .train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    torch.manual_seed(0)
    cfg = SyntheticRetrievalConfig(num_train_examples=16, num_val_examples=4, block_size=32, min_filler_tokens=4,
                                   max_filler_tokens=12, num_keys_per_example=2, vocab_filler_size=32,
                                   num_key_types=8, num_value_types=16, batch_size=4)
    train, _, tok = create_synthetic_retrieval_dataloaders(cfg)
    model = KimiK3(kimi_k3_cpu_tiny_config())
    opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(muon_lr=0.01))
    stats = train_one_epoch(model, train, opt, grad_clip=1.0, use_mtp=True, moe_controller=MoEController(model))
    ids = next(iter(train))["input_ids"][:1, :12]
    out = generate_tokens(model, ids, generation_config=GenerationConfig(max_new_tokens=8))
    print(json.dumps({"loss": stats["loss"], "steps": stats["optimizer_steps"],
                      "generated": out.generated_ids.tolist(), "decoded": tok.decode(out.generated_ids[0].tolist())}))
    return 0


def cmd_profiles(args) -> int:
    from .config.profiles import write_all_pipelines
    for p in write_all_pipelines(args.output):
        print(p)
    return 0


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(prog="kimi_k3_b200", description="Kimi K3 (B200) framework")
    sub = ap.add_subparsers(dest="command", required=True)
    for name in ("train", "infer", "validate"):
        p = sub.add_parser(name)
        p.add_argument("--profile")
        p.add_argument("--data-config")
        p.add_argument("--model-config")
        p.add_argument("--training-config")
        if name == "train":
            p.add_argument("--validate-only", action="store_true")
        if name == "infer":
            p.add_argument("--checkpoint", required=True)
            p.add_argument("--prompt", required=True)
            p.add_argument("--inference-config")
            p.add_argument("--max-new-tokens", type=int, default=None,
                           help="overrides the inference YAML (default 32 without one)")
            p.add_argument("--precision", choices=("model", "fp32", "bf16", "fp16"), default="model")
            p.add_argument("--graph", action="store_true",
                           help="serve the decode loop from one captured CUDA graph per token")
    sub.add_parser("smoke")
    pp = sub.add_parser("profiles")
    pp.add_argument("--output", default="configs/kimi_full_pipeline")
    return ap


def main(argv=None) -> int:
    args = build_parser().parse_args(argv)
    return {"train": cmd_train, "infer": cmd_infer, "validate": cmd_validate, "smoke": cmd_smoke,
            "profiles": cmd_profiles}[args.command](args)


if __name__ == "__main__":
    sys.exit(main())
