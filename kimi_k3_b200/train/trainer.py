"""Master trainer: ``train_kimiK3`` and the YAML entry point ``train_kimi_from_yaml``.

Parity: ``training/train_kimi_k3.py:133-772`` and ``training/yaml_config.py:176-233``
(reference): distributed setup and per-replica seeding, precision, TP/EP sharding then data
parallelism, the progressive context curriculum with loader rebuilds on transitions, the
canonical Per-Head Muon + Muon + AdamW optimizer and first-update-aware warmup-cosine
schedule, EMA, Quantile-Balancing windows, diagnostics, resume from a single or distributed
checkpoint, per-epoch evaluation / preview / atomic checkpoints with pruning.

B200 specifics: ``data_parallel.mode`` ``ddp`` uses the overlapped bucketed reducer and
``fsdp`` shards parameters, gradients and optimizer state per token mixer / FFN unit
(``parallel/fsdp.py``); the EMA shadow stays on the GPU.
"""
from __future__ import annotations

import math
import random
from pathlib import Path
from typing import Any

import numpy as np
import torch

from .checkpoints import load_checkpoint, prune_checkpoints, save_checkpoint, write_latest_pointer
from .config import (CheckpointConfig, OptimizerConfig, PredictionConfig, PretrainingLossConfig, SchedulerConfig,
                     TrainingConfig, load_training_config, validate_pipeline_compatibility)
from .curriculum import ContextCurriculumConfig, ProgressiveContextCurriculum, build_context_loader
from .diagnostics import DiagnosticsConfig, KimiDiagnosticCollector
from .ema import EMA
from .engine import MoEController
from .loop import eval_one_epoch, next_token_preview, print_next_token_preview, train_one_epoch
from .optimizer import KimiOptimizerConfig, build_kimi_optimizer, build_parameter_registry
from .printing import KimiTrainingPrinter, print_topology
from .scheduler import build_warmup_cosine_scheduler
from .state import JSONLLogger, MemoryLogger, TrainerState, make_grad_scaler


def set_seed(seed: int, deterministic: bool = False) -> None:
    random.seed(seed)
    np.random.seed(seed % (2 ** 32))
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)
    if deterministic:
        torch.use_deterministic_algorithms(True, warn_only=True)


def resolve_device(device) -> torch.device:
    if device in (None, "auto"):
        return torch.device("cuda" if torch.cuda.is_available() else "cpu")
    return torch.device(device)


def _loader_batches(loader, cap):
    try:
        n = len(loader)
    except TypeError:
        n = cap or 1
    return min(n, cap) if cap is not None else n


def _merge_segments(segments: list) -> dict:
    if len(segments) == 1:
        return segments[0]
    tok = sum(s.get("tokens", 0.0) for s in segments) or 1.0
    out = dict(segments[-1])
    for k in ("loss", "ntp_loss"):
        out[k] = sum(s[k] * s.get("tokens", 0.0) for s in segments) / tok
    for k in ("num_batches", "optimizer_steps", "skipped_optimizer_steps", "num_samples", "tokens", "ntp_tokens",
              "mtp_tokens", "epoch_time_seconds"):
        out[k] = sum(s.get(k, 0.0) for s in segments)
    out["context_transition"] = [s.get("context_transition") for s in segments if s.get("context_transition")]
    return out


def train_kimiK3(*, model, train_loader=None, train_loader_factory=None, val_loader=None, device="auto",
                 training_config: TrainingConfig | None = None, loss_config: PretrainingLossConfig | None = None,
                 optimizer_config: OptimizerConfig | None = None,
                 kimi_optimizer_config: KimiOptimizerConfig | None = None,
                 scheduler_config: SchedulerConfig | None = None, diagnostics_config: DiagnosticsConfig | None = None,
                 context_curriculum_config: ContextCurriculumConfig | None = None,
                 checkpoint_config: CheckpointConfig | None = None, prediction_config: PredictionConfig | None = None,
                 optimizer=None, scheduler=None, ema=None, use_ema: bool = False, ema_decay: float = 0.999,
                 eval_use_ema: bool = False, curriculum=None, logger=None, tokenizer=None, id_to_text=None,
                 total_steps: int | None = None, verbose: bool = True, distributed_config=None,
                 distributed_context=None) -> dict:
    """Train a Kimi K3 model end to end (reference signature)."""
    from ..parallel.config import DistributedConfig
    from ..parallel.environment import setup_distributed
    from ..parallel.parallelize import parallelize_kimi_model
    tc = training_config or TrainingConfig()
    dcfg = distributed_config or DistributedConfig()
    if loss_config is not None:
        from ..models.losses import KimiPretrainingLoss
        mtp = getattr(getattr(model, "config", None), "mtp", None)
        default_w = float(getattr(mtp, "loss_weight", 0.0)) if tc.use_mtp else 0.0
        model.pretraining_loss = KimiPretrainingLoss(
            lambda_mtp=default_w if loss_config.mtp_loss_weight is None else loss_config.mtp_loss_weight,
            ignore_index=loss_config.ignore_index, label_smoothing=loss_config.label_smoothing,
            label_alignment=loss_config.label_alignment)
    legacy = optimizer_config
    optimizer_config = optimizer_config or OptimizerConfig()
    if kimi_optimizer_config is None:
        kimi_optimizer_config = (KimiOptimizerConfig(kind="adamw", adamw_lr=optimizer_config.learning_rate,
                                                     adamw_betas=tuple(optimizer_config.betas),
                                                     adamw_eps=optimizer_config.eps,
                                                     weight_decay=optimizer_config.weight_decay,
                                                     qk_clip_enabled=False)
                                 if legacy is not None else KimiOptimizerConfig())
    scheduler_config = scheduler_config or SchedulerConfig()
    diagnostics_config = diagnostics_config or DiagnosticsConfig()
    context_curriculum_config = context_curriculum_config or ContextCurriculumConfig()
    checkpoint_config = checkpoint_config or CheckpointConfig()
    prediction_config = prediction_config or PredictionConfig()
    owns_ctx = distributed_context is None
    ctx = distributed_context if distributed_context is not None else setup_distributed(dcfg)
    if ctx.world_size != dcfg.logical_world_size:
        raise RuntimeError("distributed context and configuration disagree")
    replica_rank = ctx.dp_rank * (1 if ctx.ep_overlays_tp else ctx.ep_size) + (0 if ctx.ep_overlays_tp else ctx.ep_rank)
    set_seed(tc.seed + replica_rank, deterministic=tc.deterministic)
    dev = ctx.device if dcfg.enabled else resolve_device(device)
    if tc.precision == "fp16" and dev.type != "cuda":
        raise RuntimeError("FP16 training requires CUDA")
    amp = tc.precision != "fp32"
    scaler = make_grad_scaler(tc.precision, dev)
    model.to(dev)
    plan = zero = None
    if dcfg.enabled:
        plan = parallelize_kimi_model(model, dcfg, ctx)
        model.to(dev)
        if dcfg.data_parallel.mode == "fsdp" and (use_ema or ema is not None):
            raise ValueError("EMA is unsupported with the sharded (fsdp) data-parallel mode")
        plan.broadcast_parameters()
        if dcfg.data_parallel.mode == "fsdp":
            # parameters, gradients and optimizer state sharded over the data-parallel group
            from ..parallel.fsdp import shard_kimi_model
            shard_kimi_model(model, dcfg, ctx)
    raw_cfg = getattr(model, "config", None)
    if train_loader is not None and train_loader_factory is not None:
        raise ValueError("pass train_loader or train_loader_factory, not both")
    if curriculum is not None and context_curriculum_config.enabled:
        raise ValueError("pass curriculum or context_curriculum_config, not both")
    if curriculum is None and context_curriculum_config.enabled:
        mtp = getattr(raw_cfg, "mtp", None)
        curriculum = ProgressiveContextCurriculum(
            context_curriculum_config, training_max_seq_len=tc.max_seq_len,
            model_max_seq_len=getattr(raw_cfg, "max_seq_len", tc.max_seq_len),
            mtp_min_seq_len=int(getattr(mtp, "future_offset", 2)) + 1 if tc.use_mtp else 1)
    if curriculum is not None and curriculum.enabled and curriculum.config.reset_dataloader_on_transition \
            and train_loader_factory is None:
        raise ValueError("enabled PCC with loader reset requires train_loader_factory")
    ctx_len = curriculum.current_max_seq_len() if curriculum is not None else tc.max_seq_len
    if train_loader_factory is not None:
        train_loader = build_context_loader(train_loader_factory, ctx_len)
    if train_loader is None:
        raise ValueError("train_loader or train_loader_factory is required")
    optimizer_info = None
    if optimizer is None:
        optimizer, registry = build_kimi_optimizer(model, kimi_optimizer_config)
        optimizer_info = registry.to_dict() if hasattr(registry, "to_dict") else registry
    else:
        registry = (optimizer.parameter_assignment_report() if hasattr(optimizer, "parameter_assignment_report")
                    else build_parameter_registry(model, kind="adamw", strict=False))
    step_optimizer, grad_sync, grad_norm = optimizer, None, None
    if plan is not None:
        grad_sync, grad_norm = plan.sync_gradients, plan.grad_norm
    if dcfg.enabled and dcfg.data_parallel.mode == "fsdp":
        from ..parallel.fsdp import sharded_grad_norm
        reducers = list(plan.reducers) if plan is not None else []
        params_all = [p for p in model.parameters() if p.requires_grad]

        def grad_sync():  # the sharded gradients were reduce-scattered in backward; other groups here
            for r in reducers:
                if r.group is not ctx.dp_group:
                    r.all_reduce_gradients()

        def grad_norm():
            return sharded_grad_norm(params_all)
        qk = getattr(optimizer, "qk_clip", None)
        if qk is not None:
            qk.replica_group = ctx.dp_group
    if total_steps is None:
        per_epoch = math.ceil(_loader_batches(train_loader, tc.max_batches_per_epoch) / tc.gradient_accumulation_steps)
        total_steps = max(per_epoch * tc.epochs, 1)
    warmup = scheduler_config.resolve_warmup_steps(total_steps)
    if scheduler is None:
        scheduler = build_warmup_cosine_scheduler(
            optimizer, total_steps=total_steps, warmup_steps=warmup,
            min_lr=kimi_optimizer_config.adamw_lr * scheduler_config.min_lr_ratio,
            min_muon_lr=kimi_optimizer_config.resolved_muon_lr * scheduler_config.min_lr_ratio,
            prepare_first_update=True)
    if ema is None and use_ema:
        ema = EMA(model, decay=ema_decay)
    if eval_use_ema and ema is None:
        raise ValueError("eval_use_ema=True requires use_ema or an EMA object")
    state = TrainerState()
    qb_reducer = plan.qb_reducer() if plan is not None else None
    moe_ctl = MoEController(model, reducer=qb_reducer)
    collector = KimiDiagnosticCollector(model, diagnostics_config, parameter_specs=registry.specs)
    if dcfg.enabled and ctx.initialized and ctx.world_size > 1:
        collector.budget_device = ctx.device   # every rank degrades diagnostics on the same steps
    log_rank = dcfg.diagnostics.log_rank
    is_log = ctx.global_rank == log_rank
    printer = KimiTrainingPrinter() if verbose and is_log else None
    out_dir = Path(checkpoint_config.output_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    owns_logger = logger is None
    if logger is None:
        logger = JSONLLogger(out_dir / f"{checkpoint_config.run_name}.jsonl") if is_log else MemoryLogger()
    history = {"train": [], "validation": [], "predictions": []}
    if checkpoint_config.resume_from is not None:
        history = _resume(checkpoint_config, dcfg, ctx, model, step_optimizer, scheduler, scaler, ema, state,
                          curriculum, collector, history)
        model.to(dev)
        if curriculum is not None:
            if curriculum.state.tokens_seen != state.tokens_seen:
                raise ValueError("trainer and context curriculum token counts disagree")
            state.curriculum_stage_index = curriculum.stage_index
            if train_loader_factory is not None:
                train_loader = build_context_loader(train_loader_factory, curriculum.current_max_seq_len())
    if printer is not None:
        if dcfg.enabled:
            print_topology(ctx, log_rank=log_rank, per_rank_debug=dcfg.diagnostics.per_rank_debug,
                           wrapper_mode=dcfg.data_parallel.mode, checkpoint_format=dcfg.checkpoint.format,
                           global_batch_size=getattr(train_loader, "batch_size", 0) * ctx.data_replicas
                           * tc.gradient_accumulation_steps)
        printer.print_run_header(run_name=checkpoint_config.run_name, model=model, device=dev,
                                 precision=tc.precision, optimizer_kind=kimi_optimizer_config.kind, epochs=tc.epochs,
                                 total_steps=total_steps, warmup_steps=warmup, registry=registry)
    last_ckpt = None
    try:
        for epoch in range(state.epoch, tc.epochs):
            sampler = getattr(train_loader, "sampler", None)
            if hasattr(sampler, "set_epoch"):
                sampler.set_epoch(epoch)

            def on_step(m):
                alerts = m.pop("_alerts", ())
                if printer is not None and state.optimizer_step % max(tc.log_every_steps, 1) == 0:
                    printer.print_step(state.optimizer_step, m, alerts)

            segments, remaining = [], tc.max_batches_per_epoch
            while True:
                seg = train_one_epoch(model, train_loader, step_optimizer, device=dev, scheduler=scheduler,
                                      scaler=scaler, ema=ema, amp_enabled=amp, amp_dtype=tc.precision,
                                      grad_accum_steps=tc.gradient_accumulation_steps, grad_clip=tc.grad_clip_norm,
                                      max_batches=remaining, use_mtp=tc.use_mtp, state=state, moe_controller=moe_ctl,
                                      curriculum=curriculum, log_every=tc.log_every_steps, logger=logger,
                                      on_optimizer_step=on_step, diagnostics=collector, max_seq_len=tc.max_seq_len,
                                      stop_on_context_transition=curriculum is not None and train_loader_factory
                                      is not None, distributed_context=ctx if dcfg.enabled else None,
                                      grad_reducer=grad_sync, grad_norm_fn=grad_norm)
                segments.append(seg)
                if remaining is not None:
                    remaining -= int(seg["num_batches"])
                if seg.get("context_transition") is None or curriculum is None or train_loader_factory is None \
                        or (remaining is not None and remaining <= 0):
                    break
                train_loader = build_context_loader(train_loader_factory, curriculum.current_max_seq_len())
                sampler = getattr(train_loader, "sampler", None)
                if hasattr(sampler, "set_epoch"):
                    sampler.set_epoch(epoch)
            train_stats = _merge_segments(segments)
            history["train"].append(train_stats)
            eval_stats = None
            if val_loader is not None and (epoch + 1) % tc.eval_every_epochs == 0:
                eval_stats = eval_one_epoch(model, val_loader, device=dev, amp_enabled=amp, amp_dtype=tc.precision,
                                            max_batches=tc.max_eval_batches, use_mtp=tc.use_mtp, ema=ema,
                                            use_ema=eval_use_ema, distributed_context=ctx if dcfg.enabled else None)
                history["validation"].append(eval_stats)
                if state.best_eval_loss is None or eval_stats["loss"] < state.best_eval_loss:
                    state.best_eval_loss = float(eval_stats["loss"])
            pe = tc.prediction_every_epochs
            if pe is not None and (epoch + 1) % pe == 0:
                src = val_loader if val_loader is not None else train_loader
                batch = next(iter(src), None)
                if batch is not None:
                    pred = next_token_preview(model, batch, device=dev, amp_enabled=amp, amp_dtype=tc.precision,
                                              use_mtp=tc.use_mtp, sample_index=prediction_config.sample_index,
                                              max_tokens=prediction_config.max_tokens, tokenizer=tokenizer,
                                              id_to_text=id_to_text)
                    pred["epoch"] = epoch
                    history["predictions"].append(pred)
                    if verbose and is_log:
                        print_next_token_preview(pred, title=f"Kimi K3 next-token preview | epoch={epoch}")
            state.epoch = epoch + 1
            logger.log(state.optimizer_step, {"epoch": epoch, "train/loss": float(train_stats["loss"]),
                                              "eval/loss": None if eval_stats is None else float(eval_stats["loss"]),
                                              "tokens_seen": state.tokens_seen,
                                              "context_stage": state.curriculum_stage_index})
            if (epoch + 1) % tc.checkpoint_every_epochs == 0 or epoch + 1 == tc.epochs:
                moe_ctl.assert_clean()
                last_ckpt = _save(out_dir, checkpoint_config, dcfg, ctx, model, step_optimizer, scheduler, scaler,
                                  ema, state, curriculum, collector, train_loader, raw_cfg, registry, epoch, history,
                                  dict(training=tc, loss=loss_config, optimizer=optimizer_config,
                                       kimi_optimizer=kimi_optimizer_config, scheduler=scheduler_config,
                                       diagnostics=diagnostics_config,
                                       context_curriculum=(curriculum.config if curriculum is not None
                                                           else context_curriculum_config),
                                       checkpoint=checkpoint_config, distributed=dcfg), is_log)
            if printer is not None:
                printer.print_epoch_summary(epoch=epoch, state=state, train_stats=train_stats, eval_stats=eval_stats,
                                            checkpoint=last_ckpt)
    finally:
        if owns_logger and hasattr(logger, "close"):
            logger.close()
        if owns_ctx:
            ctx.close()
    return {"model": model, "optimizer": optimizer, "optimizer_info": optimizer_info, "scheduler": scheduler,
            "ema": ema, "state": state, "history": history, "last_checkpoint": last_ckpt, "curriculum": curriculum,
            "diagnostics": collector, "total_steps": total_steps, "distributed_plan": plan}


def _serialise(configs: dict) -> dict:
    return {k: (None if v is None else (v.to_dict() if hasattr(v, "to_dict") else v)) for k, v in configs.items()}


def _save(out_dir, ck, dcfg, ctx, model, optimizer, scheduler, scaler, ema, state, curriculum, collector, loader,
          raw_cfg, registry, epoch, history, configs, is_log):
    from ..parallel.checkpoint import save_distributed_checkpoint
    name = f"{ck.run_name}_epoch_{epoch:04d}"
    if dcfg.enabled:
        path = out_dir / name
        save_distributed_checkpoint(path, model=model, context=ctx, step=state.optimizer_step,
                                    optimizer=optimizer if ck.save_optimizer else None, scheduler=scheduler,
                                    scaler=scaler, ema=ema, trainer_state=state, curriculum=curriculum,
                                    diagnostics=collector, sampler=getattr(loader, "sampler", None),
                                    model_config=None if raw_cfg is None else raw_cfg.to_dict(),
                                    training_config=_serialise(configs), registry_fingerprint=registry.fingerprint,
                                    save_rng=ck.save_rng_state and dcfg.checkpoint.save_rng_per_rank,
                                    extra={"history": history, "optimizer_type": type(optimizer).__name__})
    else:
        path = out_dir / f"{name}.pt"
        save_checkpoint(path, model, optimizer=optimizer if ck.save_optimizer else None, scheduler=scheduler,
                        scaler=scaler, ema=ema, trainer_state=state, curriculum=curriculum, epoch=epoch,
                        global_step=state.optimizer_step, model_config=raw_cfg, training_config=_serialise(configs),
                        history=history, metadata={"optimizer_type": type(optimizer).__name__},
                        save_rng_state=ck.save_rng_state, diagnostics=collector)
    if is_log:
        write_latest_pointer(out_dir, path)
        if not dcfg.enabled:
            prune_checkpoints(out_dir, ck.keep_last_n, pattern=f"{ck.run_name}_epoch_*.pt", protect=(path,))
        else:
            import shutil
            dirs = sorted(p for p in out_dir.glob(f"{ck.run_name}_epoch_*") if p.is_dir())
            for p in dirs[:-ck.keep_last_n] if ck.keep_last_n > 0 else []:
                shutil.rmtree(p, ignore_errors=True)
    return path


def _resume(ck, dcfg, ctx, model, optimizer, scheduler, scaler, ema, state, curriculum, collector, history):
    from ..parallel.checkpoint import load_distributed_checkpoint
    from .checkpoints import resolve_resume_path
    src = resolve_resume_path(ck.resume_from, ck.output_dir) if ck.resume_from == "latest" else ck.resume_from
    if dcfg.enabled:
        r = load_distributed_checkpoint(src, model=model, context=ctx, optimizer=optimizer if ck.save_optimizer
                                        else None, scheduler=scheduler, scaler=scaler, ema=ema, trainer_state=state,
                                        curriculum=curriculum, diagnostics=collector, restore_rng=ck.save_rng_state)
        return r.get("extra", {}).get("history") or history
    r = load_checkpoint(src, model, optimizer=optimizer if ck.save_optimizer else None, scheduler=scheduler,
                        scaler=scaler, ema=ema, trainer_state=state, curriculum=curriculum, diagnostics=collector,
                        map_location="cpu", strict=True, restore_rng=ck.save_rng_state)
    return r.get("history") or history


def train_kimi_from_yaml(path, *, model, data, logger=None, distributed_context=None) -> dict:
    """Train ``model`` on ``data`` (a DataBundle) with one validated training YAML."""
    cfg = load_training_config(path)
    validate_pipeline_compatibility(cfg, model_config=model.config, data_config=data.config)
    reset = cfg.context_curriculum.enabled and cfg.context_curriculum.reset_dataloader_on_transition
    loaders = {"train_loader_factory": data.train_loader_factory} if reset else {"train_loader": data.train_loader}
    if cfg.kernels is not None and not cfg.kernels.native_kernels:
        import os
        os.environ["KIMI_K3_KERNELS"] = "0"
    return train_kimiK3(model=model, val_loader=data.val_loader, device=cfg.runtime.device,
                        training_config=cfg.training, loss_config=cfg.loss, kimi_optimizer_config=cfg.optimizer,
                        scheduler_config=cfg.scheduler, diagnostics_config=cfg.diagnostics,
                        context_curriculum_config=cfg.context_curriculum, checkpoint_config=cfg.checkpoint,
                        prediction_config=cfg.prediction, use_ema=cfg.runtime.use_ema, ema_decay=cfg.runtime.ema_decay,
                        eval_use_ema=cfg.runtime.eval_use_ema, logger=logger, tokenizer=data.tokenizer,
                        total_steps=cfg.runtime.total_steps, verbose=cfg.runtime.verbose,
                        distributed_config=cfg.distributed, distributed_context=distributed_context, **loaders)


__all__ = ["train_kimiK3", "train_kimi_from_yaml", "set_seed", "resolve_device"]
