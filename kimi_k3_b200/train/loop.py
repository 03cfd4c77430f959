"""Epoch loops: token-exact training windows, side-effect-free evaluation, previews.

Parity: ``training/train_one_epoch.py:63-598``, ``training/eval_one_epoch.py:22-109``,
``training/predictions.py:42-138``, ``training/model_call.py``, ``data/batch.py`` (reference).

Token-exact accumulation: a window of ``grad_accum_steps`` micro-batches optimises
``sum(ntp_sum) / N_ntp + lambda * sum(mtp_sum) / N_mtp`` with ``N`` the window's (global,
over data and expert replicas) valid-token counts. The reference keeps every micro-batch
graph alive and runs one backward over their sum. Here the normalisers are computed first on
the host copies of the window's batches (:meth:`KimiK3.loss_normalizers`; one tiny all-reduce
when distributed), then each micro-batch runs forward AND backward with the window
normalisers: the same gradient (backward is linear in the per-batch sums) with the memory of
one micro-batch. Models without ``loss_normalizers`` fall back to the retained-graph window.

With ``grad_accum_steps == 1`` on one CUDA device the window is a single batch and the step
can run through a captured CUDA graph (``engine``).
"""
from __future__ import annotations

import inspect
import math
import time
from contextlib import nullcontext
from typing import Any, Callable

import torch

from .state import (LossContribution, TrainerState, combine_distributed_window_loss, combine_window_loss,
                    compute_loss_metrics, extract_loss_contribution)

SEQUENCE_KEYS = ("input_ids", "labels", "attention_mask", "loss_mask", "boundary_mask", "token_weights",
                 "segment_ids")


# --------------------------------------------------------------------------- batches and model calls
def normalize_lm_batch(batch) -> dict:
    """dict / tensor / (ids, labels[, mask]) -> ``model(**batch)`` dict (labels default to ids)."""
    if isinstance(batch, dict):
        if "input_ids" not in batch:
            raise KeyError(f"Batch dict must contain 'input_ids'. Available keys: {list(batch.keys())}")
        if "labels" not in batch:
            batch = dict(batch, labels=batch["input_ids"])
        return batch
    if torch.is_tensor(batch):
        return {"input_ids": batch, "labels": batch}
    if isinstance(batch, (list, tuple)):
        if len(batch) == 2:
            return {"input_ids": batch[0], "labels": batch[1]}
        if len(batch) == 3:
            return {"input_ids": batch[0], "labels": batch[1], "attention_mask": batch[2]}
        raise ValueError(f"Unsupported batch tuple length {len(batch)}; expected 2 or 3.")
    raise TypeError(f"Unsupported batch type: {type(batch)}")


def move_batch_to_device(batch: dict, device, non_blocking: bool = True) -> dict:
    device = torch.device(device)
    return {k: (v.to(device, non_blocking=non_blocking and v.is_pinned()) if torch.is_tensor(v) else v)
            for k, v in batch.items()}


def filter_forward_kwargs(model, values: dict) -> dict:
    raw = model.module if hasattr(model, "module") else model
    params = inspect.signature(raw.forward).parameters
    if any(p.kind == inspect.Parameter.VAR_KEYWORD for p in params.values()):
        return values
    return {k: v for k, v in values.items() if k in params}


def call_model(model, batch: dict, *, use_mtp: bool | None = None, extra_kwargs: dict | None = None):
    values = dict(batch)
    if use_mtp is not None:
        values["use_mtp"] = use_mtp
        values["training_phase"] = "pretrain"
    if extra_kwargs:
        values.update(extra_kwargs)
    return model(**filter_forward_kwargs(model, values))


def autocast_ctx(device, enabled: bool = True, amp_dtype: str = "bf16"):
    device = torch.device(device)
    if not enabled or device.type != "cuda":
        return nullcontext()
    return torch.autocast("cuda", dtype={"bf16": torch.bfloat16, "fp16": torch.float16}.get(amp_dtype, torch.bfloat16))


def _unwrap(model):
    return model.module if hasattr(model, "module") else model


def _dist_sum(values: list, context) -> list:
    """Sum host floats over the data and expert replica groups (float64, one collective per group)."""
    if context is None or not getattr(context, "initialized", False):
        return list(values)
    t = torch.tensor(values, dtype=torch.float64, device=context.device)
    for group, size in _replica_axes(context):
        if size > 1:
            torch.distributed.all_reduce(t, group=group)
    return t.tolist()


def _replica_axes(context) -> tuple:
    if hasattr(context, "data_replica_groups"):
        return context.data_replica_groups
    return ((getattr(context, "dp_group", None), getattr(context, "dp_size", 1)),
            (getattr(context, "ep_group", None), getattr(context, "ep_size", 1)))


def _dist_all_true(flag: bool, context) -> bool:
    if context is None or not getattr(context, "initialized", False):
        return bool(flag)
    t = torch.tensor([1 if flag else 0], dtype=torch.int32, device=context.device)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
    return bool(t.item())


@torch.no_grad()
def global_grad_norm(parameters, context=None) -> torch.Tensor | None:
    """Device scalar: L2 norm over every gradient (squared norms summed across the world for
    sharded parameters; replicated gradients are identical after reduction)."""
    grads = [p.grad for p in parameters if p.grad is not None]
    if not grads:
        return None
    sq = torch.stack([n.float() for n in torch._foreach_norm(grads, 2.0)]).square().sum()
    if context is not None and getattr(context, "sharded_grads", False):
        torch.distributed.all_reduce(sq)
    return sq.sqrt()


# --------------------------------------------------------------------------- training
def train_one_epoch(model, dataloader, optimizer, *, device="cpu", scheduler=None, scaler=None, ema=None,
                    amp_enabled: bool = False, amp_dtype: str = "bf16", grad_accum_steps: int = 1,
                    grad_clip: float | None = None, max_batches: int | None = None, use_mtp: bool | None = None,
                    state: TrainerState | None = None, moe_controller=None, curriculum=None,
                    log_every: int | None = None, logger=None,
                    on_optimizer_step: Callable[[dict], None] | None = None, diagnostics=None,
                    max_seq_len: int | None = None, context_ignore_index: int = -100,
                    image_token_id: int | None = None, video_token_id: int | None = None,
                    stop_on_context_transition: bool = True, distributed_context=None, grad_reducer=None,
                    grad_norm_fn=None, engine=None) -> dict:
    """Train one epoch (reference signature plus ``grad_reducer`` / ``grad_norm_fn``: the
    gradient synchronisation and global norm of a parallel plan)."""
    from .curriculum import truncate_batch_to_context
    if grad_accum_steps <= 0:
        raise ValueError("grad_accum_steps must be positive")
    if grad_clip is not None and grad_clip <= 0:
        raise ValueError("grad_clip must be None or positive")
    if max_batches is not None and max_batches < 0:
        raise ValueError("max_batches must be None or non-negative")
    device = torch.device(device)
    from ..parallel.fsdp import reshard_all
    reshard_all(model)  # after an evaluation forward the sharded root would list gathered tensors
    model.to(device).train()
    state = TrainerState() if state is None else state
    raw = _unwrap(model)
    streaming = hasattr(raw, "loss_normalizers")
    params = [p for p in model.parameters() if p.requires_grad]
    replicas = 1
    if distributed_context is not None and getattr(distributed_context, "initialized", False):
        for _, size in _replica_axes(distributed_context):
            replicas *= size
    optimizer.zero_grad(set_to_none=True)
    totals = {"contribs": [], "steps": 0, "skipped": 0, "pre": 0.0, "post": 0.0, "n_norm": 0, "samples": 0}
    started = time.perf_counter()
    transition_event = None
    stop = False
    it = iter(dataloader)
    batch_index = 0
    exhausted = False

    def next_window():
        nonlocal batch_index, exhausted
        items = []
        data_t = time.perf_counter()
        while len(items) < grad_accum_steps and not exhausted:
            if max_batches is not None and batch_index >= max_batches:
                exhausted = True
                break
            try:
                rb = next(it)
            except StopIteration:
                exhausted = True
                break
            batch_index += 1
            b = normalize_lm_batch(rb)
            active = curriculum.current_max_seq_len() if curriculum is not None else max_seq_len
            if active is not None:
                b, cm = truncate_batch_to_context(b, active, ignore_index=context_ignore_index,
                                                  image_token_id=image_token_id, video_token_id=video_token_id)
            else:
                ids, am = b["input_ids"], b.get("attention_mask")
                cap = int(ids.numel())
                valid = cap if am is None else int(am.sum().item())
                cm = {"valid_tokens": float(valid), "padding_fraction": 1.0 - valid / max(cap, 1),
                      "sequence_length": float(ids.shape[1])}
            if curriculum is not None:
                curriculum.validate_sequence_length(int(b["input_ids"].shape[1]))
                curriculum.validate_valid_tokens(b["attention_mask"].sum(dim=1))
            items.append((b, cm))
        return items, time.perf_counter() - data_t

    try:
        while not stop:
            window, data_s = next_window()
            if not window:
                break
            t0 = time.perf_counter()
            if moe_controller is not None:
                moe_controller.begin()
            step_no = state.optimizer_step + 1
            diag_kwargs = diagnostics.model_kwargs_for_step(step_no) if diagnostics is not None else {}
            diag_metrics = {}
            fwd_s = 0.0
            counts = None
            if streaming:
                local = [0.0, 0.0]
                per = []
                for b, _ in window:
                    n = raw.loss_normalizers(b["input_ids"], b.get("labels"), b.get("attention_mask"),
                                             b.get("loss_mask"), b.get("boundary_mask"), b.get("token_weights"),
                                             use_mtp=use_mtp is not False)
                    per.append(n)
                    local[0] += n[0]
                    local[1] += n[1]
                counts = _dist_sum(local, distributed_context)
                if counts[0] <= 0:
                    raise ValueError("accumulation window contains no valid NTP tokens")
            contribs = []
            for i, (b, cm) in enumerate(window):
                db = move_batch_to_device(b, device)
                kw = diag_kwargs if i == 0 else {}
                f0 = time.perf_counter()
                with autocast_ctx(device, enabled=amp_enabled, amp_dtype=amp_dtype):
                    out = call_model(model, db, use_mtp=use_mtp, extra_kwargs=kw)
                    c = extract_loss_contribution(out, db)
                fwd_s += time.perf_counter() - f0
                if diagnostics is not None and i == 0:
                    diag_metrics = diagnostics.collect_output(out, step=step_no)
                reducer = getattr(grad_reducer, "__self__", None)
                if reducer is not None and hasattr(reducer, "armed"):
                    reducer.armed = i == len(window) - 1 or not streaming
                if streaming:
                    obj = c.ntp_loss_sum * (replicas / counts[0])
                    if c.mtp_loss_sum is not None and counts[1] > 0:
                        obj = obj + c.lambda_mtp * c.mtp_loss_sum * (replicas / counts[1])
                    (obj if scaler is None else scaler.scale(obj)).backward()
                    c = LossContribution(c.ntp_loss_sum.detach(), c.ntp_normalizer,
                                         None if c.mtp_loss_sum is None else c.mtp_loss_sum.detach(),
                                         c.mtp_normalizer, c.lambda_mtp, c.reported_loss, c.batch_tokens)
                contribs.append(c)
                state.micro_step += 1
                state.samples_seen += int(db["input_ids"].shape[0])
                state.tokens_seen += c.batch_tokens
                state.valid_ntp_tokens_seen += int(c.ntp_normalizer)
                state.valid_mtp_tokens_seen += int(c.mtp_normalizer)
                totals["samples"] += int(db["input_ids"].shape[0])
                totals["contribs"].append(c)
                del out
            b0 = time.perf_counter()
            objective, wstats = combine_distributed_window_loss(contribs, distributed_context)
            if not streaming:
                (objective if scaler is None else scaler.scale(objective)).backward()
            backward_ms = (time.perf_counter() - b0) * 1000.0
            if not _dist_all_true(math.isfinite(wstats["loss"]), distributed_context):
                if moe_controller is not None:
                    moe_controller.discard()
                optimizer.zero_grad(set_to_none=True)
                raise FloatingPointError("non-finite training loss")
            # global counters: other replicas' tokens of this window
            local_tokens = sum(c.batch_tokens for c in contribs)
            state.tokens_seen += int(wstats["tokens"] - local_tokens)
            state.valid_ntp_tokens_seen += int(wstats["ntp_tokens"] - sum(c.ntp_normalizer for c in contribs))
            state.valid_mtp_tokens_seen += int(wstats["mtp_tokens"] - sum(c.mtp_normalizer for c in contribs))
            if grad_reducer is not None:
                grad_reducer()
            if scaler is not None:
                scaler.unscale_(optimizer)
            pre_t = grad_norm_fn() if grad_norm_fn is not None else global_grad_norm(params, distributed_context)
            pre = None if pre_t is None else float(pre_t)
            finite = _dist_all_true(pre is None or math.isfinite(pre), distributed_context)
            if finite and grad_clip is not None and pre is not None:
                coef = min(1.0, float(grad_clip) / (pre + 1e-6))
                if coef < 1.0:
                    # sharded (DTensor) gradients are scaled through their local shards
                    torch._foreach_mul_([p.grad.to_local() if hasattr(p.grad, "to_local") else p.grad
                                         for p in params if p.grad is not None], coef)
            post = None if pre is None else (pre * min(1.0, float(grad_clip) / (pre + 1e-6)) if grad_clip else pre)
            opt_metrics = diagnostics.capture_before_optimizer_step() if diagnostics is not None else {}
            o0 = time.perf_counter()
            report = None
            executed = finite
            if finite:
                if scaler is None:
                    report = optimizer.step()
                    executed = bool(getattr(report, "executed", True))
                else:
                    old = float(scaler.get_scale())
                    report = scaler.step(optimizer)
                    scaler.update()
                    executed = float(scaler.get_scale()) >= old
            elif scaler is not None:
                scaler.update()
            executed = _dist_all_true(executed, distributed_context)
            opt_ms = (time.perf_counter() - o0) * 1000.0
            transition_pending = False
            if executed:
                if scheduler is not None:
                    scheduler.step()
                state.optimizer_step += 1
                totals["steps"] += 1
                if ema is not None:
                    ema.update(model, step=state.optimizer_step)
                if moe_controller is not None:
                    moe_controller.commit()
                if curriculum is not None:
                    if curriculum.update(state.tokens_seen):
                        transition_event = {**curriculum.last_transition.to_dict(),
                                            "loss_before_transition": float(wstats["loss"])}
                        transition_pending = True
                    state.curriculum_stage_index = curriculum.stage_index
            else:
                totals["skipped"] += 1
                state.skipped_optimizer_steps += 1
                if moe_controller is not None:
                    moe_controller.discard()
            optimizer.zero_grad(set_to_none=True)
            step_ms = (time.perf_counter() - t0) * 1000.0
            after, alerts = ({}, ())
            if diagnostics is not None:
                after, alerts = diagnostics.capture_after_optimizer_step(step=state.optimizer_step, step_time_ms=step_ms)
            if pre is not None:
                totals["pre"] += pre
                totals["post"] += post
                totals["n_norm"] += 1
            cap = sum(int(b["input_ids"].numel()) for b, _ in window)
            pad = sum(cm["padding_fraction"] * int(b["input_ids"].numel()) for b, cm in window)
            metrics = {**wstats,
                       **compute_loss_metrics(total_loss=wstats["loss"], ntp_loss=wstats["ntp_loss"],
                                              mtp_loss=None if not math.isfinite(wstats["mtp_loss"]) else wstats["mtp_loss"],
                                              ntp_tokens=wstats["ntp_tokens"], mtp_tokens=wstats["mtp_tokens"],
                                              lambda_mtp=contribs[0].lambda_mtp if contribs else 0.0),
                       "optimizer_step": float(state.optimizer_step), "optimizer_step_executed": float(executed),
                       "grad_norm_pre_clip": float("nan") if pre is None else pre,
                       "grad_norm_post_clip": float("nan") if post is None else post,
                       "train/grad_norm_global_preclip": float("nan") if pre is None else pre,
                       "train/grad_norm_global_postclip": float("nan") if post is None else post,
                       "train/grad_clip_coefficient": 1.0 if pre is None or grad_clip is None
                       else min(1.0, float(grad_clip) / max(pre, 1e-12)),
                       "learning_rate": float(optimizer.param_groups[0]["lr"]),
                       "accumulation_size_effective": float(len(window)), "train/step_time_ms": step_ms,
                       "train/forward_time_ms": fwd_s * 1000.0, "train/data_time_ms": data_s * 1000.0,
                       "train/backward_time_ms": backward_ms, "train/optimizer_time_ms": opt_ms,
                       "train/samples_per_second": sum(int(b["input_ids"].shape[0]) for b, _ in window) * replicas
                       / max(step_ms / 1000.0, 1e-12),
                       "train/tokens_per_second": wstats["tokens"] / max(step_ms / 1000.0, 1e-12),
                       "train/amp_scale": 1.0 if scaler is None else float(scaler.get_scale()),
                       "train/skipped_steps_total": float(state.skipped_optimizer_steps),
                       "train/overflow_steps_total": float(state.skipped_optimizer_steps),
                       "context/valid_tokens_per_step": float(wstats["tokens"]),
                       "context/padding_fraction": pad / max(cap, 1),
                       "context/tokens_per_second": wstats["tokens"] / max(step_ms / 1000.0, 1e-12),
                       "context/step_time_seconds": step_ms / 1000.0,
                       **diag_metrics, **opt_metrics, **after}
            if device.type == "cuda":
                metrics.update({"train/memory_allocated_mb": torch.cuda.memory_allocated(device) / 2 ** 20,
                                "train/memory_reserved_mb": torch.cuda.memory_reserved(device) / 2 ** 20,
                                "train/max_memory_allocated_mb": torch.cuda.max_memory_allocated(device) / 2 ** 20,
                                "context/peak_memory_mb": torch.cuda.max_memory_allocated(device) / 2 ** 20})
            if report is not None:
                if hasattr(optimizer, "materialize_report") and diagnostics is not None:
                    report = optimizer.materialize_report() or report
                metrics.update(getattr(report, "update_metrics", {}) or {})
                if hasattr(report, "adamw_lr"):
                    metrics["lr/adamw"] = float(report.adamw_lr)
                    metrics["lr/muon"] = float(report.muon_lr)
            if curriculum is not None:
                metrics.update(curriculum.metrics())
            elif max_seq_len is not None:
                metrics.update({"context/stage_index": 0.0, "context/max_seq_len": float(max_seq_len),
                                "context/tokens_seen": float(state.tokens_seen), "context/transition_count": 0.0})
            if distributed_context is not None and getattr(distributed_context, "initialized", False):
                from ..parallel.metrics import reduce_scalar_metrics
                metrics = reduce_scalar_metrics(metrics, context=distributed_context)
            if transition_pending:
                metrics.update({f"context/{k}": float(v) for k, v in transition_event.items()
                                if k in ("old_max_seq_len", "new_max_seq_len", "tokens_seen_at_transition",
                                         "loss_before_transition")})
            if logger is not None and log_every and executed and state.optimizer_step % log_every == 0:
                logger.log(state.optimizer_step, metrics)
            if on_optimizer_step is not None:
                metrics["_alerts"] = alerts
                on_optimizer_step(metrics)
            if transition_pending and stop_on_context_transition:
                stop = True
    except BaseException:
        if moe_controller is not None and getattr(moe_controller, "window_open", False):
            moe_controller.discard()
        optimizer.zero_grad(set_to_none=True)
        raise
    allc = totals["contribs"]
    if allc:
        _, epoch_stats = combine_distributed_window_loss(allc, distributed_context)
    else:
        epoch_stats = {"loss": 0.0, "ntp_loss": 0.0, "mtp_loss": float("nan"), "ntp_tokens": 0.0, "mtp_tokens": 0.0,
                       "tokens": 0.0}
    elapsed = time.perf_counter() - started
    return {**epoch_stats, "num_batches": float(len(allc)), "optimizer_steps": float(totals["steps"]),
            "skipped_optimizer_steps": float(totals["skipped"]),
            "num_samples": _dist_sum([float(totals["samples"])], distributed_context)[0],
            "grad_norm_pre_clip": totals["pre"] / max(totals["n_norm"], 1),
            "grad_norm_post_clip": totals["post"] / max(totals["n_norm"], 1),
            "epoch_time_seconds": float(elapsed),
            "tokens_per_second": float(epoch_stats["tokens"] / max(elapsed, 1e-12)),
            "context_transition": transition_event}


# --------------------------------------------------------------------------- evaluation
@torch.no_grad()
def eval_one_epoch(model, dataloader, *, device="cpu", amp_enabled: bool = False, amp_dtype: str = "bf16",
                   max_batches: int | None = None, use_mtp: bool | None = None, ema=None, use_ema: bool = False,
                   distributed_context=None) -> dict:
    if max_batches is not None and max_batches < 0:
        raise ValueError("max_batches must be None or non-negative")
    if use_ema and ema is None:
        raise ValueError("use_ema=True requires an EMA instance")
    device = torch.device(device)
    was_training = model.training
    model.to(device).eval()
    contribs = []
    samples = 0

    def run():
        nonlocal samples
        for i, rb in enumerate(dataloader):
            if max_batches is not None and i >= max_batches:
                break
            b = move_batch_to_device(normalize_lm_batch(rb), device)
            samples += int(b["input_ids"].shape[0])
            with autocast_ctx(device, enabled=amp_enabled, amp_dtype=amp_dtype):
                out = call_model(model, b, use_mtp=use_mtp)
            contribs.append(extract_loss_contribution(out, b))

    try:
        if use_ema:
            with ema.average_parameters(model):
                run()
        else:
            run()
    finally:
        model.train(was_training)
    if not contribs:
        return {"loss": 0.0, "ntp_loss": 0.0, "mtp_loss": float("nan"), "perplexity": 1.0, "ntp_perplexity": 1.0,
                "ntp_tokens": 0.0, "mtp_tokens": 0.0, "tokens": 0.0, "num_batches": 0.0, "num_samples": 0.0,
                "used_ema": float(use_ema)}
    _, stats = combine_distributed_window_loss(contribs, distributed_context)
    samples = int(_dist_sum([float(samples)], distributed_context)[0])
    ppl = math.exp(min(stats["ntp_loss"], 50.0))
    return {**stats, "perplexity": ppl, "ntp_perplexity": ppl, "num_batches": float(len(contribs)),
            "num_samples": float(samples), "used_ema": float(use_ema)}


# --------------------------------------------------------------------------- previews
def decode_token_ids(ids, *, tokenizer=None, id_to_text=None) -> str:
    values = ids.detach().cpu().tolist() if torch.is_tensor(ids) else list(ids)
    if id_to_text is not None:
        return id_to_text(values)
    if tokenizer is not None and hasattr(tokenizer, "decode"):
        return tokenizer.decode(values)
    return " ".join(str(v) for v in values)


def _last_valid_index(batch: dict, i: int) -> int:
    mask = batch.get("attention_mask")
    if mask is None:
        return int(batch["input_ids"].shape[1]) - 1
    valid = torch.nonzero(mask[i], as_tuple=False).flatten()
    if valid.numel() == 0:
        raise ValueError("preview sample has no valid tokens")
    return int(valid[-1].item())


@torch.no_grad()
def next_token_preview(model, raw_batch, *, device="cpu", amp_enabled: bool = False, amp_dtype: str = "bf16",
                       use_mtp: bool | None = None, sample_index: int = 0, max_tokens: int = 32, tokenizer=None,
                       id_to_text=None) -> dict:
    """Teacher-forced argmax predictions over the last ``max_tokens`` positions of one sample."""
    device = torch.device(device)
    batch = move_batch_to_device(normalize_lm_batch(raw_batch), device)
    if not 0 <= sample_index < int(batch["input_ids"].shape[0]):
        raise IndexError("preview sample_index is outside the batch")
    was = model.training
    model.eval()
    try:
        with autocast_ctx(device, enabled=amp_enabled, amp_dtype=amp_dtype):
            out = call_model(model, batch, use_mtp=use_mtp)
        logits = out["logits"] if isinstance(out, dict) else getattr(out, "logits", None)
        if logits is None:
            raise ValueError("model output must contain logits for preview")
        pred = logits.argmax(-1)
        last = _last_valid_index(batch, sample_index)
        start = max(0, last + 1 - max_tokens)
        labels = batch.get("labels")
        inp = batch["input_ids"][sample_index, start:last + 1]
        pr = pred[sample_index, start:last + 1]
        rf = None if not torch.is_tensor(labels) else labels[sample_index, start:last + 1]
        dec = dict(tokenizer=tokenizer, id_to_text=id_to_text)
        return {"sample_index": int(sample_index), "position": last, "input_ids": inp.cpu().tolist(),
                "predicted_ids": pr.cpu().tolist(), "reference_ids": None if rf is None else rf.cpu().tolist(),
                "next_token_id": int(pred[sample_index, last]),
                "reference_next_token_id": None if rf is None else int(labels[sample_index, last]),
                "context": decode_token_ids(inp, **dec), "prediction": decode_token_ids(pr, **dec),
                "reference": None if rf is None else decode_token_ids(rf, **dec)}
    finally:
        model.train(was)


def print_next_token_preview(preview: dict, *, title: str = "Next-token preview") -> None:
    print(f"\n  {title} (sample {preview['sample_index']}, position {preview['position']})")
    print(f"    context    : {preview['context']}")
    print(f"    prediction : {preview['prediction']}")
    if preview.get("reference") is not None:
        print(f"    reference  : {preview['reference']}")
    print(f"    next token : {preview['next_token_id']} (reference {preview['reference_next_token_id']})")


__all__ = ["normalize_lm_batch", "move_batch_to_device", "filter_forward_kwargs", "call_model", "autocast_ctx",
           "global_grad_norm", "train_one_epoch", "eval_one_epoch", "decode_token_ids", "next_token_preview",
           "print_next_token_preview"]
