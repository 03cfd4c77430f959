"""Console reporting of training runs (reference: ``training/diagnostics/printing.py:8-229``)."""
from __future__ import annotations

import math


def fmt(value) -> str:
    if value is None:
        return "-"
    if isinstance(value, bool):
        return "yes" if value else "no"
    if isinstance(value, int):
        return f"{value:,}"
    if isinstance(value, float):
        if not math.isfinite(value):
            return str(value)
        if value != 0 and (abs(value) >= 1e5 or abs(value) < 1e-3):
            return f"{value:.3e}"
        return f"{value:.4f}"
    return str(value)


def rule(width: int = 104, ch: str = "-") -> str:
    return ch * width


SECTIONS = (
    ("Convergence", (("train/loss_total", "Total loss"), ("train/loss_ntp", "NTP loss"), ("train/loss_mtp", "MTP loss"),
                     ("train/perplexity_ntp_clipped", "NTP perplexity"), ("train/valid_ntp_tokens", "Valid NTP tokens"))),
    ("Throughput & runtime", (("train/tokens_per_second", "Tokens / second"),
                              ("train/samples_per_second", "Samples / second"), ("train/step_time_ms", "Step time (ms)"),
                              ("train/data_time_ms", "Data time (ms)"), ("train/forward_time_ms", "Forward time (ms)"),
                              ("train/backward_time_ms", "Backward time (ms)"),
                              ("train/optimizer_time_ms", "Optimizer time (ms)"),
                              ("train/memory_allocated_mb", "Memory allocated (MB)"))),
    ("Optimization health", (("learning_rate", "Learning rate"), ("lr/adamw", "AdamW LR"), ("lr/muon", "Muon LR"),
                             ("grad_norm_pre_clip", "Gradient norm pre-clip"),
                             ("grad_norm_post_clip", "Gradient norm post-clip"),
                             ("train/update_to_parameter_ratio_sampled", "Update / parameter"),
                             ("muon/ns_gain", "Muon NS gain"), ("qk_clip/events", "QK-Clip events"))),
    ("Diagnostics budget", (("train/diagnostics_time_ms", "Diagnostics time (ms)"),
                            ("train/diagnostics_time_fraction", "Diagnostics / step"),
                            ("diagnostics/persistent_gpu_bytes", "Persistent sampled bytes"),
                            ("diagnostics/scalars_emitted", "Scalars emitted"),
                            ("diagnostics/layers_sampled", "Layers sampled"),
                            ("diagnostics/degradation_level", "Degraded mode"))),
    ("Progressive context", (("context/stage_index", "Stage"), ("context/max_seq_len", "Active max sequence"),
                             ("context/tokens_seen", "Tokens seen"), ("context/transition_count", "Transitions"),
                             ("context/padding_fraction", "Padding fraction"),
                             ("context/old_max_seq_len", "Previous max sequence"),
                             ("context/new_max_seq_len", "New max sequence"))),
)


class KimiTrainingPrinter:
    def __init__(self, width: int = 104):
        self.width = width

    def title(self, text: str) -> None:
        print("\n" + rule(self.width, "="))
        print(text)
        print(rule(self.width, "="))

    def block(self, title: str, metrics: dict, rows) -> None:
        have = [(n, l) for n, l in rows if n in metrics]
        if not have:
            return
        print(f"\n  {title}")
        print("  " + rule(min(self.width - 2, 88)))
        w = max(len(l) for _, l in have)
        for n, l in have:
            print(f"  {l:<{w}} : {fmt(metrics[n]):>12}")

    def print_run_header(self, *, run_name, model, device, precision, optimizer_kind, epochs, total_steps,
                         warmup_steps, registry=None) -> None:
        self.title(f"Kimi K3 training - {run_name}")
        n = sum(p.numel() for p in model.parameters())
        print(f"  Parameters       : {n:,}")
        print(f"  Device/precision : {device} / {precision}")
        print(f"  Optimizer        : {optimizer_kind}")
        print(f"  Schedule         : epochs={epochs} - total_steps={total_steps} - warmup_steps={warmup_steps}")
        if registry is not None and hasattr(registry, "to_dict"):
            fams = {}
            for s in registry.specs:
                fams[s.optimizer_family] = fams.get(s.optimizer_family, 0) + s.parameter.numel()
            tot = max(sum(fams.values()), 1)
            print("  Parameter map    : " + " - ".join(f"{k}={100 * v / tot:.1f}%" for k, v in sorted(fams.items())))
        print(rule(self.width))

    def print_step(self, step: int, metrics: dict, alerts=()) -> None:
        self.title(f"Optimizer step {step:06d}")
        for title, rows in SECTIONS:
            self.block(title, metrics, rows)
        arch = [(n, n) for n in sorted(metrics) if n.split("/", 1)[0] in ("attnres", "kda", "mla", "moe", "mtp")
                and "/layer_" not in n]
        self.block("Architecture", metrics, arch[:24])
        if alerts:
            print("\n  Alerts")
            for a in alerts:
                print(f"  [{a.severity}] {a.code}: {a.message} ({a.metric_name}={fmt(a.observed_value)})")

    def print_epoch_summary(self, *, epoch, state, train_stats, eval_stats=None, checkpoint=None) -> None:
        self.title(f"Epoch {epoch} summary")
        print(f"  Optimizer steps  : {state.optimizer_step:,}   tokens seen: {state.tokens_seen:,}")
        print(f"  Train loss       : {fmt(train_stats.get('loss'))}   tokens/s: {fmt(train_stats.get('tokens_per_second'))}")
        if eval_stats is not None:
            print(f"  Eval loss        : {fmt(eval_stats.get('loss'))}   perplexity: {fmt(eval_stats.get('perplexity'))}")
        if checkpoint is not None:
            print(f"  Checkpoint       : {checkpoint}")


def print_topology(context, *, log_rank: int = 0, per_rank_debug: bool = False, wrapper_mode: str = "none",
                   checkpoint_format: str = "distributed", global_batch_size: int = 0) -> None:
    if context.global_rank != log_rank and not per_rank_debug:
        return
    print(f"  Topology: world={context.world_size} dp={context.dp_size} tp={context.tp_size} ep={context.ep_size}"
          f"{' (ep overlays tp)' if getattr(context, 'ep_overlays_tp', False) else ''} backend={context.backend} "
          f"data-parallel={wrapper_mode} checkpoint={checkpoint_format} global batch={global_batch_size}")


__all__ = ["KimiTrainingPrinter", "print_topology", "fmt"]
