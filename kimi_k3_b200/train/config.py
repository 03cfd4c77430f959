"""Training configuration: the strict ``training.yaml`` schema and its typed sections.

Parity: ``training/config.py`` and ``training/yaml_config.py:22-176`` (reference):
sections ``runtime, training, loss, optimizer, scheduler, diagnostics,
context_curriculum, checkpoint, prediction, distributed``; unknown keys raise.
An optional ``kernels:`` section carries B200-only knobs so reference profiles
still parse unchanged.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from pathlib import Path

from ..config.yaml_utils import ConfigError, dataclass_kwargs, expect_mapping, load_yaml_mapping, reject_unknown_keys
from .optimizer import KimiOptimizerConfig


def _pos_opt(name, value):
    if value is not None and value <= 0:
        raise ValueError(f"{name} must be None or a positive integer")


@dataclass(frozen=True)
class TrainingConfig:
    epochs: int = 1
    gradient_accumulation_steps: int = 1
    precision: str = "bf16"
    grad_clip_norm: float | None = 1.0
    use_mtp: bool = True
    max_batches_per_epoch: int | None = None
    max_eval_batches: int | None = None
    log_every_steps: int = 10
    eval_every_epochs: int = 1
    checkpoint_every_epochs: int = 1
    prediction_every_epochs: int | None = 1
    seed: int = 1337
    deterministic: bool = False
    max_seq_len: int = 8192

    def __post_init__(self) -> None:
        if self.epochs <= 0 or self.gradient_accumulation_steps <= 0 or self.max_seq_len <= 0:
            raise ValueError("epochs, gradient_accumulation_steps and max_seq_len must be positive")
        if self.precision not in ("fp32", "bf16", "fp16"):
            raise ValueError("precision must be 'fp32', 'bf16', or 'fp16'")
        if self.grad_clip_norm is not None and self.grad_clip_norm <= 0:
            raise ValueError("grad_clip_norm must be None or positive")
        for n in ("max_batches_per_epoch", "max_eval_batches", "log_every_steps", "eval_every_epochs",
                  "checkpoint_every_epochs", "prediction_every_epochs"):
            _pos_opt(n, getattr(self, n))

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class PretrainingLossConfig:
    ignore_index: int = -100
    label_smoothing: float = 0.0
    mtp_loss_weight: float | None = None
    label_alignment: str = "causal_shift"

    def __post_init__(self) -> None:
        if self.ignore_index >= 0:
            raise ValueError("ignore_index must be negative")
        if not 0 <= self.label_smoothing < 1:
            raise ValueError("label_smoothing must be in [0, 1)")
        if self.mtp_loss_weight is not None and self.mtp_loss_weight < 0:
            raise ValueError("mtp_loss_weight must be None or non-negative")
        if self.label_alignment not in ("causal_shift", "already_aligned"):
            raise ValueError("label_alignment must be causal_shift or already_aligned")

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class OptimizerConfig:
    """Plain AdamW configuration (legacy API); the Kimi hybrid uses KimiOptimizerConfig."""
    name: str = "adamw"
    learning_rate: float = 3e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.1

    def __post_init__(self) -> None:
        if self.name != "adamw":
            raise ValueError("the basic engine supports only AdamW")
        if self.learning_rate <= 0 or self.eps <= 0 or self.weight_decay < 0:
            raise ValueError("invalid AdamW configuration")

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class SchedulerConfig:
    kind: str = "cosine"
    warmup_ratio: float | None = 0.01
    warmup_steps: int | None = None
    min_lr_ratio: float = 0.0

    def __post_init__(self) -> None:
        if self.kind != "cosine":
            raise ValueError("only the cosine scheduler is supported")
        if self.warmup_ratio is not None and self.warmup_steps is not None:
            raise ValueError("set warmup_ratio or warmup_steps, not both")
        if self.warmup_ratio is not None and not 0 <= self.warmup_ratio <= 1:
            raise ValueError("warmup_ratio must be in [0, 1]")
        if self.warmup_steps is not None and self.warmup_steps < 0:
            raise ValueError("warmup_steps must be non-negative")
        if not 0 <= self.min_lr_ratio <= 1:
            raise ValueError("min_lr_ratio must be in [0, 1]")

    def resolve_warmup_steps(self, total_steps: int) -> int:
        if total_steps <= 0:
            raise ValueError("total_steps must be positive")
        if self.warmup_steps is not None:
            return min(self.warmup_steps, total_steps)
        r = int(total_steps * (self.warmup_ratio or 0.0))
        if (self.warmup_ratio or 0.0) > 0 and total_steps > 1:
            r = max(1, r)
        return min(r, total_steps)

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class CheckpointConfig:
    output_dir: str = "checkpoints/kimi_k3"
    run_name: str = "kimi_k3"
    keep_last_n: int = 3
    save_optimizer: bool = True
    save_rng_state: bool = True
    atomic_write: bool = True
    resume_from: str | None = None

    def __post_init__(self) -> None:
        if not self.run_name or self.keep_last_n <= 0:
            raise ValueError("run_name must be set and keep_last_n positive")
        if not self.atomic_write:
            raise ValueError("atomic checkpoint writes cannot be disabled")

    def to_dict(self) -> dict:
        v = asdict(self)
        v["output_dir"] = str(self.output_dir)
        v["resume_from"] = None if self.resume_from is None else str(self.resume_from)
        return v


@dataclass(frozen=True)
class PredictionConfig:
    sample_index: int = 0
    max_tokens: int = 32

    def __post_init__(self) -> None:
        if self.sample_index < 0 or self.max_tokens <= 0:
            raise ValueError("invalid prediction configuration")

    def to_dict(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class TrainingRuntimeConfig:
    device: str = "auto"
    total_steps: int | None = None
    verbose: bool = True
    use_ema: bool = False
    ema_decay: float = 0.999
    eval_use_ema: bool = False

    def __post_init__(self) -> None:
        if not self.device:
            raise ValueError("runtime.device must not be empty")
        if self.total_steps is not None and self.total_steps <= 0:
            raise ValueError("runtime.total_steps must be None or positive")
        if not 0 < self.ema_decay < 1:
            raise ValueError("runtime.ema_decay must be in (0, 1)")
        if self.eval_use_ema and not self.use_ema:
            raise ValueError("runtime.eval_use_ema requires use_ema=true")


@dataclass(frozen=True)
class KernelsConfig:
    """B200-only switches (absent from reference profiles; all default on)."""
    native_kernels: bool = True
    fused_head_loss: bool = True
    muon_ns_dtype: str = "auto"

    def __post_init__(self) -> None:
        if self.muon_ns_dtype not in ("auto", "float32", "bfloat16"):
            raise ValueError("kernels.muon_ns_dtype must be auto, float32 or bfloat16")


@dataclass(frozen=True)
class TrainingYamlConfig:
    runtime: TrainingRuntimeConfig
    training: TrainingConfig
    loss: PretrainingLossConfig
    optimizer: KimiOptimizerConfig
    scheduler: SchedulerConfig
    diagnostics: object
    context_curriculum: object
    checkpoint: CheckpointConfig
    prediction: PredictionConfig
    distributed: object
    source_path: Path | None = None
    kernels: KernelsConfig = field(default_factory=KernelsConfig)


def _section(root, name, cls, *, required=True):
    values = expect_mapping(root, name, path="root", required=required)
    if isinstance(values.get("adamw_betas"), list):
        values["adamw_betas"] = tuple(values["adamw_betas"])
    try:
        return cls(**dataclass_kwargs(values, cls, path=name))
    except (TypeError, ValueError) as exc:
        if isinstance(exc, ConfigError):
            raise
        raise ConfigError(f"{name}: {exc}") from exc


def training_config_from_mapping(root: dict, source: Path | None = None) -> TrainingYamlConfig:
    from ..parallel.config import distributed_config_from_dict
    from .curriculum import ContextCurriculumConfig, ContextStage
    from .diagnostics import DiagnosticsConfig
    root = dict(root)
    runtime = _section(root, "runtime", TrainingRuntimeConfig, required=False)
    training = _section(root, "training", TrainingConfig)
    loss = _section(root, "loss", PretrainingLossConfig, required=False)
    optimizer = _section(root, "optimizer", KimiOptimizerConfig)
    scheduler = _section(root, "scheduler", SchedulerConfig)
    diagnostics = _section(root, "diagnostics", DiagnosticsConfig, required=False)
    cur = expect_mapping(root, "context_curriculum", path="root", required=False)
    if "stages" in cur:
        if not isinstance(cur["stages"], list):
            raise ConfigError("context_curriculum.stages must be a list")
        cur["stages"] = tuple(ContextStage(**s) if isinstance(s, dict) else s for s in cur["stages"])
    curriculum = ContextCurriculumConfig(**dataclass_kwargs(cur, ContextCurriculumConfig, path="context_curriculum"))
    checkpoint = _section(root, "checkpoint", CheckpointConfig, required=False)
    prediction = _section(root, "prediction", PredictionConfig, required=False)
    distributed = distributed_config_from_dict(expect_mapping(root, "distributed", path="root", required=False))
    kernels = _section(root, "kernels", KernelsConfig, required=False)
    reject_unknown_keys(root, path="root")
    return TrainingYamlConfig(runtime, training, loss, optimizer, scheduler, diagnostics, curriculum, checkpoint,
                              prediction, distributed, source, kernels)


def load_training_config(path: str | Path) -> TrainingYamlConfig:
    source, root = load_yaml_mapping(path)
    return training_config_from_mapping(root, source)


def validate_pipeline_compatibility(config: TrainingYamlConfig, *, model_config, data_config) -> None:
    if config.training.use_mtp and not model_config.enable_mtp:
        raise ConfigError("training.use_mtp=true but model MTP is disabled")
    if config.training.max_seq_len > data_config.max_seq_len:
        raise ConfigError(f"training.max_seq_len ({config.training.max_seq_len}) exceeds data block_size "
                          f"({data_config.max_seq_len})")
    cur = config.context_curriculum
    if cur.enabled:
        final = cur.stages[-1].max_seq_len
        if final > config.training.max_seq_len or final > data_config.max_seq_len:
            raise ConfigError("final context stage exceeds training.max_seq_len or data block_size")
    if config.distributed.data_parallel.mode == "fsdp" and config.runtime.use_ema:
        raise ConfigError("runtime.use_ema=true is unsupported with FSDP")
    from ..parallel.parallelize import validate_distributed_model_config
    validate_distributed_model_config(config.distributed, model_config)


__all__ = [
    "TrainingConfig", "PretrainingLossConfig", "OptimizerConfig", "SchedulerConfig", "CheckpointConfig",
    "PredictionConfig", "TrainingRuntimeConfig", "KernelsConfig", "TrainingYamlConfig", "load_training_config",
    "training_config_from_mapping", "validate_pipeline_compatibility",
]
