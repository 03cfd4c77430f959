"""Strict distributed configuration (the ``distributed:`` section of training/inference YAML).

Parity: ``training/distributed/config.py:1-254`` (reference): the same nested sections, field
names, defaults and validation, so a reference YAML loads unchanged. Additions for this
framework, all off by default:

* ``expert_parallel.overlay_tensor_parallel`` - EP and TP use the SAME rank group (EP = TP),
  so e.g. 8 GPUs run EP8 experts and TP8-sharded attention at once (the reference needs
  ``world = DP * TP * EP``);
* ``data_parallel.bucket_mb`` - gradient all-reduce bucket size of the native reducer;
* ``kernels.fused_collectives`` - use the fused peer-memory kernels where they exist.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any, Literal

from ..config.yaml_utils import ConfigError, dataclass_kwargs


@dataclass(frozen=True)
class DataParallelConfig:
    mode: Literal["none", "ddp", "fsdp"] = "none"
    size: int = 1
    find_unused_parameters: bool = False
    gradient_as_bucket_view: bool = True
    static_graph: bool = False
    bucket_mb: float = 64.0

    def __post_init__(self) -> None:
        if self.mode not in ("none", "ddp", "fsdp"):
            raise ValueError("data_parallel.mode must be none, ddp or fsdp")
        if self.size <= 0:
            raise ValueError("data_parallel.size must be positive")
        if self.mode == "none" and self.size != 1:
            raise ValueError("data_parallel.size must be 1 when mode=none")
        if self.mode != "none" and self.size == 1:
            raise ValueError("data_parallel.size must be > 1 when data parallelism is enabled")
        if self.bucket_mb <= 0:
            raise ValueError("data_parallel.bucket_mb must be positive")


@dataclass(frozen=True)
class FSDPConfig:
    sharding_strategy: Literal["full_shard", "shard_grad_op", "no_shard"] = "full_shard"
    auto_wrap_policy: Literal["kimi_block", "size_based", "none"] = "kimi_block"
    min_num_params: int = 0
    mixed_precision: Literal["inherit", "fp32", "bf16", "fp16"] = "inherit"
    cpu_offload: bool = False
    use_orig_params: bool = True
    forward_prefetch: bool = False
    backward_prefetch: Literal["backward_pre", "backward_post", "none"] = "backward_pre"
    limit_all_gathers: bool = True
    state_dict_type: Literal["sharded", "rank0_full"] = "sharded"

    def __post_init__(self) -> None:
        if self.min_num_params < 0:
            raise ValueError("fsdp.min_num_params must be non-negative")


@dataclass(frozen=True)
class TensorParallelConfig:
    enabled: bool = False
    size: int = 1
    shard_embeddings: bool = True
    shard_lm_head: bool = True
    sequence_parallel_norms: bool = False
    shard_kda_heads: bool = True
    shard_mla_heads: bool = True
    shard_moe_latent_projections: bool = False
    mla_cache_layout: Literal["replicated", "latent_sharded"] = "replicated"
    # Run each attention shard's output projection and its all-reduce as one kernel (tcgen05 GEMM
    # + NVLink reduction over symmetric memory) on CUDA; CPU ranks keep the separate all-reduce.
    fused_output_reduce: bool = False

    def __post_init__(self) -> None:
        if self.size <= 0:
            raise ValueError("tensor_parallel.size must be positive")
        if self.enabled != (self.size > 1):
            raise ValueError("tensor_parallel.enabled must be true exactly when size > 1")
        if self.mla_cache_layout == "latent_sharded":
            raise ValueError("latent-sharded MLA cache is reserved for a later phase; use mla_cache_layout=replicated")
        if self.shard_embeddings != self.shard_lm_head:
            raise ValueError("tied Kimi vocabulary weights require embedding and LM-head sharding to be enabled or "
                             "disabled together")


@dataclass(frozen=True)
class ExpertParallelConfig:
    enabled: bool = False
    size: int = 1
    # "all_to_all": NCCL all-to-alls (the reference's exchange); "nvlink_fused": device-initiated
    # dispatch into the owners' grouped expert inputs and the combine fused into the expert
    # down-GEMM epilogue, over symmetric memory (CUDA ranks of one NVLink domain)
    dispatch: Literal["all_to_all", "nvlink_fused"] = "all_to_all"
    expert_placement: Literal["contiguous"] = "contiguous"
    shared_experts: Literal["replicated"] = "replicated"
    drop_tokens: bool = False
    capacity_factor: float | None = None
    overlay_tensor_parallel: bool = False

    def __post_init__(self) -> None:
        if self.size <= 0:
            raise ValueError("expert_parallel.size must be positive")
        if self.enabled != (self.size > 1):
            raise ValueError("expert_parallel.enabled must be true exactly when size > 1")
        if self.drop_tokens:
            raise ValueError("Kimi expert parallelism never drops routed tokens")
        if self.capacity_factor is not None:
            raise ValueError("capacity_factor is unsupported by the no-drop baseline")


@dataclass(frozen=True)
class InactiveParallelConfig:
    enabled: bool = False
    size: int = 1

    def __post_init__(self) -> None:
        if self.enabled or self.size != 1:
            raise ValueError("pipeline/context parallelism is validation metadata only and must remain disabled with "
                             "size=1")


@dataclass(frozen=True)
class DistributedCheckpointConfig:
    format: Literal["distributed", "rank0_full"] = "distributed"
    async_save: bool = False
    save_rng_per_rank: bool = True

    def __post_init__(self) -> None:
        if self.async_save:
            raise ValueError("asynchronous distributed saves are not implemented")


@dataclass(frozen=True)
class DistributedDiagnosticsConfig:
    aggregate_across_data_parallel: bool = True
    log_rank: int = 0
    per_rank_debug: bool = False

    def __post_init__(self) -> None:
        if self.log_rank < 0:
            raise ValueError("distributed.diagnostics.log_rank must be >= 0")


@dataclass(frozen=True)
class DistributedKernelsConfig:
    fused_collectives: bool = True
    nvls: Literal["auto", "off"] = "auto"


@dataclass(frozen=True)
class DistributedConfig:
    enabled: bool = False
    backend: Literal["auto", "gloo", "nccl"] = "auto"
    init_method: Literal["env"] = "env"
    timeout_seconds: int = 1800
    data_parallel: DataParallelConfig = field(default_factory=DataParallelConfig)
    fsdp: FSDPConfig = field(default_factory=FSDPConfig)
    tensor_parallel: TensorParallelConfig = field(default_factory=TensorParallelConfig)
    expert_parallel: ExpertParallelConfig = field(default_factory=ExpertParallelConfig)
    pipeline_parallel: InactiveParallelConfig = field(default_factory=InactiveParallelConfig)
    context_parallel: InactiveParallelConfig = field(default_factory=InactiveParallelConfig)
    checkpoint: DistributedCheckpointConfig = field(default_factory=DistributedCheckpointConfig)
    diagnostics: DistributedDiagnosticsConfig = field(default_factory=DistributedDiagnosticsConfig)
    kernels: DistributedKernelsConfig = field(default_factory=DistributedKernelsConfig)

    def __post_init__(self) -> None:
        if self.timeout_seconds <= 0:
            raise ValueError("distributed.timeout_seconds must be positive")
        if self.expert_parallel.overlay_tensor_parallel and self.expert_parallel.size != self.tensor_parallel.size:
            raise ValueError("expert_parallel.overlay_tensor_parallel requires expert_parallel.size == "
                             "tensor_parallel.size")
        if not self.enabled and self.logical_world_size != 1:
            raise ValueError("distributed.enabled=false requires DP=TP=EP=1")
        if self.enabled and self.logical_world_size <= 1:
            raise ValueError("distributed.enabled=true requires at least one parallel size > 1")
        if self.diagnostics.log_rank >= self.logical_world_size:
            raise ValueError("distributed.diagnostics.log_rank must be inside world size")

    @property
    def logical_world_size(self) -> int:
        ep = 1 if self.expert_parallel.overlay_tensor_parallel else self.expert_parallel.size
        return self.data_parallel.size * self.tensor_parallel.size * ep

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


SECTIONS = {"data_parallel": DataParallelConfig, "fsdp": FSDPConfig, "tensor_parallel": TensorParallelConfig,
            "expert_parallel": ExpertParallelConfig, "pipeline_parallel": InactiveParallelConfig,
            "context_parallel": InactiveParallelConfig, "checkpoint": DistributedCheckpointConfig,
            "diagnostics": DistributedDiagnosticsConfig, "kernels": DistributedKernelsConfig}


def distributed_config_from_dict(values: dict | None) -> DistributedConfig:
    """Strict nested configuration from a YAML mapping (unknown keys are errors)."""
    root = dict(values or {})
    nested = {}
    for name, cls in SECTIONS.items():
        raw = root.pop(name, {})
        if raw is None:
            raw = {}
        if not isinstance(raw, dict):
            raise ConfigError(f"distributed.{name} must be a mapping")
        nested[name] = cls(**dataclass_kwargs(raw, cls, path=f"distributed.{name}"))
    return DistributedConfig(**dataclass_kwargs(root, DistributedConfig, path="distributed"), **nested)


__all__ = ["DataParallelConfig", "FSDPConfig", "TensorParallelConfig", "ExpertParallelConfig",
           "InactiveParallelConfig", "DistributedCheckpointConfig", "DistributedDiagnosticsConfig",
           "DistributedKernelsConfig", "DistributedConfig", "distributed_config_from_dict"]
