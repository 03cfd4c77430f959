"""Process-group lifecycle, rank-local runtime state and the DP x TP x EP mesh.

Parity: ``training/distributed/environment.py:32-184`` and ``mesh.py:14-110`` (reference):
``env://`` initialisation (backend ``auto`` = NCCL with CUDA, else Gloo), one owned process
group destroyed once, rank = ``(dp * TP + tp) * EP + ep`` and every axis subgroup created in
identical order on all ranks.

Additions: with ``expert_parallel.overlay_tensor_parallel`` the expert group IS the tensor
group (rank = ``dp * TP + tp``), so EP and TP share ranks; a short default process-group
timeout is applied when the configuration leaves the reference's 30 minutes and
``KIMI_PG_TIMEOUT`` is set (failure detection in tests); NCCL's device id is bound at init so
communicators are created eagerly on the right GPU.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, replace
from datetime import timedelta
from itertools import product
from typing import Mapping

import torch
import torch.distributed as dist

from .config import DistributedConfig


def _env_int(env: Mapping[str, str], name: str, default: int) -> int:
    raw = env.get(name)
    if raw is None:
        return default
    try:
        v = int(raw)
    except ValueError as exc:
        raise ValueError(f"{name} must be an integer, got {raw!r}") from exc
    if v < 0:
        raise ValueError(f"{name} must be non-negative")
    return v


@dataclass(frozen=True)
class DistributedEnvironment:
    rank: int
    world_size: int
    local_rank: int
    local_world_size: int

    @classmethod
    def from_environ(cls, environment: Mapping[str, str] | None = None) -> "DistributedEnvironment":
        env = os.environ if environment is None else environment
        world = _env_int(env, "WORLD_SIZE", 1)
        if world <= 0:
            raise ValueError("WORLD_SIZE must be positive")
        lws = _env_int(env, "LOCAL_WORLD_SIZE", world)
        if lws <= 0:
            raise ValueError("LOCAL_WORLD_SIZE must be positive")
        out = cls(_env_int(env, "RANK", 0), world, _env_int(env, "LOCAL_RANK", 0), lws)
        if out.rank >= out.world_size:
            raise ValueError("RANK must be smaller than WORLD_SIZE")
        if out.local_rank >= out.local_world_size:
            raise ValueError("LOCAL_RANK must be smaller than LOCAL_WORLD_SIZE")
        return out


@dataclass(frozen=True)
class DistributedContext:
    initialized: bool
    owns_process_group: bool
    backend: str
    global_rank: int
    local_rank: int
    world_size: int
    local_world_size: int
    device: torch.device
    mesh: object | None = None
    dp_group: object | None = None
    tp_group: object | None = None
    ep_group: object | None = None
    dp_rank: int = 0
    tp_rank: int = 0
    ep_rank: int = 0
    dp_size: int = 1
    tp_size: int = 1
    ep_size: int = 1
    ep_overlays_tp: bool = False
    sharded_grads: bool = False

    @property
    def data_replica_groups(self) -> tuple:
        """``(group, size)`` of the axes whose ranks see different data: DP, and EP unless EP
        overlays TP (then the EP ranks share one token stream)."""
        axes = [(self.dp_group, self.dp_size)]
        if not self.ep_overlays_tp:
            axes.append((self.ep_group, self.ep_size))
        return tuple(axes)

    @property
    def data_replicas(self) -> int:
        n = 1
        for _, size in self.data_replica_groups:
            n *= size
        return n

    @property
    def is_global_zero(self) -> bool:
        return self.global_rank == 0

    @property
    def should_log(self) -> bool:
        return self.is_global_zero

    def barrier(self) -> None:
        if self.initialized and self.world_size > 1:
            if self.backend == "nccl":
                dist.barrier(device_ids=[self.device.index])
            else:
                dist.barrier()

    def close(self) -> None:
        if self.owns_process_group and dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


def resolve_backend(config: DistributedConfig) -> str:
    if config.backend != "auto":
        if config.backend == "nccl" and not torch.cuda.is_available():
            raise RuntimeError("NCCL requires CUDA")
        return config.backend
    return "nccl" if torch.cuda.is_available() else "gloo"


def initialize_distributed(config: DistributedConfig, *, environment: Mapping[str, str] | None = None
                           ) -> DistributedContext:
    """Initialise ``env://`` once and return the context (not yet split into axis groups)."""
    env = DistributedEnvironment.from_environ(environment)
    if not config.enabled:
        if env.world_size != 1:
            raise RuntimeError("torchrun detected WORLD_SIZE>1 but distributed.enabled=false")
        dev = torch.device("cuda", 0) if torch.cuda.is_available() else torch.device("cpu")
        return DistributedContext(False, False, "none", 0, 0, 1, 1, dev)
    if env.world_size != config.logical_world_size:
        raise RuntimeError(f"WORLD_SIZE={env.world_size} does not match configured DP x TP x EP="
                           f"{config.logical_world_size}")
    backend = resolve_backend(config)
    device = torch.device("cuda", env.local_rank) if backend == "nccl" else torch.device("cpu")
    if device.type == "cuda":
        torch.cuda.set_device(device)
    owned = not dist.is_initialized()
    if owned:
        timeout = int(os.environ.get("KIMI_PG_TIMEOUT", config.timeout_seconds))
        kw = dict(backend=backend, init_method="env://", rank=env.rank, world_size=env.world_size,
                  timeout=timedelta(seconds=timeout))
        if device.type == "cuda":
            kw["device_id"] = device
        dist.init_process_group(**kw)
    elif dist.get_world_size() != env.world_size or dist.get_rank() != env.rank:
        raise RuntimeError("existing process group disagrees with torchrun env")
    return DistributedContext(True, owned, backend, env.rank, env.local_rank, env.world_size, env.local_world_size,
                              device, dp_size=config.data_parallel.size, tp_size=config.tensor_parallel.size,
                              ep_size=config.expert_parallel.size,
                              ep_overlays_tp=config.expert_parallel.overlay_tensor_parallel,
                              sharded_grads=config.data_parallel.mode == "fsdp")


def with_topology(context: DistributedContext, **updates) -> DistributedContext:
    return replace(context, **updates)


# --------------------------------------------------------------------------- mesh
def rank_from_coordinates(dp_rank: int, tp_rank: int, ep_rank: int, *, tp_size: int, ep_size: int) -> int:
    return (dp_rank * tp_size + tp_rank) * ep_size + ep_rank


def coordinates_from_rank(rank: int, *, tp_size: int, ep_size: int) -> tuple:
    dp, rem = divmod(rank, tp_size * ep_size)
    tp, ep = divmod(rem, ep_size)
    return dp, tp, ep


def axis_rank_lists(dp_size: int, tp_size: int, ep_size: int, *, overlay: bool = False) -> tuple:
    """Rank lists of every DP, TP and EP group (each list of groups in a fixed global order)."""
    if overlay:
        # EP == TP on the same ranks: rank = dp * TP + tp
        dp_groups = [[dp * tp_size + t for dp in range(dp_size)] for t in range(tp_size)]
        tp_groups = [[dp * tp_size + t for t in range(tp_size)] for dp in range(dp_size)]
        return dp_groups, tp_groups, [list(g) for g in tp_groups]
    r = lambda d, t, e: rank_from_coordinates(d, t, e, tp_size=tp_size, ep_size=ep_size)  # noqa: E731
    dp_groups = [[r(d, t, e) for d in range(dp_size)] for t, e in product(range(tp_size), range(ep_size))]
    tp_groups = [[r(d, t, e) for t in range(tp_size)] for d, e in product(range(dp_size), range(ep_size))]
    ep_groups = [[r(d, t, e) for e in range(ep_size)] for d, t in product(range(dp_size), range(tp_size))]
    return dp_groups, tp_groups, ep_groups


def build_device_mesh(context: DistributedContext, config: DistributedConfig) -> DistributedContext:
    """Create every axis subgroup in identical order on all ranks; attach this rank's."""
    if not context.initialized:
        return context
    dp, tp, ep = config.data_parallel.size, config.tensor_parallel.size, config.expert_parallel.size
    overlay = config.expert_parallel.overlay_tensor_parallel
    lists = axis_rank_lists(dp, tp, ep, overlay=overlay)
    chosen = [None, None, None]
    coords = [0, 0, 0]
    made = {}
    for axis, groups in enumerate(lists):
        for ranks in groups:
            key = tuple(ranks)
            if key not in made:
                made[key] = None if len(ranks) == 1 else dist.new_group(ranks=list(ranks))
            if context.global_rank in ranks:
                chosen[axis] = made[key]
                coords[axis] = ranks.index(context.global_rank)
    mesh = None
    try:
        from torch.distributed.device_mesh import DeviceMesh
        shape = (dp, tp) if overlay else (dp, tp, ep)
        names = ("dp", "tp") if overlay else ("dp", "tp", "ep")
        mesh = DeviceMesh(context.device.type, torch.arange(context.world_size).reshape(shape), mesh_dim_names=names,
                          _init_backend=False)
    except (ImportError, TypeError, RuntimeError):
        mesh = None
    return with_topology(context, mesh=mesh, dp_group=chosen[0], tp_group=chosen[1], ep_group=chosen[2],
                         dp_rank=coords[0], tp_rank=coords[1], ep_rank=coords[2])


def setup_distributed(config: DistributedConfig, *, environment=None) -> DistributedContext:
    """``initialize_distributed`` + ``build_device_mesh``."""
    return build_device_mesh(initialize_distributed(config, environment=environment), config)


__all__ = ["DistributedEnvironment", "DistributedContext", "initialize_distributed", "with_topology",
           "resolve_backend", "rank_from_coordinates", "coordinates_from_rank", "axis_rank_lists",
           "build_device_mesh", "setup_distributed"]
