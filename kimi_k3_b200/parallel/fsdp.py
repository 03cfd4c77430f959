"""Fully sharded data parallelism (parameters, gradients and optimizer state) for Kimi K3.

Parameters are sharded along their first dimension over the data-parallel group with
``torch.distributed``'s FSDP2 (``fully_shard``), one unit per token mixer (KDA / MLA) and per FFN /
MoE of every hybrid layer (the ``kimi_block`` policy) or per module holding at least
``min_num_params`` parameters, plus the root (embeddings, norms, depth mixers, heads).
Before a unit runs, its parameters are all-gathered (prefetched for the next unit, overlapping the
current one's kernels); after it, they are freed again (``full_shard``) or kept until backward
(``shard_grad_op``).  Gradients are reduce-scattered in fp32, so each rank ends a step holding
1/N of every parameter, gradient and optimizer-state tensor.

Compute is unchanged: the unsharded parameters are ordinary tensors while a unit runs, so every
projection, attention and MoE kernel of this package is used as in the single-GPU step.

Optimizers on the shards:
  * AdamW is elementwise and runs on the local shards directly.
  * Muon needs whole matrices for Newton-Schulz: momentum is kept per shard, the momentum-updated
    matrix is all-gathered, orthogonalised, and each rank applies its own rows of the update
    (:meth:`kimi_k3_b200.train.optimizer.KimiMuon.step` handles DTensor parameters that way).
  * QK-Clip scales of the local batch are MAX-reduced over the data-parallel group, so every
    shard of a query / key matrix is scaled by the same factor.

Reference: ``training/distributed/wrapping.py:90-127`` (PyTorch FSDP FULL_SHARD with a
``kimi_block`` auto-wrap policy).
"""
from __future__ import annotations

import torch
import torch.nn as nn


def _units(model: nn.Module, policy: str, min_num_params: int):
    from ..models.backbone import HybridAttentionLayer
    if policy == "kimi_block":
        # a layer's token mixer and its FFN / MoE: their parameters are read only inside their own
        # forward (the layer's depth mixers are called by the backbone between layers and stay with
        # the root unit, whose parameters are gathered for the whole step)
        units = []
        for m in model.modules():
            if isinstance(m, HybridAttentionLayer):
                units += [u for u in (m.attention, m.ffn) if u is not None]
        return units
    if policy == "size_based":
        picked, covered = [], set()
        for m in sorted(model.modules(), key=lambda mod: sum(p.numel() for p in mod.parameters())):
            own = [p for p in m.parameters() if id(p) not in covered]
            if m is not model and sum(p.numel() for p in own) >= min_num_params and own:
                picked.append(m)
                covered.update(id(p) for p in m.parameters())
        return picked
    return []


def _register_output_types() -> None:
    """FSDP2 re-gathers a unit's parameters for backward through hooks on the tensors its forward
    returns; the token mixers and MoE return dataclasses, so those become pytree nodes (the hooks
    then reach the hidden states inside them)."""
    import dataclasses
    from torch.utils import _pytree as pytree
    from ..models.kda import KDAOutput
    from ..models.mla import GatedMLAOutput
    from ..models.moe import StableLatentMoEOutput
    from ..models.primitives import AttentionModuleOutput
    for cls in (KDAOutput, GatedMLAOutput, StableLatentMoEOutput, AttentionModuleOutput):
        if cls in pytree.SUPPORTED_NODES:
            continue
        names = [f.name for f in dataclasses.fields(cls)]
        pytree.register_pytree_node(
            cls, lambda obj, names=names: ([getattr(obj, n) for n in names], None),
            lambda children, _ctx, cls=cls: cls(*children))


def shard_kimi_model(model: nn.Module, config, context) -> nn.Module:
    """Shard ``model`` in place over ``context.dp_group``; returns it (same object)."""
    _register_output_types()
    from torch.distributed.device_mesh import DeviceMesh
    from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard
    fs = config.fsdp
    if fs.sharding_strategy == "no_shard":
        raise ValueError("fsdp.sharding_strategy=no_shard is data_parallel.mode=ddp")
    if fs.cpu_offload:
        raise ValueError("fsdp.cpu_offload is not supported: the kernels read device-resident weights")
    dev_type = context.device.type if context.device is not None else "cpu"
    mesh = DeviceMesh.from_group(context.dp_group, dev_type)
    if context.tp_size > 1 or (config.expert_parallel.enabled and config.expert_parallel.size > 1):
        raise ValueError("data_parallel.mode=fsdp shards over pure data parallelism; combine tensor or expert "
                         "parallelism with data_parallel.mode=ddp")
    # Parameters are gathered in their own dtype (the kernels read fp32 norm / conv / decay parameters
    # and cast projection weights to bf16 per use); gradients are reduce-scattered in fp32 (float64
    # models keep float64).
    dtypes = {p.dtype for p in model.parameters()}
    mp = MixedPrecisionPolicy(param_dtype=None, reduce_dtype=None if torch.float64 in dtypes else torch.float32)
    reshard = fs.sharding_strategy == "full_shard"
    units = _units(model, fs.auto_wrap_policy, fs.min_num_params)
    for unit in units:
        fully_shard(unit, mesh=mesh, mp_policy=mp, reshard_after_forward=reshard)
    # the root (embeddings, tied heads, norms, depth mixers) stays gathered from forward to the end of
    # backward: its tensors are read again by the losses' backward and the MTP head
    fully_shard(model, mesh=mesh, mp_policy=mp, reshard_after_forward=False)
    if fs.forward_prefetch and len(units) > 1:
        for cur, nxt in zip(units[:-1], units[1:]):
            cur.set_modules_to_forward_prefetch([nxt])
    if fs.backward_prefetch == "backward_pre" and len(units) > 1:
        for cur, prv in zip(units[1:], units[:-1]):
            cur.set_modules_to_backward_prefetch([prv])
    model._kimi_fsdp_mesh = mesh
    return model


def reshard_all(model: nn.Module) -> None:
    """Put every sharded unit back on its shards.  The root unit keeps its gathered parameters
    registered after a forward (backward reuses them), so a parameter list or state dict read
    after an evaluation forward would otherwise hold the gathered root tensors instead of the
    DTensor shards that receive the reduce-scattered gradients.  A no-op without sharding."""
    try:
        from torch.distributed.fsdp import FSDPModule
    except ImportError:  # pragma: no cover - every supported torch has it
        return
    for m in model.modules():
        if isinstance(m, FSDPModule):
            m.reshard()


def is_sharded(p: torch.Tensor) -> bool:
    from torch.distributed.tensor import DTensor
    return isinstance(p, DTensor)


def local_shard_bytes(model: nn.Module) -> int:
    """Bytes of parameters this rank holds (its shards)."""
    total = 0
    for p in model.parameters():
        t = p.to_local() if is_sharded(p) else p
        total += t.numel() * t.element_size()
    return total


@torch.no_grad()
def sharded_grad_norm(params) -> torch.Tensor:
    """Global L2 norm of DTensor gradients (one all-reduce of the local sums of squares)."""
    import torch.distributed as dist
    sq = None
    group = None
    for p in params:
        if p.grad is None:
            continue
        g = p.grad
        if is_sharded(g):
            group = g.device_mesh.get_group()
            g = g.to_local()
        s = g.float().square().sum()
        sq = s if sq is None else sq + s
    if sq is None:
        return torch.zeros(())
    if group is not None and dist.get_world_size(group) > 1:
        dist.all_reduce(sq, group=group)
    return sq.sqrt()


@torch.no_grad()
def clip_sharded_gradients(params, max_norm: float | None) -> torch.Tensor:
    total = sharded_grad_norm(params)
    if max_norm is not None:
        coef = (max_norm / (total + 1e-6)).clamp(max=1.0)
        for p in params:
            if p.grad is not None:
                (p.grad.to_local() if is_sharded(p.grad) else p.grad).mul_(coef)
    return total


__all__ = ["shard_kimi_model", "is_sharded", "local_shard_bytes", "sharded_grad_norm", "clip_sharded_gradients"]
