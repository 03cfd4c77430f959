"""Apply a distributed configuration to a KimiK3 model and synchronise its gradients.

Parity: ``training/distributed/parallelize.py:23-203`` and ``wrapping.py:16-196`` (reference):
topology validation before allocation (divisibility of heads, vocabulary and experts), TP
attention, vocabulary shards, EP experts, a broadcast of the initial state, gradient
synchronisation and the global gradient norm that counts every logical parameter once.

Gradient groups (data replicas of a parameter class):

* replicated parameters (norms, router, MoE projections, shared experts, unsharded
  embeddings): averaged over every rank that holds the same tensor-parallel coordinate and
  sees different data (DP x EP, or DP when EP overlays TP);
* tensor-parallel shards: averaged over DP x EP (their TP peers own other shards);
* local routed experts: averaged over DP, then divided by EP (their tokens come from every
  EP rank whose loss is already scaled by the replica count);
* TP-partial parameters (replicated inside a TP block but fed by this rank's heads or tokens
  only: KDA ``alpha_down``, MLA latent compression, MoE layers whose tokens are split over an
  overlaid EP=TP group): summed over TP and averaged over data replicas in one all-reduce.

The reference registers one un-bucketed all-reduce hook per parameter; here each class is
one bucketed reducer whose buckets launch from backward hooks (overlapped with backward).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn

from ..config.yaml_utils import ConfigError
from .config import DistributedConfig
from .data_parallel import GradientAllReducer, QBReducer
from .tensor_parallel import group_size


def validate_distributed_model_config(config: DistributedConfig, model_config) -> None:
    """Reject invalid topologies before the model or the optimizer is allocated."""
    if not config.enabled:
        return
    tp, ep = config.tensor_parallel, config.expert_parallel
    bb = model_config.backbone
    kda, mla, moe = bb.kda_config, bb.mla_config, bb.stable_latent_moe_config
    if config.checkpoint.format != "distributed":
        raise ConfigError("distributed checkpoint format rank0_full is export-only; training must use "
                          "format=distributed and call export_rank0_full_checkpoint explicitly")
    if config.data_parallel.mode == "fsdp" and config.fsdp.state_dict_type != "sharded":
        raise ConfigError("FSDP training checkpoints currently require fsdp.state_dict_type=sharded")
    if tp.enabled:
        if tp.sequence_parallel_norms:
            raise ConfigError("sequence_parallel_norms is reserved but not implemented; use false")
        need = {"model d_model": model_config.d_model, "KDA heads": kda.num_heads, "MLA heads": mla.num_heads}
        if tp.shard_embeddings:
            need["vocabulary"] = model_config.vocab_size
        bad = {k: v for k, v in need.items() if v % tp.size}
        if bad:
            raise ConfigError(f"TP size {tp.size} does not divide " + ", ".join(f"{k}={v}" for k, v in bad.items()))
        if not tp.shard_kda_heads or not tp.shard_mla_heads:
            raise ConfigError("the Kimi TP plan requires both KDA and MLA head sharding")
        if tp.shard_moe_latent_projections:
            raise ConfigError("shard_moe_latent_projections is not part of the complete-head plan; use EP to shard "
                              "routed experts")
    if ep.enabled:
        if moe.num_routed_experts % ep.size:
            raise ConfigError(f"routed experts={moe.num_routed_experts} must be divisible by EP size={ep.size}")
        if moe.top_k > moe.num_routed_experts:
            raise ConfigError("MoE top-k exceeds routed expert count")


def _tag(params, **flags) -> None:
    for p in params:
        for k, v in flags.items():
            setattr(p, k, v)


class ParallelPlan:
    """What ``parallelize_kimi_model`` did, and how to synchronise gradients afterwards."""

    def __init__(self, model, context, config: DistributedConfig, tp_layers: int, ep_layers: int, vocab):
        self.model, self.context, self.config = model, context, config
        self.tp_layers, self.ep_layers, self.vocab = tp_layers, ep_layers, vocab
        params = [p for p in model.parameters() if p.requires_grad]
        experts = [p for p in params if getattr(p, "_kimi_local_expert", False)]
        partial = [p for p in params if getattr(p, "_kimi_tp_partial", False)
                   and not getattr(p, "_kimi_local_expert", False)]
        rest = [p for p in params if not getattr(p, "_kimi_local_expert", False)
                and not getattr(p, "_kimi_tp_partial", False)]
        bucket = int(config.data_parallel.bucket_mb * (1 << 20))
        replica_group = self._replica_group(context, config)
        self.replica_group = replica_group
        self.reducers = []
        if group_size(replica_group) > 1 and rest:
            self.reducers.append(GradientAllReducer(model, replica_group, bucket, params=rest, overlap=True))
        if partial and context.initialized and context.world_size > 1:
            # sum over TP and average over the data replicas in one all-reduce over the world
            self.reducers.append(GradientAllReducer(model, dist.group.WORLD, bucket, params=partial, overlap=True,
                                                    scale=context.tp_size / context.world_size))
        # EP ranks are data replicas unless EP overlays TP (one shared token stream)
        ep = (config.expert_parallel.size if config.expert_parallel.enabled
              and not config.expert_parallel.overlay_tensor_parallel else 1)
        self.expert_scale_only = None
        if experts and group_size(context.dp_group) > 1:
            scale = 1.0 / (group_size(context.dp_group) * ep)
            self.reducers.append(GradientAllReducer(model, context.dp_group, bucket, params=experts, overlap=True,
                                                    scale=scale))
        elif experts and ep > 1:
            self.expert_scale_only = (experts, 1.0 / ep)
        self._armed = True

    @staticmethod
    def _replica_group(context, config):
        """Ranks holding the same tensor-parallel coordinate that see different data."""
        if not context.initialized:
            return None
        dp, tp = config.data_parallel.size, config.tensor_parallel.size
        ep = 1 if config.expert_parallel.overlay_tensor_parallel else config.expert_parallel.size
        if ep == 1:
            return context.dp_group
        if dp == 1:
            return context.ep_group
        # DP x EP ranks at this TP coordinate: rank = (d * TP + t) * EP + e
        groups = {}
        for t in range(tp):
            ranks = [(d * tp + t) * ep + e for d in range(dp) for e in range(ep)]
            groups[t] = dist.new_group(ranks=ranks)
        return groups[context.tp_rank]

    @property
    def armed(self) -> bool:
        return self._armed

    @armed.setter
    def armed(self, value: bool) -> None:
        self._armed = bool(value)
        for r in self.reducers:
            r.armed = self._armed

    @torch.no_grad()
    def broadcast_parameters(self) -> None:
        """Identical initial state inside every data-replica group: each reducer broadcasts its
        own parameter class over its group; buffers go over the replica group."""
        for r in self.reducers:
            r.broadcast_parameters()
        if group_size(self.replica_group) > 1:
            src = dist.get_global_rank(self.replica_group, 0)
            for b in self.model.buffers():
                dist.broadcast(b, src=src, group=self.replica_group)

    def sync_gradients(self) -> None:
        for r in self.reducers:
            r.all_reduce_gradients()
        if self.expert_scale_only is not None:
            params, scale = self.expert_scale_only
            grads = [p.grad for p in params if p.grad is not None]
            if grads:
                torch._foreach_mul_(grads, scale)

    def qb_reducer(self):
        """Outer Quantile-Balancing reducer: the data replicas (EP layers add their own group)."""
        return QBReducer(self.context.dp_group) if group_size(self.context.dp_group) > 1 else None

    @torch.no_grad()
    def grad_norm(self) -> torch.Tensor | None:
        """Global L2 norm counting each logical parameter once (device scalar, same on all ranks)."""
        params = [p for p in self.model.parameters() if p.grad is not None]
        if not params:
            return None
        dev = params[0].grad.device

        def sq(ps):
            if not ps:
                return torch.zeros((), device=dev, dtype=torch.float32)
            return torch.stack([n.float() for n in torch._foreach_norm([p.grad for p in ps], 2.0)]).square().sum()
        tp_shard = [p for p in params if getattr(p, "_kimi_tp_shard", False)]
        expert = [p for p in params if getattr(p, "_kimi_local_expert", False)]
        other = [p for p in params if not getattr(p, "_kimi_tp_shard", False)
                 and not getattr(p, "_kimi_local_expert", False)]
        s_tp, s_ep, s_rep = sq(tp_shard), sq(expert), sq(other)
        if group_size(self.context.tp_group) > 1:
            dist.all_reduce(s_tp, group=self.context.tp_group)
        if group_size(self.context.ep_group) > 1:
            dist.all_reduce(s_ep, group=self.context.ep_group)
        return (s_tp + s_ep + s_rep).sqrt()


def parallelize_kimi_model(model: nn.Module, config: DistributedConfig, context) -> ParallelPlan:
    """Shard attention heads, vocabulary and experts in place; return the gradient plan."""
    from .expert_parallel import shard_kimi_experts
    from .kimi_tp import TensorParallelKDA, TensorParallelMLA, shard_kimi_attention
    from .tensor_parallel import shard_vocabulary
    raw = model.module if hasattr(model, "module") else model
    if config.enabled:
        validate_distributed_model_config(config, raw.config)
    tp_layers = ep_layers = 0
    vocab = None
    if config.enabled and config.tensor_parallel.enabled:
        tp_layers = shard_kimi_attention(raw, group=context.tp_group, shard_kda=config.tensor_parallel.shard_kda_heads,
                                         shard_mla=config.tensor_parallel.shard_mla_heads,
                                         fused_output=config.tensor_parallel.fused_output_reduce)
        for m in raw.modules():
            if isinstance(m, (TensorParallelKDA, TensorParallelMLA)):
                _tag([p for p in m.parameters() if not getattr(p, "_kimi_tp_partial", False)], _kimi_tp_shard=True)
        if config.tensor_parallel.shard_embeddings:
            vocab = shard_vocabulary(raw, group=context.tp_group)
            _tag([raw.get_input_embeddings().weight, raw.get_output_embeddings().weight], _kimi_tp_shard=True)
    if config.enabled and config.expert_parallel.enabled:
        ep_layers = shard_kimi_experts(raw, group=context.ep_group,
                                       token_split=config.expert_parallel.overlay_tensor_parallel,
                                       fused_comm=config.expert_parallel.dispatch == "nvlink_fused")
    plan = ParallelPlan(raw, context, config, tp_layers, ep_layers, vocab)
    return plan


__all__ = ["validate_distributed_model_config", "parallelize_kimi_model", "ParallelPlan"]
