"""Complete-head tensor parallelism for KDA and gated MLA.

Parity: ``training/distributed/kimi_tensor_parallel.py:127-586`` (reference): each TP rank
owns whole heads. KDA: q, k, v, beta, alpha_up and the output gate are column-sharded by
head; the short convolutions, ``A_log``, the head norm and ``b_alpha`` are sliced per head;
``alpha_down`` is replicated (its gradient is summed over the group); the output projection is
row-parallel. MLA: query, key_up, value_up and the gate are column-sharded; the latent
compression is replicated (gradient summed) so the latent cache is identical on every rank;
the output projection is row-parallel.

Design: instead of re-implementing the layers, each wrapper holds an ordinary
``KimiDeltaAttention`` / ``GatedMLA`` built for the LOCAL head count (so every fused sm_100a
kernel, the decode paths and the caches are reused unchanged) and surrounds it with the two
collectives of a Megatron block: the copy-to-region on the input and the all-reduce of the
row-parallel output.
"""
from __future__ import annotations

import copy

import torch
import torch.nn as nn

from ..models.kda import KimiDeltaAttention
from ..models.mla import GatedMLA
from .tensor_parallel import (copy_to_tensor_parallel_region, group_rank, group_size,
                              reduce_from_tensor_parallel_region)


def local_head_config(config, heads: int):
    """A copy of a KDA / MLA config with ``num_heads`` set to the local head count. The
    canonical ``d_model == num_heads * value_dim`` check does not apply to a shard, so the copy
    is made without re-running the dataclass validation."""
    local = copy.copy(config)
    object.__setattr__(local, "num_heads", int(heads))
    return local


def head_slice(num_heads: int, group) -> tuple:
    size, rank = group_size(group), group_rank(group)
    if num_heads % size:
        raise ValueError(f"num_heads={num_heads} is not divisible by tensor-parallel size {size}")
    per = num_heads // size
    return rank * per, (rank + 1) * per


def mark_tp_partial(param: nn.Parameter) -> None:
    """A parameter replicated over the TP group whose local gradient only covers this rank's
    heads (or tokens): the gradient plan SUMS it over TP (and averages over data replicas)."""
    param._kimi_tp_partial = True


@torch.no_grad()
def _copy(dst: torch.Tensor, src: torch.Tensor) -> None:
    if dst.shape != src.shape:
        raise ValueError(f"shard shape {tuple(src.shape)} does not match local parameter {tuple(dst.shape)}")
    dst.copy_(src)


def _tag_shards(inner: nn.Module, shard_dims: dict, group) -> None:
    """Record on each sharded parameter the dimension it is split along and the group that holds
    the other pieces: optimizers that need whole matrices (Muon) gather over that group."""
    params = dict(inner.named_parameters())
    for name, dim in shard_dims.items():
        if dim is not None and name in params:
            params[name]._kimi_tp_dim = dim
            params[name]._kimi_tp_group = group


def _install_fused_output(inner: nn.Module, group, enabled: bool) -> bool:
    """Swap the shard's output projection for the fused GEMM + all-reduce (one tcgen05 kernel
    over symmetric memory, ``parallel/symmetric.py``); the wrapper then skips its own reduce."""
    if not enabled:
        return False
    from .symmetric import FusedRowParallelOutput
    gate = inner.output_gate
    gate.output_proj = FusedRowParallelOutput(gate.output_proj, group)
    return True


class TensorParallelKDA(nn.Module):
    """KDA with complete recurrent heads per TP rank (local state ``[B, H/TP, K, V]``)."""

    def __init__(self, module: KimiDeltaAttention, *, group=None, fused_output: bool = False):
        super().__init__()
        c = module.config
        if c.output_bias or c.projection_bias or c.beta_bias or c.output_gate_bias or c.short_conv_bias:
            raise ValueError("tensor-parallel KDA supports bias-free projections")
        self.group = group
        s, e = head_slice(c.num_heads, group)
        self.head_start, self.head_end, self.num_heads = s, e, e - s
        self.config = c
        self.inner = KimiDeltaAttention(local_head_config(c, e - s)).to(device=module.projections.q_proj.weight.device,
                                                                        dtype=module.projections.q_proj.weight.dtype)
        kd, vd = c.key_head_dim, c.value_head_dim
        src, dst = module.projections, self.inner.projections
        _copy(dst.q_proj.weight, src.q_proj.weight[s * kd:e * kd])
        _copy(dst.k_proj.weight, src.k_proj.weight[s * kd:e * kd])
        _copy(dst.v_proj.weight, src.v_proj.weight[s * vd:e * vd])
        _copy(dst.q_conv.weight, src.q_conv.weight[s * kd:e * kd])
        _copy(dst.k_conv.weight, src.k_conv.weight[s * kd:e * kd])
        _copy(dst.v_conv.weight, src.v_conv.weight[s * vd:e * vd])
        _copy(dst.beta_proj.weight, src.beta_proj.weight[s:e])
        _copy(dst.alpha_down.weight, src.alpha_down.weight)
        _copy(dst.alpha_up.weight, src.alpha_up.weight[s * kd:e * kd])
        _copy(dst.b_alpha, src.b_alpha[s:e])
        _copy(self.inner.decay.A_log, module.decay.A_log[s:e])
        if module.output_norm.weight is not None:
            w = module.output_norm.weight
            _copy(self.inner.output_norm.weight, w[s:e] if module.output_norm.per_head_affine else w)
        og_src, og_dst = module.output_gate, self.inner.output_gate
        _copy(og_dst.gate_proj.weight, og_src.gate_proj.weight[s * vd:e * vd])
        _copy(og_dst.output_proj.weight, og_src.output_proj.weight[:, s * vd:e * vd])
        mark_tp_partial(dst.alpha_down.weight)
        if module.output_norm.weight is not None and not module.output_norm.per_head_affine:
            mark_tp_partial(self.inner.output_norm.weight)
        # dimension along which each inner parameter is a shard of the full one (None: replicated)
        self.shard_dims = {"projections.q_proj.weight": 0, "projections.k_proj.weight": 0,
                           "projections.v_proj.weight": 0, "projections.q_conv.weight": 0,
                           "projections.k_conv.weight": 0, "projections.v_conv.weight": 0,
                           "projections.beta_proj.weight": 0, "projections.alpha_down.weight": None,
                           "projections.alpha_up.weight": 0, "projections.b_alpha": 0, "decay.A_log": 0,
                           "output_norm.weight": 0 if module.output_norm.per_head_affine else None,
                           "output_gate.gate_proj.weight": 0, "output_gate.output_proj.weight": 1}
        _tag_shards(self.inner, self.shard_dims, group)
        self.fused_output = _install_fused_output(self.inner, group, fused_output)

    def forward(self, hidden_states, attention_mask=None, state=None, mode="chunkwise", output_final_state=False,
                output_diagnostics=False):
        x = copy_to_tensor_parallel_region(hidden_states, self.group)
        out = self.inner(x, attention_mask=attention_mask, state=state, mode=mode,
                         output_final_state=output_final_state, output_diagnostics=output_diagnostics)
        if not self.fused_output:
            out.hidden_states = reduce_from_tensor_parallel_region(out.hidden_states, self.group)
        return out


class TensorParallelMLA(nn.Module):
    """Gated MLA with complete heads per TP rank and a replicated latent cache."""

    def __init__(self, module: GatedMLA, *, group=None, fused_output: bool = False):
        super().__init__()
        c = module.config
        if c.projection_bias or c.output_bias or c.output_gate_bias:
            raise ValueError("tensor-parallel MLA supports bias-free projections")
        self.group = group
        s, e = head_slice(c.num_heads, group)
        self.head_start, self.head_end, self.num_heads = s, e, e - s
        self.config = c
        p = module.projections.query.weight
        self.inner = GatedMLA(local_head_config(c, e - s)).to(device=p.device, dtype=p.dtype)
        dq, dv = c.q_head_dim, c.v_head_dim
        src, dst = module.projections, self.inner.projections
        _copy(dst.query.weight, src.query.weight[s * dq:e * dq])
        _copy(dst.latent_kv.compression.weight, src.latent_kv.compression.weight)
        _copy(dst.latent_kv.key_up.weight, src.latent_kv.key_up.weight[s * dq:e * dq])
        _copy(dst.latent_kv.value_up.weight, src.latent_kv.value_up.weight[s * dv:e * dv])
        _copy(self.inner.output_gate.gate_proj.weight, module.output_gate.gate_proj.weight[s * dv:e * dv])
        _copy(self.inner.output_gate.output_proj.weight, module.output_gate.output_proj.weight[:, s * dv:e * dv])
        mark_tp_partial(dst.latent_kv.compression.weight)
        self.shard_dims = {"projections.query.weight": 0, "projections.latent_kv.compression.weight": None,
                           "projections.latent_kv.key_up.weight": 0, "projections.latent_kv.value_up.weight": 0,
                           "output_gate.gate_proj.weight": 0, "output_gate.output_proj.weight": 1}
        _tag_shards(self.inner, self.shard_dims, group)
        self.fused_output = _install_fused_output(self.inner, group, fused_output)
        self.inner._kimi_qk_group = group  # QK-Clip takes the MAX scale over the heads of all ranks
        for attr in ("absorbed_decode",):
            if hasattr(module, attr):
                setattr(self.inner, attr, getattr(module, attr))

    def forward(self, hidden_states, attention_mask=None, cache=None, use_cache=False, output_attentions=False,
                output_diagnostics=False, **kw):
        x = copy_to_tensor_parallel_region(hidden_states, self.group)
        out = self.inner(x, attention_mask=attention_mask, cache=cache, use_cache=use_cache,
                         output_attentions=output_attentions, output_diagnostics=output_diagnostics, **kw)
        if not self.fused_output:
            out.hidden_states = reduce_from_tensor_parallel_region(out.hidden_states, self.group)
        return out


def shard_kimi_attention(model: nn.Module, *, group=None, shard_kda: bool = True, shard_mla: bool = True,
                         fused_output: bool = False) -> int:
    """Replace every KDA / gated-MLA attention of every hybrid layer in place; returns the count.
    ``fused_output`` runs each shard's output projection and its all-reduce as one kernel."""
    from ..models.backbone import HybridAttentionLayer
    raw = model.module if hasattr(model, "module") else model
    n = 0
    for layer in raw.modules():
        if not isinstance(layer, HybridAttentionLayer):
            continue
        att = layer.attention
        if isinstance(att, KimiDeltaAttention) and shard_kda:
            layer.attention = TensorParallelKDA(att, group=group, fused_output=fused_output)
            n += 1
        elif isinstance(att, GatedMLA) and shard_mla:
            layer.attention = TensorParallelMLA(att, group=group, fused_output=fused_output)
            n += 1
    return n


__all__ = ["TensorParallelKDA", "TensorParallelMLA", "shard_kimi_attention", "head_slice", "mark_tp_partial"]
