"""Tensor-parallel building blocks (Megatron-style regions, column/row linears, vocabulary).

Parity: ``training/distributed/tensor_parallel.py:25-369`` (reference): copy-to-region
(identity forward, all-reduce backward), reduce-from-region (all-reduce forward), gather of
the last dimension, column/row parallel linears built from an existing ``nn.Linear``,
contiguous vocabulary shards for the embedding and the LM head, vocabulary-parallel CE.

Differences by design:

* the LM head used by the training losses never gathers logits: the fused vocabulary-parallel
  linear cross-entropy below computes each row's log-sum-exp from per-shard maxima and sums
  (two small all-reduces per chunk) and forms dH / dW in the forward pass (the reference
  gathers the full ``[B, T, V]`` logits on every rank);
* shard weights carry ``_kimi_vocab_parallel`` metadata so the loss code picks this path.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn as nn

from ..debug import nvtx
import torch.nn.functional as F


def group_size(group) -> int:
    """Size of a parallel-axis group; ``None`` is an axis of size one (pass ``dist.group.WORLD``
    explicitly for the whole world)."""
    if group is None or not (dist.is_available() and dist.is_initialized()):
        return 1
    return dist.get_world_size(group)


def group_rank(group) -> int:
    if group is None or not (dist.is_available() and dist.is_initialized()):
        return 0
    return dist.get_rank(group)


def partition(total: int, group, name: str) -> tuple:
    size, rank = group_size(group), group_rank(group)
    if total % size:
        raise ValueError(f"{name}={total} is not divisible by tensor-parallel size {size}")
    per = total // size
    return rank * per, (rank + 1) * per


class _CopyToRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        if group_size(ctx.group) > 1:
            g = g.contiguous()
            dist.all_reduce(g, group=ctx.group)
        return g, None


class _ReduceFromRegion(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        if group_size(group) > 1:
            x = x.contiguous().clone()
            dist.all_reduce(x, group=group)
        return x

    @staticmethod
    def backward(ctx, g):
        return g, None


class _GatherLastDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        n = group_size(group)
        if n == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(n)]
        dist.all_gather(parts, x.contiguous(), group=group)
        ctx.width = x.shape[-1]
        return torch.cat(parts, dim=-1)

    @staticmethod
    def backward(ctx, g):
        if group_size(ctx.group) == 1:
            return g, None
        r = group_rank(ctx.group)
        return g[..., r * ctx.width:(r + 1) * ctx.width].contiguous(), None


def copy_to_tensor_parallel_region(x, group=None):
    return _CopyToRegion.apply(x, group)


def reduce_from_tensor_parallel_region(x, group=None):
    with nvtx("tp all-reduce"):
        return _ReduceFromRegion.apply(x, group)


def gather_from_tensor_parallel_region(x, group=None):
    with nvtx("tp all-gather"):
        return _GatherLastDim.apply(x, group)


class ColumnParallelLinear(nn.Module):
    """Output features sharded: rows ``[start, end)`` of the source weight."""

    def __init__(self, linear: nn.Linear, *, group=None, gather_output: bool = False, copy_input: bool = True):
        super().__init__()
        start, end = partition(linear.out_features, group, "out_features")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.local_out_features = end - start
        self.group, self.gather_output, self.copy_input = group, gather_output, copy_input
        self.weight = nn.Parameter(linear.weight.detach()[start:end].clone(), requires_grad=linear.weight.requires_grad)
        self.bias = (None if linear.bias is None else
                     nn.Parameter(linear.bias.detach()[start:end].clone(), requires_grad=linear.bias.requires_grad))

    def forward(self, x):
        if self.copy_input:
            x = copy_to_tensor_parallel_region(x, self.group)
        y = F.linear(x, self.weight, self.bias)
        return gather_from_tensor_parallel_region(y, self.group) if self.gather_output else y


class RowParallelLinear(nn.Module):
    """Input features sharded: columns ``[start, end)``; partial outputs are all-reduced.
    The bias is added once, after the reduction."""

    def __init__(self, linear: nn.Linear, *, group=None, input_is_parallel: bool = True, reduce_output: bool = True):
        super().__init__()
        start, end = partition(linear.in_features, group, "in_features")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.group, self.input_is_parallel, self.reduce_output = group, input_is_parallel, reduce_output
        self.start, self.end = start, end
        self.weight = nn.Parameter(linear.weight.detach()[:, start:end].clone(),
                                   requires_grad=linear.weight.requires_grad)
        self.bias = (None if linear.bias is None else
                     nn.Parameter(linear.bias.detach().clone(), requires_grad=linear.bias.requires_grad))

    def forward(self, x):
        if not self.input_is_parallel:
            x = x[..., self.start:self.end]
        y = F.linear(x, self.weight)
        if self.reduce_output:
            y = reduce_from_tensor_parallel_region(y, self.group)
        return y if self.bias is None else y + self.bias


class VocabParallelEmbedding(nn.Module):
    """Contiguous vocabulary shard; out-of-shard ids contribute zeros, outputs are all-reduced."""

    def __init__(self, embedding: nn.Embedding, *, group=None):
        super().__init__()
        start, end = partition(embedding.num_embeddings, group, "vocab_size")
        self.num_embeddings, self.embedding_dim = embedding.num_embeddings, embedding.embedding_dim
        self.vocab_start, self.vocab_end, self.group = start, end, group
        self.padding_idx = embedding.padding_idx
        self._kimi_role = "embedding"
        self.weight = nn.Parameter(embedding.weight.detach()[start:end].clone(),
                                   requires_grad=embedding.weight.requires_grad)
        self.weight._kimi_vocab_parallel = (start, end, embedding.num_embeddings, group)

    def forward(self, input_ids):
        outside = (input_ids < self.vocab_start) | (input_ids >= self.vocab_end)
        local = (input_ids - self.vocab_start).masked_fill(outside, 0)
        pad = (self.padding_idx - self.vocab_start
               if self.padding_idx is not None and self.vocab_start <= self.padding_idx < self.vocab_end else None)
        out = F.embedding(local, self.weight, padding_idx=pad).masked_fill(outside[..., None], 0)
        return reduce_from_tensor_parallel_region(out, self.group)


class VocabParallelLMHead(nn.Module):
    """Vocabulary-sharded head. ``forward`` returns gathered logits for API compatibility
    (generation, previews); the training losses use the fused vocabulary-parallel CE."""

    def __init__(self, linear: nn.Linear, *, group=None, gather_output: bool = True,
                 tied_weight: nn.Parameter | None = None):
        super().__init__()
        start, end = partition(linear.out_features, group, "vocab_size")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.local_out_features = end - start
        self.vocab_start, self.vocab_end, self.group, self.gather_output = start, end, group, gather_output
        self._kimi_role = "lm_head"
        self.weight = tied_weight if tied_weight is not None else nn.Parameter(
            linear.weight.detach()[start:end].clone(), requires_grad=linear.weight.requires_grad)
        self.weight._kimi_vocab_parallel = (start, end, linear.out_features, group)
        self.bias = (None if linear.bias is None else
                     nn.Parameter(linear.bias.detach()[start:end].clone(), requires_grad=linear.bias.requires_grad))

    def forward(self, hidden):
        local = F.linear(copy_to_tensor_parallel_region(hidden, self.group), self.weight, self.bias)
        return gather_from_tensor_parallel_region(local, self.group) if self.gather_output else local


# --------------------------------------------------------------------------- vocabulary-parallel CE
class _VocabParallelCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, local_logits, targets, start, end, ignore_index, group):
        x = local_logits.float()
        gmax = x.max(dim=-1).values
        if group_size(group) > 1:
            dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
        ex = torch.exp(x - gmax[..., None])
        den = ex.sum(-1)
        if group_size(group) > 1:
            dist.all_reduce(den, group=group)
        prob = ex / den[..., None]
        here = (targets >= start) & (targets < end)
        safe = (targets - start).masked_fill(~here, 0)
        sel = x.gather(-1, safe[..., None]).squeeze(-1).masked_fill(~here, 0)
        if group_size(group) > 1:
            dist.all_reduce(sel, group=group)
        valid = targets != ignore_index
        loss = (gmax + den.log() - sel).masked_fill(~valid, 0)
        ctx.save_for_backward(prob, safe, here, valid)
        return loss

    @staticmethod
    def backward(ctx, g):
        prob, safe, here, valid = ctx.saved_tensors
        onehot = torch.zeros_like(prob).scatter_(-1, safe[..., None], 1.0) * here[..., None]
        return (prob - onehot) * valid[..., None] * g[..., None], None, None, None, None, None


def vocab_parallel_cross_entropy(local_logits, targets, *, vocab_start: int, vocab_end: int, ignore_index: int = -100,
                                 group=None):
    """Unreduced CE over vocabulary-sharded logits (global logits never materialised)."""
    if local_logits.shape[:-1] != targets.shape:
        raise ValueError("targets must match logits except for vocabulary axis")
    return _VocabParallelCE.apply(local_logits, targets, vocab_start, vocab_end, ignore_index, group)


class _VocabParallelLinearCE(torch.autograd.Function):
    """``sum_valid CE(h W_shard^T)`` with the row log-sum-exp reduced over the shards."""

    @staticmethod
    def forward(ctx, h, w, targets, valid, start, group, chunk_rows):
        n, d = h.shape
        dh = torch.zeros(n, d, device=h.device, dtype=torch.float32)
        dw = torch.zeros(w.shape, device=w.device, dtype=torch.float32)
        loss = torch.zeros((), device=h.device, dtype=torch.float32)
        wl = w.to(h.dtype)
        multi = group_size(group) > 1
        for s in range(0, n, chunk_rows):
            e = min(n, s + chunk_rows)
            hc = h[s:e]
            x = (hc @ wl.t()).float()
            m = x.max(-1).values
            if multi:
                dist.all_reduce(m, op=dist.ReduceOp.MAX, group=group)
            ex = torch.exp(x - m[:, None])
            here = (targets[s:e] >= start) & (targets[s:e] < start + w.shape[0])
            safe = (targets[s:e] - start).clamp(0, w.shape[0] - 1)
            sums = torch.stack((ex.sum(-1), x.gather(-1, safe[:, None]).squeeze(-1) * here), 0)
            if multi:
                dist.all_reduce(sums, group=group)
            lse = m + sums[0].log()
            ok = valid[s:e]
            loss += ((lse - sums[1]) * ok).sum()
            gl = ex / sums[0][:, None]
            gl.scatter_add_(-1, safe[:, None], -here.float()[:, None])
            gl *= ok.float()[:, None]
            dh[s:e] = gl @ wl.float()
            dw += gl.t() @ hc.float()
        if multi:
            dist.all_reduce(dh, group=group)  # h is replicated across the shards
        ctx.save_for_backward(dh, dw)
        ctx.dtypes = (h.dtype, w.dtype)
        return loss

    @staticmethod
    def backward(ctx, g):
        dh, dw = ctx.saved_tensors
        return (dh * g).to(ctx.dtypes[0]), (dw * g).to(ctx.dtypes[1]), None, None, None, None, None


def vocab_parallel_linear_cross_entropy(hidden, weight_shard, targets, valid, *, vocab_start: int, group=None,
                                        chunk_rows: int = 8192):
    """Fused LM head + CE over a contiguous vocabulary shard; returns the valid-row loss sum."""
    h = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    return _VocabParallelLinearCE.apply(h, weight_shard, targets.reshape(-1).long(), valid.reshape(-1).bool(),
                                        int(vocab_start), group, int(chunk_rows))


@dataclass(frozen=True)
class TensorParallelMetadata:
    size: int
    rank: int
    vocab_start: int | None
    vocab_end: int | None
    cache_layout: str
    transformed_attention_layers: int = 0


def shard_vocabulary(model: nn.Module, *, group=None, gather_logits: bool = True) -> TensorParallelMetadata:
    """Replace the (tied) embedding and LM head with contiguous vocabulary shards in place."""
    raw = model.module if hasattr(model, "module") else model
    emb = raw.get_input_embeddings()
    head = raw.get_output_embeddings()
    tied = head is not None and emb is not None and head.weight is emb.weight
    new_emb = VocabParallelEmbedding(emb, group=group)
    new_head = VocabParallelLMHead(head, group=group, gather_output=gather_logits,
                                   tied_weight=new_emb.weight if tied else None)
    raw.set_input_embeddings(new_emb)
    raw.set_output_embeddings(new_head)
    if hasattr(raw, "tie_weights") and tied:
        raw.tie_weights()
    return TensorParallelMetadata(group_size(group), group_rank(group), new_emb.vocab_start, new_emb.vocab_end,
                                  "replicated")


__all__ = ["group_size", "group_rank", "partition", "copy_to_tensor_parallel_region",
           "reduce_from_tensor_parallel_region", "gather_from_tensor_parallel_region", "ColumnParallelLinear",
           "RowParallelLinear", "VocabParallelEmbedding", "VocabParallelLMHead", "vocab_parallel_cross_entropy",
           "vocab_parallel_linear_cross_entropy", "TensorParallelMetadata", "shard_vocabulary"]
