"""No-drop expert parallelism for Stable LatentMoE.

Parity: ``training/distributed/expert_parallel.py:18-317`` (reference): each EP rank keeps a
contiguous block of routed experts; router, down/up projections, aggregate norm and shared
experts are replicated; every (token, slot) assignment is sent to the rank owning its expert,
computed there, and the weighted latent rows come back for the per-token sum; Quantile
Balancing stays exact across ranks (histograms all-reduced, exact scores all-gathered); no
token is ever dropped.

Data movement here: one ``all_to_all_single`` of the per-rank counts (read on the host for
the split sizes), one for the latent rows (activation dtype) and one for a packed fp32
``[local expert id | routing weight]`` pair per row (the reference sends ids and weights
separately); the local experts run as grouped GEMMs on device, and one ``all_to_all_single``
returns the weighted rows. Autograd flows through ``torch.distributed.nn`` collectives.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from ..models.moe import GroupedRoutedExperts, StableLatentMoE, vectorized_sparse_dispatch
from .. import ops as _ops
from ..debug import nvtx
from .data_parallel import QBReducer
from .tensor_parallel import group_rank, group_size


# inference-time fused-exchange workspaces shared by all MoE layers of one shape:
# key -> (process group, workspace)
_SHARED_WORKSPACES: dict = {}


def release_shared_workspaces() -> None:
    """Drop the inference-time exchange workspaces (before destroying their process groups)."""
    _SHARED_WORKSPACES.clear()


def expert_range(num_experts: int, group) -> tuple:
    size, rank = group_size(group), group_rank(group)
    if num_experts % size:
        raise ValueError(f"num_routed_experts={num_experts} is not divisible by expert-parallel size {size}")
    per = num_experts // size
    return rank * per, (rank + 1) * per


def _a2a(x: torch.Tensor, out_splits: list, in_splits: list, group) -> torch.Tensor:
    from torch.distributed.nn.functional import all_to_all_single
    out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
    return all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=group)


class _TakeRows(torch.autograd.Function):
    """Forward: this rank's contiguous row block of a replicated tensor. Backward: all-gather
    the blocks' gradients so every replica receives the full gradient."""

    @staticmethod
    def forward(ctx, x, group, start, end, padded):
        ctx.group, ctx.shape, ctx.start, ctx.end, ctx.padded = group, x.shape, start, end, padded
        return x[start:end]

    @staticmethod
    def backward(ctx, g):
        n = group_size(ctx.group)
        blk = ctx.padded // n
        buf = g.new_zeros((blk,) + tuple(g.shape[1:]))
        buf[: g.shape[0]] = g
        parts = [torch.empty_like(buf) for _ in range(n)]
        dist.all_gather(parts, buf.contiguous(), group=ctx.group)
        full = torch.cat(parts, 0)[: ctx.shape[0]]
        return full, None, None, None, None


class _GatherRows(torch.autograd.Function):
    """Forward: all-gather row blocks into the replicated full tensor. Backward: keep this
    rank's block of the (replicated) upstream gradient, no reduction."""

    @staticmethod
    def forward(ctx, x, group, total, padded):
        n = group_size(group)
        blk = padded // n
        ctx.rows, ctx.rank, ctx.blk = x.shape[0], group_rank(group), blk
        buf = x.new_zeros((blk,) + tuple(x.shape[1:]))
        buf[: x.shape[0]] = x
        parts = [torch.empty_like(buf) for _ in range(n)]
        dist.all_gather(parts, buf.contiguous(), group=group)
        return torch.cat(parts, 0)[:total]

    @staticmethod
    def backward(ctx, g):
        s = ctx.rank * ctx.blk
        return g[s: s + ctx.rows].contiguous(), None, None, None


def exchange_counts(send_counts: torch.Tensor, group) -> list:
    recv = torch.empty_like(send_counts)
    dist.all_to_all_single(recv, send_counts.contiguous(), group=group)
    return recv.tolist()


class ExpertParallelMoE(StableLatentMoE):
    """A ``StableLatentMoE`` whose routed experts are split over an expert-parallel group."""

    def __init__(self, module: StableLatentMoE, *, group=None, token_split: bool = False, fused_comm: bool = False):
        nn.Module.__init__(self)
        self.__dict__.update({k: v for k, v in module.__dict__.items() if k not in ("_modules", "_parameters",
                                                                                      "_buffers")})
        self._modules = dict(module._modules)
        self._parameters = dict(module._parameters)
        self._buffers = dict(module._buffers)
        self.group = group
        c = module.config
        s, e = expert_range(c.num_routed_experts, group)
        self.expert_start, self.expert_end = s, e
        full = module.routed_experts
        local = GroupedRoutedExperts(e - s, full.width, full.hidden_dim, full.beta_gate, full.beta_up, c.init_std)
        local = local.to(device=full.gate_proj.device, dtype=full.gate_proj.dtype)
        with torch.no_grad():
            local.gate_proj.copy_(full.gate_proj[s:e])
            local.up_proj.copy_(full.up_proj[s:e])
            local.down_proj.copy_(full.down_proj[s:e])
        local._kimi_expert_parallel = (s, e, c.num_routed_experts)
        local._kimi_ep_group = group
        self.routed_experts = local
        for p in local.parameters():
            p._kimi_local_expert = True
        self._qb_reducer = QBReducer(group)
        # CUDA ranks: device-initiated NVLink exchange (``ep_fused``) instead of NCCL all-to-alls
        self.fused_comm = bool(fused_comm)
        self._ep_workspace = None
        self._token_block = None
        # EP overlaid on TP: the group shares one token stream, so each rank takes a block of
        # the tokens, and the replicated MoE weights see only that block (sum over the group).
        self.token_split = bool(token_split)
        if self.token_split:
            for p in self.parameters():
                if not getattr(p, "_kimi_local_expert", False):
                    p._kimi_tp_partial = True

    def forward(self, inputs, **kw):
        if not self.token_split or group_size(self.group) == 1:
            return super().forward(inputs, **kw)
        shape = inputs.shape
        flat = inputs.reshape(-1, shape[-1])
        m, n, r = flat.shape[0], group_size(self.group), group_rank(self.group)
        blk = -(-m // n)
        s, e = min(r * blk, m), min((r + 1) * blk, m)
        local = _TakeRows.apply(flat, self.group, s, e, blk * n)
        self._token_block = blk  # equal on every rank: the fused exchange's row capacity
        try:
            out = super().forward(local, **kw)
        finally:
            self._token_block = None
        hidden = out if torch.is_tensor(out) else out.hidden_states
        full = _GatherRows.apply(hidden, self.group, m, blk * n).reshape(shape)
        if torch.is_tensor(out):
            return full
        out.hidden_states = full
        return out

    def finalize_and_commit_balance(self, reducer=None, keep_old=None):
        """Global statistics over the expert group (and then any outer reducer)."""
        class _Chain:
            def __init__(self, first, second):
                self.first, self.second = first, second

            def reduce_histogram(self, balancer):
                self.first.reduce_histogram(balancer)
                if self.second is not None:
                    self.second.reduce_histogram(balancer)

            def gather_exact(self, scores, cutoffs):
                scores, cutoffs = self.first.gather_exact(scores, cutoffs)
                if self.second is not None:
                    scores, cutoffs = self.second.gather_exact(scores, cutoffs)
                return scores, cutoffs
        return super().finalize_and_commit_balance(_Chain(self._qb_reducer, reducer), keep_old=keep_old)

    @property
    def device_exchange(self) -> bool:
        """True when routed rows move through the device-initiated NVLink exchange: no host
        synchronisation, so the layer can run inside a captured CUDA graph."""
        c = self.config
        return (self.fused_comm and self.routed_experts.gate_proj.is_cuda and c.latent_dim % 64 == 0
                and c.routed_expert_hidden_dim % 128 == 0 and c.routed_accumulation_dtype == "float32")

    def _fused_workspace(self, tokens: int, top_k: int, latent: int):
        """The symmetric buffers of the fused exchange for ``tokens`` rows per rank.  Training keeps
        one per layer (backward reads the rows its forward dispatched); without autograd every layer
        of the same shape shares one from a process-wide pool, since layers run one after another."""
        from .ep_fused import EPWorkspace
        key = (id(self.group), tokens, top_k, latent, self.config.num_routed_experts)
        shared = not torch.is_grad_enabled()
        if shared:
            hit = _SHARED_WORKSPACES.get(key)
            # the entry keeps its group alive, so a recycled id cannot alias another group
            ws = hit[1] if hit is not None and hit[0] is self.group else None
        else:
            ws = self._ep_workspace
        if ws is None or ws.tokens != tokens or ws.top_k != top_k or ws.latent != latent:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the expert-parallel workspace must exist before CUDA-graph capture")
            ws = EPWorkspace(self.group, torch.device("cuda", torch.cuda.current_device()), tokens=tokens, top_k=top_k,
                             latent=latent, num_experts=self.config.num_routed_experts)
            if shared:
                _SHARED_WORKSPACES[key] = (self.group, ws)
            else:
                self._ep_workspace = ws
        return ws

    def _fused_routed(self, latent, ro):
        """The fused exchange over a row count that is the same on every rank (the exchange encodes
        source rows as ``rank * rows + row``): with the token split, rows are padded to the block
        size with zero-weight assignments whose results are dropped."""
        from .ep_fused import fused_ep_experts
        m, l = latent.shape
        sel, w = ro.selected_experts, ro.selected_weights
        k = sel.shape[1]
        cap = self._token_block if self._token_block is not None else m
        if cap > m:
            pad = cap - m
            e = self.config.num_routed_experts
            latent = torch.cat((latent, latent.new_zeros(pad, l)), 0)
            fill = (torch.arange(pad * k, device=sel.device) % e).view(pad, k).to(sel.dtype)
            sel = torch.cat((sel, fill), 0)
            w = torch.cat((w, w.new_zeros(pad, k)), 0)
        ws = self._fused_workspace(cap, k, l)
        out = fused_ep_experts(latent, sel, w, self.routed_experts, ws, self.config.beta_gate, self.config.beta_up)
        return out[:m] if cap > m else out

    def routed_aggregate(self, latent, ro, accumulation_dtype):
        with nvtx("expert exchange"):
            return self._routed_aggregate(latent, ro, accumulation_dtype)

    def _routed_aggregate(self, latent, ro, accumulation_dtype):
        m, l = latent.shape
        k = ro.selected_experts.shape[1]
        if (self.fused_comm and _ops.use_kernels(latent) and accumulation_dtype == torch.float32 and l % 64 == 0
                and self.config.routed_expert_hidden_dim % 128 == 0):
            return self._fused_routed(latent, ro)
        group, world = self.group, group_size(self.group)
        per = self.expert_end - self.expert_start
        flat_e = ro.selected_experts.reshape(-1).long()
        flat_w = ro.selected_weights.reshape(-1)
        flat_t = torch.arange(m, device=latent.device).repeat_interleave(k)
        owner = torch.div(flat_e, per, rounding_mode="floor")
        order = torch.argsort(owner, stable=True)
        send_counts = torch.bincount(owner, minlength=world).to(torch.int64)
        in_splits = send_counts.tolist()
        out_splits = exchange_counts(send_counts, group)
        # latent rows in the activation dtype; [local expert id | routing weight] in fp32
        rows = latent.index_select(0, flat_t[order])
        meta = torch.stack(((flat_e[order] - owner[order] * per).to(torch.float32), flat_w[order].float()), 1)
        r_lat = _a2a(rows, out_splits, in_splits, group)
        r_meta = _a2a(meta, out_splits, in_splits, group)
        r_eid, r_w = r_meta[:, 0].round().long(), r_meta[:, 1]
        if r_lat.shape[0]:
            if (_ops.use_kernels(r_lat) and accumulation_dtype == torch.float32 and l % 64 == 0
                    and self.config.routed_expert_hidden_dim % 128 == 0):
                out = _ops.moe_grouped_experts(r_lat, r_eid[:, None], r_w[:, None], self.routed_experts.gate_proj,
                                               self.routed_experts.up_proj, self.routed_experts.down_proj,
                                               self.config.beta_gate, self.config.beta_up)
            else:
                out = vectorized_sparse_dispatch(r_lat, self.routed_experts, r_eid[:, None], r_w[:, None],
                                                 accumulation_dtype=accumulation_dtype)
        else:
            out = r_lat.new_zeros(0, l, dtype=accumulation_dtype) + 0.0 * self.routed_experts.down_proj.sum()
        back = _a2a(out.to(accumulation_dtype), in_splits, out_splits, group)
        agg = torch.zeros(m, l, device=latent.device, dtype=accumulation_dtype)
        return agg.index_add(0, flat_t[order], back)


def shard_kimi_experts(model: nn.Module, *, group=None, token_split: bool = False, fused_comm: bool = False) -> int:
    """Replace every balanced StableLatentMoE by its expert-parallel form; returns the count."""
    raw = model.module if hasattr(model, "module") else model
    count = 0
    for parent in list(raw.modules()):
        for name, child in list(parent.named_children()):
            if isinstance(child, StableLatentMoE) and not isinstance(child, ExpertParallelMoE):
                setattr(parent, name, ExpertParallelMoE(child, group=group, token_split=token_split,
                                                        fused_comm=fused_comm))
                count += 1
    return count


def local_expert_parameter_ids(model: nn.Module) -> set:
    return {id(p) for p in model.parameters() if getattr(p, "_kimi_local_expert", False)}


@torch.no_grad()
def scale_local_expert_gradients(model: nn.Module, *, group=None) -> None:
    """Local experts receive the tokens of every EP rank, each rank's loss already scaled by
    the replica count: divide by the EP size (replicated parameters are averaged instead)."""
    n = group_size(group)
    if n <= 1:
        return
    grads = [p.grad for p in model.parameters() if getattr(p, "_kimi_local_expert", False) and p.grad is not None]
    if grads:
        torch._foreach_mul_(grads, 1.0 / n)


__all__ = ["ExpertParallelMoE", "shard_kimi_experts", "expert_range", "exchange_counts", "release_shared_workspaces",
           "local_expert_parameter_ids", "scale_local_expert_gradients"]
