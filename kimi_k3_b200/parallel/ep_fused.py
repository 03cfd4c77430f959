"""Expert parallelism with device-initiated NVLink transfers instead of NCCL all-to-alls.

The routed experts of an :class:`~kimi_k3_b200.parallel.expert_parallel.ExpertParallelMoE` run
through the kernels of ``csrc/ep_comm.cu`` over one symmetric buffer per MoE layer
(``torch.distributed._symmetric_memory``): the per-expert counts are exchanged on the device, every
source writes its latent rows directly into the owner's grouped expert-input buffer at their final
rows, the owner's down-projection GEMM adds the weighted results straight into the source's
aggregate over NVLink (the combine lives in the GEMM epilogue), and the backward reads the output
gradients and returns the input gradients with peer loads.  Nothing waits for the host, so the
whole training step (including these layers) can be captured in one CUDA graph.

Contract: every rank of the expert group runs the same layers in the same order with the same
number of tokens per layer (one forward, then its backward, before that layer's next forward).
Waits on peers are bounded (``timeout_s``); a timeout records a status that :meth:`check` turns
into an exception, after which :meth:`reset` must run on every rank.

Parity: same routing, no-drop exchange and per-token weighted sum as
``training/distributed/expert_parallel.py:24-128`` (reference).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_ALIGN = 1 << 12
_FLAG_BYTES = 1 << 12       # 8 kinds x 8 sources x 4 bytes, padded
_REGIONS = ("flags", "counts", "xs", "row_token", "row_weight", "agg", "dagg", "dxs", "dw_row")


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class EPWorkspace:
    """Symmetric buffers of one expert-parallel MoE layer (collective construction)."""

    _kimi_rendezvous = True  # one per process and peer set: model copies share it, never copy it

    def __init__(self, group, device, *, tokens: int, top_k: int, latent: int, num_experts: int,
                 timeout_s: float = 10.0):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.rank, self.world = dist.get_rank(self.group), dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("the fused expert-parallel exchange supports groups of at most 8 ranks")
        if num_experts % self.world or latent % 64:
            raise ValueError("experts must split evenly over the group and the latent width be a multiple of 64")
        self.device = torch.device(device)
        self.tokens, self.top_k, self.latent, self.num_experts = tokens, top_k, latent, num_experts
        self.per = num_experts // self.world
        self.r_max = self.world * tokens * top_k + self.per * 128
        self.timeout_ns = int(timeout_s * 1e9)
        sizes = {"flags": _FLAG_BYTES, "counts": self.world * num_experts * 4,
                 "xs": self.r_max * latent * 2, "row_token": self.r_max * 4, "row_weight": self.r_max * 4,
                 "agg": tokens * latent * 4, "dagg": tokens * latent * 4, "dxs": self.r_max * latent * 2,
                 "dw_row": self.r_max * 4}
        self.offsets = {}
        off = 0
        for name in _REGIONS:
            self.offsets[name] = off
            off += _align(sizes[name])
        buf = symm_mem.empty(off, dtype=torch.uint8, device=self.device)
        buf.zero_()
        torch.cuda.synchronize(self.device)
        self.handle = symm_mem.rendezvous(buf, self.group)
        self.buffer = buf
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.peer_list = [ptrs[r] + self.offsets[name] for name in _REGIONS for r in range(self.world)]
        self.agg_peers = [ptrs[r] + self.offsets["agg"] for r in range(self.world)]
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)

        def view(name, dtype, shape):
            o = self.offsets[name]
            n = 1
            for d in shape:
                n *= d
            return buf[o: o + n * torch.empty((), dtype=dtype).element_size()].view(dtype).view(*shape)

        self.xs = view("xs", torch.bfloat16, (self.r_max, latent))
        self.row_token = view("row_token", torch.int32, (self.r_max,))
        self.row_weight = view("row_weight", torch.float32, (self.r_max,))
        self.agg = view("agg", torch.float32, (tokens, latent))
        self.dagg = view("dagg", torch.float32, (tokens, latent))
        self.dxs = view("dxs", torch.bfloat16, (self.r_max, latent))
        # local scratch
        self.cnt = torch.zeros(num_experts, dtype=torch.int32, device=self.device)
        self.base = torch.zeros(num_experts, dtype=torch.int32, device=self.device)
        self.cursor = torch.zeros(num_experts, dtype=torch.int32, device=self.device)
        self.offsets_local = torch.zeros(self.per + 1, dtype=torch.int32, device=self.device)
        dist.barrier(group=self.group)

    @property
    def peer_args(self):
        return (self.peer_list, self.rank, self.world, self.status, self.timeout_ns)

    def check(self) -> None:
        code = int(self.status.item())
        if code:
            raise RuntimeError(f"fused expert-parallel exchange failed (status {code}): a peer did not arrive in "
                               "time; call reset() on every rank")

    def reset(self) -> None:
        torch.cuda.synchronize(self.device)
        self.buffer[: _FLAG_BYTES].zero_()
        self.status.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)


class _EPFusedExperts(torch.autograd.Function):
    @staticmethod
    def forward(ctx, latent, weights, selected, gate_w, up_w, down_w, bg, bu, ws):
        from ..ops import _loader
        C = _loader.require()
        m, l = latent.shape
        k = selected.shape[1]
        e_loc, h, _ = gate_w.shape
        pa = ws.peer_args
        sel = selected.long().contiguous()
        bf = torch.bfloat16
        wg, wu, wd = (w.to(bf).contiguous() for w in (gate_w, up_w, down_w))
        C.ep_count(sel, ws.num_experts, ws.cnt, ws.agg)
        C.ep_exchange(*pa, ws.cnt, ws.num_experts, ws.per, l, ws.offsets_local, ws.base, ws.cursor)
        slot_pos = torch.empty(m * k, dtype=torch.int32, device=latent.device)
        C.ep_dispatch(*pa, latent.to(bf), sel, weights.detach(), ws.num_experts, ws.per, ws.base, ws.cursor,
                      slot_pos)
        C.ep_wait(*pa, 1, C.ep_dispatch_grid(m * k))
        offs = ws.offsets_local
        hh, gg, uu = C.tc_gemm_grouped(1, ws.xs, wg, wu, False, False, offs, ws.r_max, h, l, 1, None, False, bg, bu,
                                       None, None, 0, 256)
        C.tc_gemm_grouped_remote(hh, wd, offs, ws.r_max, l, h, ws.row_token, ws.row_weight, ws.agg_peers, m, 128)
        C.ep_signal_wait(*pa, 2)
        agg = ws.agg.clone()
        ctx.save_for_backward(sel, slot_pos, gg, uu, hh, wg, wu, wd)
        ctx.ws = ws
        ctx.c = (m, k, h, l, float(bg), float(bu), latent.dtype, gate_w.dtype)
        return agg

    @staticmethod
    def backward(ctx, dagg):
        from ..ops import _loader
        C = _loader.require()
        sel, slot_pos, gg, uu, hh, wg, wu, wd = ctx.saved_tensors
        ws = ctx.ws
        m, k, h, l, bg, bu, ldt, wdt = ctx.c
        pa = ws.peer_args
        offs = ws.offsets_local
        ws.dagg.copy_(dagg)
        C.ep_signal_wait(*pa, 3)
        y, = C.tc_gemm_grouped(1, hh, wd, None, False, False, offs, ws.r_max, l, h, 0, None, False, bg, bu, None,
                               None, 0, 256)
        dy = C.ep_dy(*pa, offs, m, y)
        dh, = C.tc_gemm_grouped(1, dy, wd, None, False, True, offs, ws.r_max, h, l, 0, None, False, bg, bu, None,
                                None, 0, 256)
        dwd, = C.tc_gemm_grouped(2, dy, hh, None, True, True, offs, l, h, ws.r_max, 0, None, True, bg, bu, None,
                                 None, 0, 256)
        dgu = C.situ_bwd_cat(dh, gg, uu, bg, bu)
        C.tc_gemm_grouped(1, dgu, wg, wu, False, True, offs, ws.r_max, l, 2 * h, 0, ws.dxs, False, bg, bu, None,
                          None, h, 256)
        dwg, = C.tc_gemm_grouped(2, dgu[:, :h], ws.xs, None, True, True, offs, h, l, ws.r_max, 0, None, True, bg,
                                 bu, None, None, 0, 256)
        dwu, = C.tc_gemm_grouped(2, dgu[:, h:], ws.xs, None, True, True, offs, h, l, ws.r_max, 0, None, True, bg,
                                 bu, None, None, 0, 256)
        C.ep_signal_wait(*pa, 4)
        dlat, dweights = C.ep_slot_sum(*pa, sel, slot_pos, ws.num_experts, ws.per, l, ldt == torch.float32)
        return (dlat.to(ldt), dweights, None, dwg.to(wdt), dwu.to(wdt), dwd.to(wdt), None, None, None)


def fused_ep_experts(latent, selected, weights, experts, workspace: EPWorkspace, beta_gate, beta_up):
    """``sum_slot w * expert(latent)`` over the expert group, fp32 [M, L]; ``experts`` holds this
    rank's contiguous block of routed experts (stacked gate / up / down weights)."""
    return _EPFusedExperts.apply(latent, weights, selected, experts.gate_proj, experts.up_proj, experts.down_proj,
                                 float(beta_gate), float(beta_up), workspace)


__all__ = ["EPWorkspace", "fused_ep_experts"]
