"""Symmetric-memory workspaces and the fused GEMM + cross-rank reduction of tensor parallelism.

A row-parallel projection computes a partial product on every rank of the tensor-parallel
group and sums it over the group.  Here both happen in ONE kernel (``tc_gemm_comm`` of the
extension): the tcgen05 GEMM's epilogue writes each partial tile into this rank's slice of a
symmetric buffer (one allocation mapped on every rank, ``torch.distributed._symmetric_memory``)
and signals the tile's owner; comm warps of the same kernel reduce the owned tiles over NVLink
while the tensor cores work on later tiles -- with one NVLS multicast ``multimem.ld_reduce`` per
16 bytes when the group has a multicast object, peer loads and stores otherwise.  The
all-reduce result is copied out tile by tile; the reduce-scatter result lands directly in the
owner's output rows.  Flags are counting semaphores in the same buffer, so calls (and CUDA-graph
replays) need no host bookkeeping.  Every wait on a peer is bounded (``timeout_s``) and raises
through the status word; after a timeout the workspace must be ``reset()`` by all ranks.

Parity: replaces the ``all_reduce`` of the reference's tensor-parallel outputs
(``training/distributed/tensor_parallel.py:38-76,130`` reduce-from-region / row-parallel linear,
used by ``training/distributed/kimi_tensor_parallel.py``) with the fused kernel; the math is
the same sum.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_TILES_CAP = 1 << 15        # flag words per direction (tiles of one launch)
_ALIGN = 1 << 16
_workspaces: dict = {}


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class SymmetricWorkspace:
    """A symmetric buffer ``[partials | ready flags | done flags]`` for one process group and device.

    Construction and :meth:`grow` are collective over the group (every rank must call them with
    the same sizes, in the same order)."""

    _kimi_rendezvous = True  # one per process and peer set: model copies share it, never copy it

    def __init__(self, group=None, device=None, partial_bytes: int = 1 << 24, *, use_multicast: bool = True):
        self.group = group if group is not None else dist.group.WORLD
        self.device = torch.device(device if device is not None else "cuda", torch.cuda.current_device()) \
            if device is None or torch.device(device).index is None else torch.device(device)
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("the fused reduction supports tensor-parallel groups of at most 8 ranks")
        self.use_multicast = use_multicast
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._allocate(partial_bytes)

    def _allocate(self, partial_bytes: int) -> None:
        import torch.distributed._symmetric_memory as symm_mem
        self.partial_bytes = _align(partial_bytes)
        flag_bytes = _align(2 * _TILES_CAP * 4)
        buf = symm_mem.empty(self.partial_bytes + flag_bytes, dtype=torch.uint8, device=self.device)
        buf.zero_()
        torch.cuda.synchronize(self.device)
        self.handle = symm_mem.rendezvous(buf, self.group)
        self.buffer = buf
        self.peer_ptrs = [int(p) for p in self.handle.buffer_ptrs]
        mc = int(getattr(self.handle, "multicast_ptr", 0) or 0)
        self.multicast_ptr = mc if self.use_multicast else 0
        self.flag_ptrs = [p + self.partial_bytes for p in self.peer_ptrs]
        dist.barrier(group=self.group)

    def grow(self, partial_bytes: int) -> None:
        """Reallocate for at least ``partial_bytes`` of partials (collective)."""
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the symmetric workspace cannot grow during CUDA-graph capture; size it first")
        torch.cuda.synchronize(self.device)
        self._allocate(max(partial_bytes, 2 * self.partial_bytes))

    def partial(self, rows: int, cols: int) -> torch.Tensor:
        return self.buffer[: rows * cols * 2].view(torch.bfloat16).view(rows, cols)

    def check(self) -> None:
        """Raise if a wait on a peer timed out (one host sync)."""
        code = int(self.status.item())
        if code:
            raise RuntimeError(f"fused tensor-parallel reduction failed (status {code}): a peer did not arrive in "
                               "time; call reset() on every rank before the next use")

    def reset(self) -> None:
        """Zero the flags and the status after a failed call (collective)."""
        torch.cuda.synchronize(self.device)
        self.buffer[self.partial_bytes:].zero_()
        self.status.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    @property
    def has_multicast(self) -> bool:
        return self.multicast_ptr != 0


def workspace_for(group, device, partial_bytes: int) -> SymmetricWorkspace:
    """The cached workspace of ``(group, device)``, grown (collectively) when too small."""
    key = (id(group) if group is not None else None, str(device))
    ws = _workspaces.get(key)
    if ws is None:
        ws = SymmetricWorkspace(group, device, partial_bytes)
        _workspaces[key] = ws
    elif ws.partial_bytes < partial_bytes:
        ws.grow(partial_bytes)
    return ws


def release_workspaces() -> None:
    _workspaces.clear()


def fused_matmul_reduce(x: torch.Tensor, weight: torch.Tensor, workspace: SymmetricWorkspace, *,
                        reduce: str = "all_reduce", out: torch.Tensor | None = None,
                        timeout_s: float = 10.0) -> torch.Tensor:
    """``sum over ranks of x @ weight^T`` in one kernel.

    ``x`` [M, K] and ``weight`` [N, K] are bf16 (N % 8 == 0).  ``reduce="all_reduce"`` returns
    [M, N] on every rank; ``"reduce_scatter"`` returns this rank's [M / world, N] row block
    (M / world a multiple of 128)."""
    from ..ops import _loader
    C = _loader.require()
    if x.dim() != 2 or weight.dim() != 2 or x.shape[1] != weight.shape[1]:
        raise ValueError("x must be [M, K] and weight [N, K]")
    m, n = x.shape[0], weight.shape[0]
    mode = {"all_reduce": 1, "reduce_scatter": 2}[reduce]
    if mode == 2 and (m % workspace.world or (m // workspace.world) % 128):
        raise ValueError("reduce_scatter needs M / world to be a multiple of 128")
    x = x.to(torch.bfloat16).contiguous()
    w = weight.to(torch.bfloat16).contiguous()
    if m * n * 2 > workspace.partial_bytes:
        workspace.grow(m * n * 2)
    bn = 256 if n >= 256 else 128
    if C.tc_gemm_tiles(m, n, bn) > _TILES_CAP:
        raise ValueError("too many output tiles for one fused launch; split the rows")
    rows = m if mode == 1 else m // workspace.world
    if out is None:
        out = torch.empty(rows, n, dtype=torch.bfloat16, device=x.device)
    part = workspace.partial(m, n)
    C.tc_gemm_comm(x, w, False, bn, mode, workspace.rank, workspace.world, part, workspace.peer_ptrs,
                   workspace.multicast_ptr, workspace.flag_ptrs, _TILES_CAP, out, workspace.status,
                   int(timeout_s * 1e9))
    return out


class _FusedRowParallel(torch.autograd.Function):
    """Row-parallel linear whose forward all-reduce is fused into the GEMM.  Backward needs no
    communication: the output gradient is replicated, ``dx = dy W`` and ``dW = dy^T x`` are local."""

    @staticmethod
    def forward(ctx, x, weight, group):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        ws = workspace_for(group, x.device, x2.shape[0] * weight.shape[0] * 2)
        y = fused_matmul_reduce(x2, weight, ws)
        ctx.save_for_backward(x2, weight)
        ctx.shape = shape
        return y.view(*shape[:-1], weight.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, weight = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16)
        dx = (dy2 @ weight.to(torch.bfloat16)).to(x2.dtype).view(ctx.shape)
        dw = (dy2.t().float() @ x2.float()).to(weight.dtype)
        return dx, dw, None


class FusedRowParallelOutput(torch.nn.Module):
    """Drop-in for the (bias-free) output projection of a tensor-parallel attention shard: the
    local partial product and its all-reduce over ``group`` run as one kernel on CUDA."""

    def __init__(self, linear: torch.nn.Linear, group=None):
        super().__init__()
        if linear.bias is not None:
            raise ValueError("the fused row-parallel output takes a bias-free projection")
        self.weight = linear.weight
        self.bias = None
        self.group = group
        self.in_features, self.out_features = linear.in_features, linear.out_features

    def forward(self, x):
        if x.is_cuda and self.out_features % 8 == 0:
            return _FusedRowParallel.apply(x, self.weight, self.group)
        from .tensor_parallel import reduce_from_tensor_parallel_region
        return reduce_from_tensor_parallel_region(torch.nn.functional.linear(x, self.weight.to(x.dtype)), self.group)


class AllGatherWorkspace:
    """Symmetric ``[row shard | flags]`` buffer for :func:`fused_allgather_matmul` (collective
    construction): each rank's bf16 shard ``[rows, cols]`` is read by every rank's GEMM."""

    _kimi_rendezvous = True  # one per process and peer set: model copies share it, never copy it

    _FLAGS = 1 << 12

    def __init__(self, group=None, device=None, *, rows: int, cols: int, timeout_s: float = 10.0):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.rank, self.world = dist.get_rank(self.group), dist.get_world_size(self.group)
        if self.world > 8 or rows % 128 or cols % 8:
            raise ValueError("fused all-gather GEMM: at most 8 ranks, rows % 128 == 0, cols % 8 == 0")
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.rows, self.cols = rows, cols
        full_rows = self.world * rows
        shard_bytes = _align(full_rows * cols * 2)
        buf = symm_mem.empty(shard_bytes + self._FLAGS, dtype=torch.uint8, device=self.device)
        buf.zero_()
        torch.cuda.synchronize(self.device)
        self.handle = symm_mem.rendezvous(buf, self.group)
        self.buffer = buf
        ptrs = [int(p) for p in self.handle.buffer_ptrs]
        self.buffer_peers = ptrs
        # [world * rows, cols] gather buffer; this rank's shard is its row block
        self.gather = buf[: full_rows * cols * 2].view(torch.bfloat16).view(full_rows, cols)
        self.shard = self.gather[self.rank * rows: (self.rank + 1) * rows]
        self.block_flags = torch.zeros(full_rows // 128, dtype=torch.int32, device=self.device)
        self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        flags = [p + shard_bytes for p in ptrs]
        # the flag-barrier kernels take the expert-parallel peer table; only its flag region is used
        self.peer_list = flags + [0] * (8 * self.world)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timeout_ns = int(timeout_s * 1e9)
        self.shard_bytes = shard_bytes
        dist.barrier(group=self.group)

    def barrier(self, kind: int) -> None:
        from ..ops import _loader
        _loader.require().ep_signal_wait(self.peer_list, self.rank, self.world, self.status, self.timeout_ns, kind)

    def check(self) -> None:
        code = int(self.status.item())
        if code:
            raise RuntimeError(f"fused all-gather GEMM failed (status {code}): a peer did not arrive in time")

    def reset(self) -> None:
        torch.cuda.synchronize(self.device)
        self.buffer[self.shard_bytes:].zero_()
        self.status.zero_()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)


def fused_allgather_matmul(x_shard: torch.Tensor, weight: torch.Tensor, workspace: AllGatherWorkspace, *,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """``all_gather(x_shard over the group) @ weight^T`` with the gather inside the GEMM.

    ``x_shard`` [rows, K] is this rank's block of rows (rank order); ``weight`` [N, K].  The shard
    is published in its row block of the workspace's gather buffer and a device-side flag barrier
    makes every shard visible; then ONE kernel computes the local rows' tiles first while its
    comm warps copy each remote 128-row block over NVLink into the local gather buffer (every
    byte crosses once) and release a per-block flag that the TMA producer waits on before the
    remote rows' tiles.  A second barrier keeps a rank from overwriting its shard while peers
    still read it.  Returns [world * rows, N] (bf16).

    Parity: replaces the all-gather before a sequence-parallel column-parallel projection (the
    reference's ``_CopyToRegion`` / all-gather path, ``training/distributed/tensor_parallel.py:25-60``)."""
    from ..ops import _loader
    C = _loader.require()
    ws = workspace
    rows, k = x_shard.shape
    if rows != ws.rows or k != ws.cols:
        raise ValueError("x_shard must match the workspace's [rows, cols]")
    w = weight.to(torch.bfloat16).contiguous()
    if out is None:
        out = torch.empty(ws.world * rows, w.shape[0], dtype=torch.bfloat16, device=x_shard.device)
    ws.shard.copy_(x_shard)
    ws.barrier(5)
    C.tc_gemm_allgather(ws.gather, w, ws.buffer_peers, ws.rank, rows, ws.block_flags, ws.epoch, ws.status, out,
                        256 if w.shape[0] >= 256 else 128)
    ws.epoch.add_(1)
    ws.barrier(6)
    return out


__all__ = ["SymmetricWorkspace", "workspace_for", "release_workspaces", "fused_matmul_reduce",
           "FusedRowParallelOutput", "AllGatherWorkspace", "fused_allgather_matmul"]
