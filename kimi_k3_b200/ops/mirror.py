"""bf16 mirrors of fp32 master weights for the tensor-core projections.

Training keeps fp32 master weights (the optimizer state and update are fp32) while every
projection runs on bf16 operands.  Casting each weight inside every forward costs one read of
the fp32 tensor and one write of a bf16 copy per use; on the flagship step those casts were
several milliseconds of copy kernels.  A :class:`WeightMirror` keeps one persistent bf16 copy
per registered weight instead and refreshes all of them with one launch right after the
optimizer has written the masters (``refresh``), so a forward reads 2 bytes per weight element
and casts nothing.

Staleness: a mirror records the parameter's version counter and storage address at refresh
time.  Anything that changes a master outside the optimizer through PyTorch (``load_state_dict``,
``copy_``, an EMA swap, re-initialisation) bumps that counter, and :func:`bf16_weight` then
re-casts the one weight on its next use.  CUDA-graph replays run no Python, so the step engine
calls :meth:`WeightMirror.refresh_if_stale` before each replay.
"""
from __future__ import annotations

import weakref

import torch

from . import _loader

_REGISTRY: "weakref.WeakValueDictionary[int, _Entry]" = weakref.WeakValueDictionary()
# projection groups: tuple of parameter ids -> the bf16 buffer their mirrors are row slices of
_GROUPS: "dict[tuple, torch.Tensor]" = {}


class _Entry:
    __slots__ = ("param_ref", "mirror", "version", "ptr", "owner", "__weakref__")

    def __init__(self, param, mirror, owner):
        self.param_ref = weakref.ref(param)
        self.mirror = mirror
        self.version = -1
        self.ptr = -1
        self.owner = owner

    def fresh(self, p) -> bool:
        return p._version == self.version and p.data_ptr() == self.ptr


class WeightMirror:
    """Persistent bf16 copies of a set of fp32 CUDA parameters."""

    def __init__(self, params, groups=()):
        """``groups``: lists of 2-D weights with equal column counts that one fused projection reads as
        a single ``[sum of rows, cols]`` matrix; their mirrors become row slices of one buffer."""
        params = list(params)
        group_of = {}
        for grp in groups:
            grp = [p for p in grp]
            if len(grp) < 2 or any(p.ndim != 2 or p.shape[1] != grp[0].shape[1] or not p.is_cuda
                                   or p.dtype != torch.float32 for p in grp):
                continue
            buf = torch.empty(sum(p.shape[0] for p in grp), grp[0].shape[1], dtype=torch.bfloat16,
                              device=grp[0].device)
            row = 0
            for p in grp:
                group_of[id(p)] = buf[row:row + p.shape[0]]
                row += p.shape[0]
            _GROUPS[tuple(id(p) for p in grp)] = buf
            params.extend(grp)
        seen, ps = set(), []
        for p in params:
            if id(p) in seen or not isinstance(p, torch.Tensor) or not p.is_cuda or p.dtype != torch.float32:
                continue
            if p.data_ptr() % 16 or p.numel() == 0 or not p.is_contiguous():
                continue
            seen.add(id(p))
            ps.append(p)
        self.params = ps
        self.entries = []
        self._tables = None
        self._ptrs = []
        self._total_vec = 0
        for p in ps:
            mirror = group_of.get(id(p))
            if mirror is None:
                mirror = torch.empty(p.shape, dtype=torch.bfloat16, device=p.device)
            e = _Entry(p, mirror, self)
            self.entries.append(e)
            _REGISTRY[id(p)] = e
        self.refresh()

    def _build_tables(self):
        n = len(self.params)
        rows = torch.zeros(4, n + 1, dtype=torch.int64)
        vec = 0
        for i, (p, e) in enumerate(zip(self.params, self.entries)):
            rows[0, i] = p.data_ptr()
            rows[1, i] = e.mirror.data_ptr()
            rows[2, i] = p.numel()
            rows[3, i] = vec
            vec += (p.numel() + 7) // 8
        rows[3, n] = vec
        self._tables = rows.to(self.params[0].device)
        self._total_vec = vec
        self._ptrs = [p.data_ptr() for p in self.params]

    @torch.no_grad()
    def refresh(self) -> None:
        """Re-cast every mirror from its master (one launch, stream-ordered)."""
        if not self.params:
            return
        if self._tables is None or any(p.data_ptr() != q for p, q in zip(self.params, self._ptrs)):
            self._build_tables()
        _loader.require().cast_bf16_multi(self._tables, len(self.params), self._total_vec)
        for p, e in zip(self.params, self.entries):
            e.version = p._version
            e.ptr = p.data_ptr()

    def stale(self) -> bool:
        return any(not e.fresh(p) for p, e in zip(self.params, self.entries))

    def refresh_if_stale(self) -> bool:
        if self.stale():
            self.refresh()
            return True
        return False


def bf16_weight(p: torch.Tensor) -> torch.Tensor:
    """The bf16 operand for weight ``p``: its mirror when one is registered (re-cast first if the
    master changed outside the optimizer), else a fresh cast."""
    if p.dtype == torch.bfloat16:
        return p
    e = _REGISTRY.get(id(p))
    if e is None or e.param_ref() is not p:
        return p.detach().to(torch.bfloat16)
    if not e.fresh(p):
        with torch.no_grad():
            e.mirror.copy_(p)
        e.version = p._version
        e.ptr = p.data_ptr()
    return e.mirror


def group_weight(params) -> torch.Tensor:
    """The concatenated bf16 ``[sum of rows, cols]`` operand of a projection group: the shared mirror
    buffer when the group is registered (stale members re-cast first), else a fresh concatenation."""
    buf = _GROUPS.get(tuple(id(p) for p in params))
    if buf is not None:
        views = [bf16_weight(p) for p in params]  # refreshes stale members in place
        if all(v.data_ptr() == buf[0].data_ptr() + off * buf.stride(0) * buf.element_size()
               for v, off in zip(views, _offsets(params))):
            return buf
    return torch.cat([bf16_weight(p) for p in params], 0)


def _offsets(params):
    out, row = [], 0
    for p in params:
        out.append(row)
        row += p.shape[0]
    return out


def mirror_for(p: torch.Tensor):
    e = _REGISTRY.get(id(p))
    return None if e is None or e.param_ref() is not p else e.owner


__all__ = ["WeightMirror", "bf16_weight", "group_weight", "mirror_for"]
