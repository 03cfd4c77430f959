"""Debugging aids: NVTX ranges, canary guard bands around kernel outputs, repeat-run determinism.

The reference has no race detection or profiler hooks; compute-sanitizer is not available on the
target machines.  These are the substitutes:

* :func:`nvtx` -- a named range (``torch.cuda.nvtx``) around a region when ``KIMI_K3_NVTX=1``;
  the model marks each hybrid layer, the expert exchange and the tensor-parallel collectives, the
  trainer marks forward / backward / gradient sync / optimizer.  Off, a range is one flag check.
* :class:`Guarded` -- an output matrix placed inside a larger buffer whose surrounding rows and
  columns hold a canary value; after a kernel wrote the matrix, :meth:`Guarded.violations` lists
  every canary element that changed (a write past the logical edge: a bad tile clip, a wrong
  stride, a race into a neighbour's rows).
* :func:`determinism` -- run a function several times on the same inputs and report, per output,
  whether the runs agree bitwise and the largest difference (split-K reductions and atomics
  legitimately differ in the last bits; anything else that differs is a race).
"""
from __future__ import annotations

import os
from contextlib import contextmanager, nullcontext

import torch

_NVTX = os.environ.get("KIMI_K3_NVTX", "0") not in ("", "0")


def nvtx_enabled() -> bool:
    return _NVTX


def set_nvtx(enabled: bool) -> None:
    """Turn the ranges on or off for this process (``KIMI_K3_NVTX`` sets the initial state)."""
    global _NVTX
    _NVTX = bool(enabled)


@contextmanager
def _range(name: str):
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()


def nvtx(name: str):
    """``with nvtx("layer 3"):`` -- a named NVTX range when enabled and CUDA is present."""
    if _NVTX and torch.cuda.is_available():
        return _range(name)
    return nullcontext()


class Guarded:
    """A ``[rows, cols]`` matrix inside a ``[rows + 2 * pad, ld]`` buffer (``ld >= cols + pad``)
    whose other elements hold ``canary``.  ``view`` is the matrix (row stride ``ld``)."""

    def __init__(self, rows: int, cols: int, *, dtype=torch.float32, device="cuda", pad: int = 8,
                 canary: float = -12345.0, fill: float | None = 0.0):
        self.rows, self.cols, self.pad = int(rows), int(cols), int(pad)
        align = 8  # row stride in elements: a multiple of 8 keeps rows 16-byte aligned for every dtype
        self.ld = -(-(self.cols + self.pad) // align) * align
        self.canary = canary
        self.buffer = torch.full((self.rows + 2 * self.pad, self.ld), canary, dtype=dtype, device=device)
        self.view = self.buffer[self.pad:self.pad + self.rows, :self.cols]
        if fill is not None:
            self.view.fill_(fill)

    def violations(self, limit: int = 16) -> list:
        """Up to ``limit`` ``(row, col, value)`` entries of the guard band that no longer hold the
        canary (row / col relative to the matrix origin; negative rows lie above it)."""
        band = torch.ones_like(self.buffer, dtype=torch.bool)
        band[self.pad:self.pad + self.rows, :self.cols] = False
        want = torch.tensor(self.canary, dtype=self.buffer.dtype, device=self.buffer.device)
        bad = band & (self.buffer != want)
        idx = bad.nonzero()[:limit].tolist()
        return [(r - self.pad, c, float(self.buffer[r, c])) for r, c in idx]


def _flatten_outputs(out):
    if torch.is_tensor(out):
        return [out]
    if isinstance(out, (tuple, list)):
        return [t for o in out for t in _flatten_outputs(o)]
    if isinstance(out, dict):
        return [t for v in out.values() for t in _flatten_outputs(v)]
    return []


def determinism(fn, *args, runs: int = 3, **kwargs) -> list:
    """Call ``fn(*args, **kwargs)`` ``runs`` times; for each tensor output return
    ``{"index", "bitwise", "max_abs_diff"}`` against the first run."""
    first = [t.detach().clone() for t in _flatten_outputs(fn(*args, **kwargs))]
    worst = [0.0] * len(first)
    same = [True] * len(first)
    for _ in range(runs - 1):
        outs = _flatten_outputs(fn(*args, **kwargs))
        if len(outs) != len(first):
            raise RuntimeError("the function returned a different number of tensors on a repeat run")
        for i, (a, b) in enumerate(zip(first, outs)):
            if not torch.equal(a, b.detach()):
                same[i] = False
                if a.is_floating_point():
                    worst[i] = max(worst[i], (a.double() - b.detach().double()).abs().max().item())
                else:
                    worst[i] = max(worst[i], float((a != b.detach()).sum().item()))
    return [{"index": i, "bitwise": same[i], "max_abs_diff": worst[i]} for i in range(len(first))]


__all__ = ["nvtx", "nvtx_enabled", "set_nvtx", "Guarded", "determinism"]
