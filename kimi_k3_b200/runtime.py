"""Process-wide execution switches.

``sync_free()`` marks a region whose device work must not wait for the host: a CUDA-graph
capture of a whole training step, or a replay-driven loop. Inside it the model and the
optimizer skip every check that reads a device value on the host (``.item()``, ``bool(t)``,
``.tolist()``): non-finite and out-of-range validations, all-true mask shortcuts and
zero-token guards. The caller performs the equivalent checks on the host copy of the batch
(see ``kimi_k3_b200.train.engine``), and the optimizer turns the finite-gradient check into a
device flag that suppresses the update instead of a Python branch.
"""
from __future__ import annotations

import threading
from contextlib import contextmanager

_local = threading.local()


def host_checks() -> bool:
    """True unless inside :func:`sync_free` (host-side validation allowed)."""
    return not getattr(_local, "sync_free", False)


def mask_all_valid() -> bool:
    """Inside :func:`sync_free`: the caller has verified on the host that every attention-mask
    entry of the batch is True, so layers may take their mask-free paths without looking."""
    return getattr(_local, "all_valid", False)


@contextmanager
def sync_free(enabled: bool = True, *, all_valid_mask: bool = False):
    prev = (getattr(_local, "sync_free", False), getattr(_local, "all_valid", False))
    _local.sync_free = bool(enabled) or prev[0]
    _local.all_valid = bool(enabled and all_valid_mask)
    try:
        yield
    finally:
        _local.sync_free, _local.all_valid = prev


__all__ = ["host_checks", "mask_all_valid", "sync_free"]
