"""Locate and load the in-tree CUDA extension (``kimi_k3_b200/_C*.so``).

The extension is built in place by ``python setup.py build_ext --inplace`` (or
``__graft_entry__.build()``) for ``sm_100a``.  ``require()`` raises with the build
command when the shared object is missing, so a GPU run never silently drops
to PyTorch math.
"""
from __future__ import annotations

import importlib

_EXT = None
_ERROR: Exception | None = None


def load():
    """Return the extension module or ``None`` if it cannot be imported."""
    global _EXT, _ERROR
    if _EXT is not None:
        return _EXT
    if _ERROR is not None:
        return None
    try:
        import torch  # noqa: F401  (the extension links against libtorch)
        _EXT = importlib.import_module("kimi_k3_b200._C")
    except Exception as exc:  # pragma: no cover - depends on the build
        _ERROR = exc
        return None
    return _EXT


def require():
    ext = load()
    if ext is None:
        raise RuntimeError(
            "kimi_k3_b200 CUDA extension is not built or failed to load "
            f"({_ERROR!r}); build it with `python setup.py build_ext --inplace` "
            "or set KIMI_K3_KERNELS=0 to run the PyTorch reference math on the GPU")
    return ext


def has(op: str) -> bool:
    ext = load()
    return ext is not None and hasattr(ext, op)
