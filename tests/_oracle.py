"""Helpers shared by the CPU oracle tests: the reference package import and weight mapping."""
import pytest
import torch

from conftest import import_reference, reference_available

needs_reference = pytest.mark.skipif(not reference_available(), reason="reference package not installed")


def ref():
    """Make the reference package importable (it is installed under ``baseline/_ref``)."""
    import_reference()


def expand_expert_grads(named_grads):
    """Stacked routed-expert gradients ``[E,...]`` -> the reference's per-expert parameter names."""
    out = {}
    for n, g in named_grads:
        if g is None:
            continue
        if n.endswith(("routed_experts.gate_proj", "routed_experts.up_proj", "routed_experts.down_proj")):
            pre, name = n.rsplit(".", 1)
            for e in range(g.shape[0]):
                out[f"{pre}.{e}.transform.{name}.weight"] = g[e]
        else:
            out[n] = g
    return out


def max_diff(a, b):
    return (a.double() - b.double()).abs().max().item()
