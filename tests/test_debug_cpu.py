"""Debugging aids on CPU: canary guard bands, the repeat-run determinism report, NVTX ranges."""
import torch

from kimi_k3_b200.debug import Guarded, determinism, nvtx, set_nvtx


def test_guarded_detects_writes_past_the_matrix():
    g = Guarded(5, 7, dtype=torch.float32, device="cpu", pad=3)
    assert g.view.shape == (5, 7) and g.buffer.stride(0) % 8 == 0
    g.view.copy_(torch.randn(5, 7))
    assert g.violations() == []
    g.buffer[g.pad + 2, 7] = 1.0       # one column past the right edge
    g.buffer[g.pad - 1, 0] = 2.0       # the row above the matrix
    bad = g.violations()
    assert (2, 7, 1.0) in bad and (-1, 0, 2.0) in bad and len(bad) == 2


def test_determinism_report():
    x = torch.randn(64, 64)
    rep = determinism(lambda t: (t @ t, t.sum()), x, runs=3)
    assert all(r["bitwise"] for r in rep)
    gen = torch.Generator().manual_seed(0)
    rep = determinism(lambda: torch.rand(4, generator=gen), runs=2)
    assert not rep[0]["bitwise"] and rep[0]["max_abs_diff"] > 0


def test_nvtx_ranges_are_noops_without_cuda():
    set_nvtx(True)
    try:
        with nvtx("layer 0 kda"):
            y = torch.ones(2) * 2
    finally:
        set_nvtx(False)
    assert y.sum().item() == 4.0
