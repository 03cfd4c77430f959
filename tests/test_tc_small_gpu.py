"""The small-matrix tcgen05 path (thread-written 128B-swizzled tf32 operands, TMEM
accumulators) against fp32 torch products: full products at several N and K, K slices and
B row offsets (the addressing the chunked KDA kernels use)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from kimi_k3_b200.ops import _loader
    return _loader.require()


def _rel(a, b):
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("n,k", [(16, 32), (64, 64), (128, 64), (192, 128), (256, 64)])
def test_full_product(cuda, n, k):
    torch.manual_seed(n + k)
    a = torch.randn(128, k, device=cuda)
    b = torch.randn(n, k, device=cuda)
    out, status = _C().tcs_selftest(a, b, n, 0)
    assert status.item() == 0
    assert _rel(out, a @ b.t()) < 2e-3  # tf32 operands


def test_k_slices(cuda):
    torch.manual_seed(1)
    a = torch.randn(128, 64, device=cuda)
    b = torch.randn(64, 64, device=cuda)
    out, status = _C().tcs_selftest(a, b, 64, 1)
    assert status.item() == 0
    ref = torch.cat([a[:, 16 * i:16 * i + 16] @ b[:, 16 * i:16 * i + 16].t() for i in range(4)], 1)
    assert _rel(out, ref) < 2e-3


def test_b_row_offsets(cuda):
    torch.manual_seed(2)
    a = torch.randn(128, 64, device=cuda)
    b = torch.randn(64, 64, device=cuda)
    out, status = _C().tcs_selftest(a, b, 16, 2)
    assert status.item() == 0
    ref = torch.cat([a @ b[16 * j:16 * j + 16].t() for j in range(4)], 1)
    assert _rel(out, ref) < 2e-3
