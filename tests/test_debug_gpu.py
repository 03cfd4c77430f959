"""Out-of-bounds and race checks without a sanitizer: canary guard bands around kernel outputs
(every element outside the logical matrix must keep its canary) and repeat-run determinism."""
import pytest
import torch

from kimi_k3_b200.debug import Guarded, determinism

pytestmark = pytest.mark.gpu


def _C():
    from kimi_k3_b200.ops import _loader
    return _loader.require()


@pytest.mark.parametrize("m,n,k", [(300, 200, 640), (64, 1000, 640), (129, 2304, 1536), (1, 136, 256)])
def test_gemm_store_stays_inside_the_matrix(cuda, m, n, k):
    torch.manual_seed(m + n)
    a = torch.randn(m, k, device=cuda).bfloat16()
    b = torch.randn(n, k, device=cuda).bfloat16()
    g = Guarded(m, n, dtype=torch.bfloat16, device=cuda)
    _C().tc_gemm_dense(a, b, False, False, False, 256 if n >= 320 else 128, g.view)
    assert g.violations() == []
    want = (a.float() @ b.float().t())
    assert ((g.view.float() - want).norm() / want.norm()).item() < 1e-2


@pytest.mark.parametrize("m,n,k,splits", [(130, 1356, 1536, 4), (64, 640, 640, 2), (500, 328, 2048, 8)])
def test_split_k_reduce_adds_stay_inside_the_matrix(cuda, m, n, k, splits):
    torch.manual_seed(k)
    a = torch.randn(m, k, device=cuda).bfloat16()
    b = torch.randn(n, k, device=cuda).bfloat16()
    g = Guarded(m, n, dtype=torch.float32, device=cuda)
    _C().tc_gemm_dense(a, b, False, False, True, 128, g.view, accumulate=True, ksplit=splits)
    assert g.violations() == []
    want = a.float() @ b.float().t()
    assert ((g.view - want).norm() / want.norm()).item() < 1e-3


def test_projection_group_segments_stay_inside_their_outputs(cuda):
    torch.manual_seed(5)
    widths = (640, 128, 64, 12)
    x = torch.randn(333, 640, device=cuda).bfloat16()
    w = torch.randn(sum(widths), 640, device=cuda).bfloat16()
    guards = [Guarded(333, wd, dtype=torch.bfloat16, device=cuda) for wd in widths]
    _C().tc_gemm_group(1, [g.view for g in guards], x, w, None, 256, 1, -1)
    off = 0
    for g, wd in zip(guards, widths):
        # a ragged last segment has its columns up to the next multiple of 8 written (zeros; the
        # binding requires the row stride to hold them): nothing else of the guard band may change
        pad8 = -(-wd // 8) * 8
        rest = [(r, c, v) for r, c, v in g.violations(limit=100000)
                if not (0 <= r < 333 and wd <= c < pad8 and v == 0)]
        assert rest == [], (wd, rest[:4])
        want = x.float() @ w[off:off + wd].float().t()
        assert ((g.view.float() - want).norm() / want.norm()).item() < 1e-2
        off += wd


def test_repeat_runs(cuda):
    """Kernels without reductions across CTAs are bitwise deterministic; split-K reduce-adds may
    differ in the last bits only."""
    from kimi_k3_b200 import ops
    torch.manual_seed(1)
    a = torch.randn(1000, 640, device=cuda).bfloat16()
    b = torch.randn(960, 640, device=cuda).bfloat16()
    C = _C()
    rep = determinism(lambda: C.tc_gemm_dense(a, b, False, False, False, 256, None), runs=4)
    assert rep[0]["bitwise"]

    def split():
        out = torch.zeros(96, 960, device=cuda)
        C.tc_gemm_dense(a[:96], b, False, False, True, 128, out, accumulate=True, ksplit=4)
        return out
    rep = determinism(split, runs=4)
    assert rep[0]["max_abs_diff"] < 1e-3
    x = torch.randn(4, 256, 640, device=cuda).bfloat16()
    wconv = 0.3 * torch.randn(640, 4, device=cuda)
    rep = determinism(lambda: ops.conv_silu_norm(x, wconv, 64, 1e-6, True), runs=3)
    assert all(r["bitwise"] for r in rep)
    w = torch.rand(640, device=cuda) + 0.5
    rep = determinism(lambda: ops.rms_norm(x, w, 1e-6), runs=3)
    assert all(r["bitwise"] for r in rep)
