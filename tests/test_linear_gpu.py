"""Projections on the tcgen05 GEMM (``ops.linear``) and the bf16 weight mirrors, against fp32 torch."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("shape", [(4, 333, 640, 640), (2, 1024, 1920, 640), (3, 100, 12, 640), (1, 512, 640, 64),
                                   (64, 1, 1536, 1536), (2, 16, 768, 2048)])
@pytest.mark.parametrize("bias", [False, True])
def test_linear_forward_backward(cuda, shape, bias):
    from kimi_k3_b200.models.linear import Linear
    b, t, n, k = shape
    torch.manual_seed(n + k + t)
    lin = Linear(k, n, bias=bias).to(cuda)
    x = torch.randn(b, t, k, device=cuda, requires_grad=True)
    dy = torch.randn(b, t, n, device=cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = lin(x)
    assert y.dtype == torch.bfloat16
    y.backward(dy.bfloat16())
    # fp32 reference on the bf16-rounded operands
    xr = x.detach().bfloat16().float().requires_grad_()
    wr = lin.weight.detach().bfloat16().float().requires_grad_()
    br = lin.bias.detach().clone().requires_grad_() if bias else None
    yr = F.linear(xr, wr, br)
    yr.backward(dy.bfloat16().float())
    assert _rel(y, yr) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2
    assert lin.weight.grad.dtype == torch.float32
    assert _rel(lin.weight.grad, wr.grad) < 1e-3
    if bias:
        assert _rel(lin.bias.grad, br.grad) < 1e-3


def test_weight_mirror_refresh_and_staleness(cuda):
    from kimi_k3_b200.models.linear import Linear
    from kimi_k3_b200.ops.mirror import WeightMirror, bf16_weight
    torch.manual_seed(0)
    lins = [Linear(640, n).to(cuda) for n in (640, 12, 1920)]
    mirror = WeightMirror([l.weight for l in lins])
    for l in lins:
        assert torch.equal(bf16_weight(l.weight), l.weight.detach().bfloat16())
    # an update the optimizer makes through raw pointers leaves the version alone: refresh() picks it up
    with torch.no_grad():
        for l in lins:
            l.weight.data.mul_(0.5)
    mirror.refresh()
    for l in lins:
        assert torch.equal(bf16_weight(l.weight), l.weight.detach().bfloat16())
    # a change through PyTorch bumps the version: the next use re-casts that weight
    with torch.no_grad():
        lins[1].weight.copy_(torch.randn_like(lins[1].weight))
    assert mirror.stale()
    assert torch.equal(bf16_weight(lins[1].weight), lins[1].weight.detach().bfloat16())


def test_optimizer_step_keeps_mirrors_current(cuda):
    from kimi_k3_b200.models.linear import Linear
    from kimi_k3_b200.ops.mirror import bf16_weight
    torch.manual_seed(0)
    net = torch.nn.Sequential(Linear(64, 128), torch.nn.GELU(), Linear(128, 64)).to(cuda)
    from kimi_k3_b200.train.optimizer import build_weight_mirror
    mirror = build_weight_mirror(net)
    assert mirror is not None and len(mirror.params) == 2
    opt = torch.optim.SGD(net.parameters(), lr=0.1)
    x = torch.randn(32, 64, device=cuda)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        net(x).float().square().mean().backward()
    opt.step()  # bumps versions: bf16_weight re-casts on demand even without a refresh
    for m in (net[0], net[2]):
        assert torch.equal(bf16_weight(m.weight), m.weight.detach().bfloat16())


def test_tc_gemm_group_three_kinds(cuda):
    """Segmented products of one projection group against fp32 torch: per-segment outputs, the
    K-segmented input gradient and the M-segmented weight gradients."""
    from kimi_k3_b200.ops import _loader
    C = _loader.require()
    torch.manual_seed(9)
    m, k = 1000, 640
    widths = [640, 128, 64, 10]
    w = [(torch.randn(n, k, device=cuda) / k ** 0.5).bfloat16() for n in widths]
    wcat = torch.cat(w, 0)
    x = torch.randn(m, k, device=cuda).bfloat16()
    outs = [torch.empty(m, -(-n // 8) * 8, device=cuda, dtype=torch.bfloat16)[:, :n] for n in widths]
    C.tc_gemm_group(1, outs, x, wcat, None, 256, 1, -1)
    for o, wi in zip(outs, w):
        ref = x.float() @ wi.float().t()
        assert _rel(o, ref) < 1e-2
    dys = [torch.randn(m, n, device=cuda).bfloat16() for n in widths]
    segs = [d if n % 8 == 0 else F.pad(d, (0, -(-n // 8) * 8 - n)).contiguous() for d, n in zip(dys, widths)]
    for pair in (0, 1):
        dx = torch.empty(m, k, device=cuda, dtype=torch.bfloat16)
        C.tc_gemm_group(2, segs, x, wcat, dx, 256, 1, pair)
        ref = sum(d.float() @ wi.float() for d, wi in zip(dys, w))
        assert _rel(dx, ref) < 1e-2
        dw = torch.zeros(sum(widths), k, device=cuda)
        C.tc_gemm_group(3, segs, x, wcat, dw, 256, 3, pair)
        ref = torch.cat([d.float().t() @ x.float() for d in dys], 0)
        assert _rel(dw, ref) < 1e-3


# 32 rows with a total width that is a multiple of 4: the split-K path for few rows (decode)
@pytest.mark.parametrize("rows,last", [(300, 10), (32, 12)])
def test_linear_group_matches_separate_projections(cuda, rows, last):
    from kimi_k3_b200.models.linear import Linear
    from kimi_k3_b200.ops import linear_group
    from kimi_k3_b200.ops.mirror import WeightMirror
    torch.manual_seed(4)
    lins = [Linear(640, n, bias=False).to(cuda) for n in (640, 640, 64, last)]
    mirror = WeightMirror([], groups=[[l.weight for l in lins]])
    x = torch.randn(2, rows, 640, device=cuda, requires_grad=True)
    dys = [torch.randn(2, rows, l.out_features, device=cuda) for l in lins]
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ys = linear_group(x, [l.weight for l in lins])
    sum((y.float() * d).sum() for y, d in zip(ys, dys)).backward()
    xr = x.detach().bfloat16().float().requires_grad_()
    ws = [l.weight.detach().bfloat16().float().requires_grad_() for l in lins]
    sum((F.linear(xr, wr) * d).sum() for wr, d in zip(ws, dys)).backward()
    for y, wr in zip(ys, ws):
        assert _rel(y, F.linear(xr, wr)) < 1e-2
    assert _rel(x.grad, xr.grad) < 1e-2
    for l, wr in zip(lins, ws):
        assert l.weight.grad.dtype == torch.float32 and _rel(l.weight.grad, wr.grad) < 1e-2
    assert mirror.params  # the group's mirrors were registered


def _ns_fp32(w, steps):
    """The quintic Newton-Schulz iterations in fp32 PyTorch (``a X + (b G + c G^2) X``)."""
    from kimi_k3_b200.train.optimizer import NS_COEFFS
    a, b, c = NS_COEFFS
    x = w.float()
    for _ in range(steps):
        g = x @ x.transpose(-2, -1)
        x = a * x + (b * g + c * g @ g) @ x
    return x


@pytest.mark.parametrize("e,m,n,transposed", [(3, 64, 640, False), (2, 640, 960, False), (4, 320, 640, True),
                                               (1, 128, 2560, False)])
def test_newton_schulz_on_tensor_cores(cuda, e, m, n, transposed):
    """The grouped tcgen05 Newton-Schulz (padded segments, K-major Gram products, MN-major update)
    against fp32 PyTorch on the same bf16-normalised input; ``transpose_out`` returns X^T."""
    from kimi_k3_b200.train.optimizer import _ns_on_tensor_cores, newton_schulz_iterations
    torch.manual_seed(3)
    raw = torch.randn(e, n, m, device=cuda) if transposed else torch.randn(e, m, n, device=cuda)
    w = raw.transpose(-2, -1) if transposed else raw
    w = (w / w.flatten(1).norm(dim=1)[:, None, None]).to(torch.bfloat16)
    assert _ns_on_tensor_cores(w)
    got = newton_schulz_iterations(w, 5, transpose_out=transposed, tensor_cores=True).float()
    want = _ns_fp32(w, 5)
    if transposed:
        want = want.transpose(-2, -1)
    assert got.shape == want.shape
    err = (got - want).norm() / want.norm()
    assert err < 3e-2, float(err)
    # the result is near-orthogonal: singular values inside the quintic's band
    sv = torch.linalg.svdvals(got.transpose(-2, -1) if transposed else got)
    assert float(sv.max()) < 1.3 and float(sv.min()) > 0.5
