"""Projections on the tcgen05 GEMM (``ops.linear``) and the bf16 weight mirrors, against fp32 torch."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("shape", [(4, 333, 640, 640), (2, 1024, 1920, 640), (3, 100, 12, 640), (1, 512, 640, 64)])
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
