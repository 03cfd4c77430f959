"""Device-initiated expert-parallel exchange (``ep_comm.cu`` + the remote-combine GEMM epilogue).

* one rank: the whole dispatch / expert GEMMs / combine / backward path against the local grouped
  expert kernels, for the output, the latent and routing-weight gradients and the expert weight
  gradients, over repeated calls (the counting semaphores must balance);
* one rank with a fake second rank that never signals: the count exchange runs out (bounded),
  the status word reports it, and after ``reset()`` the workspace works again;
* two ranks (needs 2 GPUs): against the local kernels run on the gathered tokens with all experts.

Children run in subprocesses (process groups and symmetric memory stay out of pytest); the
two-rank case uses torchrun on 127.0.0.1 with a hard timeout and NVLS disabled.
"""
import os
import socket
import subprocess
import sys
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HERE = os.path.abspath(__file__)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _run(args, timeout=300):
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""), NCCL_NVLS_ENABLE="0")
    r = subprocess.run(args, env=env, capture_output=True, text=True, timeout=timeout)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
    return r.stdout


def test_ep_fused_one_rank(cuda):
    assert "one-rank ok" in _run([sys.executable, HERE, "one", str(_free_port())])


def test_ep_fused_timeout_status(cuda):
    assert "timeout ok" in _run([sys.executable, HERE, "timeout", str(_free_port())])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_fused_two_ranks():
    out = _run(["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}", HERE, "multi"],
               timeout=300)
    assert "multi-rank ok" in out


# ---------------------------------------------------------------------------- children
def _init(rank, world, port=None):
    import datetime
    import torch.distributed as dist
    if port is not None:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    return dist


def _rel(a, b):
    return (a.float() - b.float()).abs().max().item() / max(b.float().abs().max().item(), 1e-6)


def _experts(e, h, l, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, device="cuda", generator=g) * 0.05)  # noqa: E731
    return mk(e, h, l), mk(e, h, l), mk(e, l, h)


def _tokens(m, l, e, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, l, device="cuda", generator=g).bfloat16()
    sel = torch.stack([torch.randperm(e, device="cuda", generator=g)[:k] for _ in range(m)])
    w = torch.rand(m, k, device="cuda", generator=g)
    return x, sel, w / w.sum(-1, keepdim=True)


def _run_fused(ws, x, sel, w, gate, up, down, dout):
    from kimi_k3_b200.parallel.ep_fused import fused_ep_experts
    xl = x.clone().requires_grad_()
    wl = w.clone().requires_grad_()
    ex = SimpleNamespace(gate_proj=gate.clone().requires_grad_(), up_proj=up.clone().requires_grad_(),
                         down_proj=down.clone().requires_grad_())
    y = fused_ep_experts(xl, sel, wl, ex, ws, 4.0, 25.0)
    y.backward(dout)
    return y, xl.grad, wl.grad, ex.gate_proj.grad, ex.up_proj.grad, ex.down_proj.grad


def _run_local(x, sel, w, gate, up, down, dout):
    from kimi_k3_b200 import ops
    xl = x.clone().requires_grad_()
    wl = w.clone().requires_grad_()
    gp, upp, dp = (t.clone().requires_grad_() for t in (gate, up, down))
    y = ops.moe_grouped_experts(xl, sel, wl, gp, upp, dp, 4.0, 25.0)
    y.backward(dout)
    return y, xl.grad, wl.grad, gp.grad, upp.grad, dp.grad


def child_one(port):
    dist = _init(0, 1, port)
    from kimi_k3_b200.parallel.ep_fused import EPWorkspace
    e, k, l, h, m = 12, 2, 320, 640, 1000
    gate, up, down = _experts(e, h, l)
    ws = EPWorkspace(None, "cuda:0", tokens=m, top_k=k, latent=l, num_experts=e)
    for it in range(3):
        x, sel, w = _tokens(m, l, e, k, seed=it)
        dout = torch.randn(m, l, device="cuda")
        got = _run_fused(ws, x, sel, w, gate, up, down, dout)
        ref = _run_local(x, sel, w, gate, up, down, dout)
        for name, a, b in zip(("y", "dx", "dw", "dgate", "dup", "ddown"), got, ref):
            r = _rel(a, b)
            assert r < 2e-2, (it, name, r)
    ws.check()
    dist.destroy_process_group()
    print("one-rank ok")


def child_timeout(port):
    dist = _init(0, 1, port)
    from kimi_k3_b200.ops import _loader
    from kimi_k3_b200.parallel.ep_fused import EPWorkspace
    C = _loader.require()
    e, k, l, m = 4, 2, 64, 64
    ws = EPWorkspace(None, "cuda:0", tokens=m, top_k=k, latent=l, num_experts=e, timeout_s=0.2)
    fake = EPWorkspace(None, "cuda:0", tokens=m, top_k=k, latent=l, num_experts=e)  # a "rank" that never runs
    # world 2: region-major peer list with the fake rank's regions as rank 1
    ptrs = []
    for i in range(9):
        ptrs += [ws.peer_list[i], fake.peer_list[i]]
    _, sel, _ = _tokens(m, l, e, k, seed=0)
    C.ep_count(sel, e, ws.cnt, ws.agg)
    offs = torch.zeros(e // 2 + 1, dtype=torch.int32, device="cuda")
    C.ep_exchange(ptrs, 0, 2, ws.status, ws.timeout_ns, ws.cnt, e, e // 2, l, offs, ws.base, ws.cursor)
    torch.cuda.synchronize()
    assert int(ws.status.item()) == 6, int(ws.status.item())
    try:
        ws.check()
        raise AssertionError("check() did not raise")
    except RuntimeError:
        pass
    ws.reset()
    gate, up, down = _experts(e, 128, l)
    x, sel, w = _tokens(m, l, e, k, seed=1)
    dout = torch.randn(m, l, device="cuda")
    got = _run_fused(ws, x, sel, w, gate, up, down, dout)
    ref = _run_local(x, sel, w, gate, up, down, dout)
    assert _rel(got[0], ref[0]) < 2e-2
    ws.check()
    dist.destroy_process_group()
    print("timeout ok")


def child_multi():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist = _init(rank, world)
    from kimi_k3_b200.parallel.ep_fused import EPWorkspace
    e, k, l, h, m = 12, 2, 320, 640, 2048
    per = e // world
    gate, up, down = _experts(e, h, l)           # identical on every rank (same seed)
    ws = EPWorkspace(None, f"cuda:{rank}", tokens=m, top_k=k, latent=l, num_experts=e)
    sl = slice(rank * per, (rank + 1) * per)
    for it in range(3):
        x, sel, w = _tokens(m, l, e, k, seed=100 * it + rank)
        dout = torch.randn(m, l, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7 + rank))
        got = _run_fused(ws, x, sel, w, gate[sl], up[sl], down[sl], dout)
        ref = _run_local(x, sel, w, gate, up, down, dout)
        for name, a, b in zip(("y", "dx", "dw"), got[:3], ref[:3]):
            r = _rel(a, b)
            assert r < 2e-2, (rank, it, name, r)
        # expert weight gradients: the sum over every rank's tokens of this rank's experts
        for name, a, b in zip(("dgate", "dup", "ddown"), got[3:], ref[3:]):
            full = b.float().contiguous()
            dist.all_reduce(full)
            r = _rel(a, full[sl])
            assert r < 2e-2, (rank, it, name, r)
    ws.check()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("multi-rank ok")


if __name__ == "__main__":
    which = sys.argv[1]
    if which == "one":
        child_one(int(sys.argv[2]))
    elif which == "timeout":
        child_timeout(int(sys.argv[2]))
    else:
        child_multi()
