"""Fused tcgen05 GEMM + cross-rank reduction (symmetric memory, NVLS or peer loads).

* one rank: the fused kernel's data path and flag protocol against ``x @ w^T``;
* one rank, a fake second rank whose flags nobody sets: every wait runs out (bounded), the kernel
  returns with the timeout status, and the workspace is usable again after ``reset()``;
* two ranks (needs 2 GPUs): all-reduce and reduce-scatter, multicast and peer paths, against
  NCCL's all-reduce of the fp32 partial products, over repeated calls;
* the all-gather fused into a GEMM's A operand (one rank and two ranks) against NCCL's
  all-gather followed by the product.

Each case runs in child processes (process groups and symmetric memory stay out of the pytest
process); the multi-rank case uses torchrun on 127.0.0.1 with a hard timeout.
"""
import os
import socket
import subprocess
import sys

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


def test_fused_reduce_one_rank(cuda):
    out = _run([sys.executable, HERE, "one", str(_free_port())])
    assert "one-rank ok" in out


def test_fused_reduce_timeout_status(cuda):
    out = _run([sys.executable, HERE, "timeout", str(_free_port())])
    assert "timeout ok" in out


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fused_reduce_two_ranks():
    out = _run(["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={_free_port()}", HERE, "multi"],
               timeout=300)
    assert "multi-rank ok" in out
    print([line for line in out.splitlines() if line.startswith("paths:")])


# ---------------------------------------------------------------------------- children
def _init(rank, world, port=None):
    import datetime
    import torch.distributed as dist
    if port is not None:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    return dist


def _close(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item()
    assert err <= tol * scale, (err, scale)


def child_one(port):
    dist = _init(0, 1, port)
    from kimi_k3_b200.parallel.symmetric import SymmetricWorkspace, fused_matmul_reduce
    ws = SymmetricWorkspace(None, "cuda:0", 1 << 22)
    torch.manual_seed(0)
    for m, n, k in ((256, 640, 320), (300, 136, 64), (1024, 1024, 512)):
        x = torch.randn(m, k, device="cuda").bfloat16()
        w = (torch.randn(n, k, device="cuda") / k ** 0.5).bfloat16()
        ref = x.float() @ w.float().t()
        for _ in range(3):  # the flag semaphores must balance from call to call
            y = fused_matmul_reduce(x, w, ws)
            _close(y, ref, 1e-2)
        if m % 128 == 0:
            _close(fused_matmul_reduce(x, w, ws, reduce="reduce_scatter"), ref, 1e-2)
    ws.check()
    # all-gather fused into the GEMM's A operand (one rank: the gather is the local shard)
    from kimi_k3_b200.parallel.symmetric import AllGatherWorkspace, fused_allgather_matmul
    ag = AllGatherWorkspace(None, "cuda:0", rows=256, cols=320)
    for it in range(3):
        x = torch.randn(256, 320, device="cuda").bfloat16()
        w = (torch.randn(640, 320, device="cuda") / 320 ** 0.5).bfloat16()
        _close(fused_allgather_matmul(x, w, ag), x.float() @ w.float().t(), 1e-2)
    ag.check()
    dist.destroy_process_group()
    print("one-rank ok")


def child_timeout(port):
    dist = _init(0, 1, port)
    from kimi_k3_b200.ops import _loader
    from kimi_k3_b200.parallel.symmetric import _TILES_CAP, SymmetricWorkspace, fused_matmul_reduce
    C = _loader.require()
    ws = SymmetricWorkspace(None, "cuda:0", 1 << 22)
    m, n, k = 256, 256, 64
    x = torch.randn(m, k, device="cuda").bfloat16()
    w = torch.randn(n, k, device="cuda").bfloat16()
    part = ws.partial(m, n)
    # a second "rank" whose partial and flags live in this rank's buffer and that never runs:
    # the tiles it owns are never reduced and the tiles this rank owns never get its partial
    fake_part = ws.peer_ptrs[0] + (ws.partial_bytes // 2)
    fake_flags = torch.zeros(2 * _TILES_CAP, dtype=torch.int32, device="cuda")
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    import time
    t0 = time.perf_counter()
    C.tc_gemm_comm(x, w, False, 256, 1, 0, 2, part, [ws.peer_ptrs[0], fake_part], 0,
                   [ws.flag_ptrs[0], fake_flags.data_ptr()], _TILES_CAP, out, ws.status, int(0.2e9))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(ws.status.item()) == 5, int(ws.status.item())  # the comm timeout code
    # one time limit (0.2 s) for the whole kernel, not one per tile: every later wait sees the
    # recorded failure and gives up at once
    assert elapsed < 2.0, elapsed
    try:
        ws.check()
        raise AssertionError("check() did not raise")
    except RuntimeError:
        pass
    ws.reset()
    y = fused_matmul_reduce(x, w, ws)  # the context and the workspace are usable again
    _close(y, x.float() @ w.float().t(), 1e-2)
    ws.check()
    dist.destroy_process_group()
    print("timeout ok")


def child_multi():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    dist = _init(rank, world)
    from kimi_k3_b200.parallel.symmetric import SymmetricWorkspace, fused_matmul_reduce
    paths = []
    for use_mc in (True, False):
        ws = SymmetricWorkspace(None, f"cuda:{rank}", 1 << 24, use_multicast=use_mc)
        if use_mc and not ws.has_multicast:
            if rank == 0:
                print("no multicast object on this group: peer path only")
            continue
        for m, n, k in ((512, 640, 320), (1024, 1536, 768), (384, 200, 128)):
            torch.manual_seed(100 + rank)
            x = torch.randn(m, k, device="cuda").bfloat16()
            w = (torch.randn(n, k, device="cuda") / k ** 0.5).bfloat16()
            ref = (x.float() @ w.float().t()).contiguous()
            dist.all_reduce(ref)
            for _ in range(3):
                _close(fused_matmul_reduce(x, w, ws), ref, 2e-2)
            if (m // world) % 128 == 0:
                rs = fused_matmul_reduce(x, w, ws, reduce="reduce_scatter")
                _close(rs, ref[rank * (m // world):(rank + 1) * (m // world)], 2e-2)
        ws.check()
        paths.append("nvls-multimem" if use_mc else "peer")
        del ws
    # all-gather fused into the GEMM: A tiles of rank r's rows come from rank r's shard over NVLink
    from kimi_k3_b200.parallel.symmetric import AllGatherWorkspace, fused_allgather_matmul
    ag = AllGatherWorkspace(None, f"cuda:{rank}", rows=384, cols=320)
    for it in range(3):
        torch.manual_seed(200 + 10 * it + rank)
        x = torch.randn(384, 320, device="cuda").bfloat16()
        torch.manual_seed(7 + it)
        w = (torch.randn(768, 320, device="cuda") / 320 ** 0.5).bfloat16()
        parts = [torch.empty_like(x) for _ in range(world)]
        dist.all_gather(parts, x)
        ref = torch.cat(parts).float() @ w.float().t()
        _close(fused_allgather_matmul(x, w, ag), ref, 1e-2)
    ag.check()
    paths.append("allgather-gemm")
    del ag
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("paths: " + "+".join(paths))
        print("multi-rank ok")


if __name__ == "__main__":
    which = sys.argv[1]
    if which == "one":
        child_one(int(sys.argv[2]))
    elif which == "timeout":
        child_timeout(int(sys.argv[2]))
    else:
        child_multi()
