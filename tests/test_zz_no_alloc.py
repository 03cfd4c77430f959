"""The allocation-free C entry point ``kimi_kda_chunk_fwd_noalloc`` against the ordinary KDA forward.

Collected last on purpose: it must pass both alone in a fresh process and after every
other test has run (with the caching allocator warm and other kernels configured).
"""
import ctypes

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _lib():
    from kimi_k3_b200.ops import _loader
    ext = _loader.require()
    lib = ctypes.CDLL(ext.__file__)
    fn = lib.kimi_kda_chunk_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 8 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    msg = lib.kimi_kda_noalloc_status_string
    msg.restype = ctypes.c_char_p
    msg.argtypes = [ctypes.c_int]
    last = lib.kimi_kda_noalloc_last_status
    last.restype = ctypes.c_int
    last.argtypes = []
    return ext, fn, msg, last


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _inputs(b, t, h, dtype, seed):
    torch.manual_seed(seed)
    dev = "cuda"
    q = F.normalize(torch.randn(b, t, h, 64, device=dev), dim=-1).to(dtype)
    k = F.normalize(torch.randn(b, t, h, 64, device=dev), dim=-1).to(dtype)
    v = torch.randn(b, t, h, 64, device=dev).to(dtype)
    g = -5.0 * torch.sigmoid(torch.randn(b, t, h, 64, device=dev) - 2.0)
    beta = torch.sigmoid(torch.randn(b, t, h, device=dev))
    h0 = 0.1 * torch.randn(b, h, 64, 64, device=dev)
    return q, k, v, g, beta, h0


@pytest.mark.parametrize("dtype,code", [(torch.float32, 0), (torch.bfloat16, 1), (torch.float16, 2)])
def test_noalloc_matches_kda_forward_twice(cuda, dtype, code):
    ext, fn, msg, last = _lib()
    stream = torch.cuda.current_stream()
    for call, (b, t, h) in enumerate([(2, 256, 4), (1, 512, 3)]):
        q, k, v, g, beta, h0 = _inputs(b, t, h, dtype, seed=10 + call)
        ref = ext.kda_fwd(q, k, v, g, beta, h0, True)
        o = torch.empty_like(v)
        ht = torch.empty(b, h, 64, 64, device="cuda")
        st = fn(code, _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0), _ptr(o), _ptr(ht), b, t, h,
                ctypes.c_void_p(stream.cuda_stream))
        assert st == 0, msg(st).decode()
        torch.cuda.synchronize()
        tol = 1e-5 if dtype == torch.float32 else 1e-2
        assert (o.float() - ref[0].float()).abs().max().item() <= tol * max(ref[0].float().abs().max().item(), 1.0)
        assert (ht - ref[1]).abs().max().item() <= 1e-5 * max(ref[1].abs().max().item(), 1.0)
        # every bounded wait inside the kernels completed
        assert last() == 0, msg(last()).decode()


def test_noalloc_calls_allocate_nothing(cuda):
    """After the first call on a device (module load and set-up), further calls leave the device's
    free memory and PyTorch's allocator untouched."""
    _, fn, msg, last = _lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    b, t, h = 2, 256, 4
    q, k, v, g, beta, h0 = _inputs(b, t, h, torch.bfloat16, seed=3)
    o = torch.empty_like(v)
    ht = torch.empty(b, h, 64, 64, device="cuda")
    args = (1, _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0), _ptr(o), _ptr(ht), b, t, h, stream)
    assert fn(*args) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    allocs0 = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
    for _ in range(2):
        st = fn(*args)
        assert st == 0, msg(st).decode()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    assert torch.cuda.memory_stats().get("allocation.all.allocated", 0) == allocs0
    assert last() == 0

def test_noalloc_rejects_oversized_problem(cuda):
    _, fn, msg, _ = _lib()
    q = torch.zeros(1, 64 * 129, 1, 64, device="cuda")
    beta = torch.zeros(1, 64 * 129, 1, device="cuda")
    st = fn(0, _ptr(q), _ptr(q), _ptr(q), _ptr(q), _ptr(beta), None, _ptr(q), None, 1, 64 * 129, 1,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 10001
    assert "exceeds the fixed scratch array" in msg(st).decode()
    st = fn(0, _ptr(q), _ptr(q), _ptr(q), _ptr(q), _ptr(beta), None, _ptr(q), None, 1, 100, 1,
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 10002
