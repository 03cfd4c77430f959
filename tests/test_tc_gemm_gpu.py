"""tcgen05 GEMM (dense, grouped-M, grouped-K; K-/MN-major operands; fused epilogues) vs fp32 torch."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from kimi_k3_b200.ops import _loader
    return _loader.require()


def _close(a, b, tol=2e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    scale = max(b.abs().max().item(), 1e-6)
    assert err <= tol * scale, f"max err {err:.4e} vs scale {scale:.4e}"


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", [(256, 384, 512), (200, 136, 72), (1024, 640, 640)])
@pytest.mark.parametrize("bn", [128, 256])
def test_dense(cuda, a_mn, b_mn, shape, bn):
    m, n, k = shape
    torch.manual_seed(m + n + k)
    a = torch.randn(m, k, device=cuda).to(torch.bfloat16)
    b = torch.randn(n, k, device=cuda).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    a_in = a.t().contiguous() if a_mn else a
    b_in = b.t().contiguous() if b_mn else b
    out = _C().tc_gemm_dense(a_in, b_in, a_mn, b_mn, False, bn, None)
    _close(out, ref)
    out32 = _C().tc_gemm_dense(a_in, b_in, a_mn, b_mn, True, bn, None)
    _close(out32, ref, 1e-3)


def _segments(counts, align):
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + align - 1) // align * align)
    return offs


@pytest.mark.parametrize("b_mn", [False, True])
def test_grouped_m_store(cuda, b_mn):
    torch.manual_seed(1)
    counts = [100, 0, 300, 5]
    offs = _segments(counts, 128)
    r, k, n, g = offs[-1], 320, 640, len(counts)
    a = torch.zeros(r, k, device=cuda, dtype=torch.bfloat16)
    for i, c in enumerate(counts):
        a[offs[i]:offs[i] + c] = torch.randn(c, k, device=cuda).to(torch.bfloat16)
    w = (0.1 * torch.randn(g, n, k, device=cuda)).to(torch.bfloat16)
    b_in = w.transpose(1, 2).contiguous() if b_mn else w
    off_t = torch.tensor(offs, device=cuda, dtype=torch.int32)
    out, = _C().tc_gemm_grouped(1, a, b_in, None, False, b_mn, off_t, r, n, k, 0, None, False, 4.0, 25.0, None, None,
                                0, 128)
    for i, c in enumerate(counts):
        if c:
            _close(out[offs[i]:offs[i] + c], a[offs[i]:offs[i] + c].float() @ w[i].float().t())


def test_grouped_m_situ_and_scatter(cuda):
    torch.manual_seed(2)
    counts = [130, 64, 0, 257]
    offs = _segments(counts, 128)
    r, l, h, g = offs[-1], 320, 640, len(counts)
    xs = torch.zeros(r, l, device=cuda, dtype=torch.bfloat16)
    for i, c in enumerate(counts):
        xs[offs[i]:offs[i] + c] = torch.randn(c, l, device=cuda).to(torch.bfloat16)
    wg = (0.1 * torch.randn(g, h, l, device=cuda)).to(torch.bfloat16)
    wu = (0.1 * torch.randn(g, h, l, device=cuda)).to(torch.bfloat16)
    off_t = torch.tensor(offs, device=cuda, dtype=torch.int32)
    hh, gg, uu = _C().tc_gemm_grouped(1, xs, wg, wu, False, False, off_t, r, h, l, 1, None, False, 4.0, 25.0, None,
                                      None, 0, 256)
    for i, c in enumerate(counts):
        if not c:
            continue
        x = xs[offs[i]:offs[i] + c].float()
        g_ref, u_ref = x @ wg[i].float().t(), x @ wu[i].float().t()
        _close(gg[offs[i]:offs[i] + c], g_ref)
        _close(uu[offs[i]:offs[i] + c], u_ref)
        h_ref = 4 * torch.tanh(g_ref / 4) * torch.sigmoid(g_ref) * 25 * torch.tanh(u_ref / 25)
        _close(hh[offs[i]:offs[i] + c], h_ref, 3e-2)
    # down projection with weighted scatter-add into 500 token rows
    wd = (0.1 * torch.randn(g, l, h, device=cuda)).to(torch.bfloat16)
    tok = torch.full((r,), -1, device=cuda, dtype=torch.int32)
    wts = torch.rand(r, device=cuda)
    for i, c in enumerate(counts):
        tok[offs[i]:offs[i] + c] = torch.randint(0, 500, (c,), device=cuda, dtype=torch.int32)
    agg = torch.zeros(500, l, device=cuda)
    _C().tc_gemm_grouped(1, hh, wd, None, False, False, off_t, r, l, h, 2, agg, True, 4.0, 25.0, tok, wts, 0, 128)
    ref = torch.zeros(500, l, device=cuda)
    for i, c in enumerate(counts):
        if c:
            y = hh[offs[i]:offs[i] + c].float() @ wd[i].float().t()
            ref.index_add_(0, tok[offs[i]:offs[i] + c].long(), y * wts[offs[i]:offs[i] + c, None])
    _close(agg, ref)


def test_grouped_m_concat_k(cuda):
    """dx = [dG | dU] @ [Wg; Wu] with MN-major weights and a split K."""
    torch.manual_seed(3)
    counts = [128, 200]
    offs = _segments(counts, 128)
    r, l, h, g = offs[-1], 320, 640, 2
    dgu = torch.randn(r, 2 * h, device=cuda).to(torch.bfloat16)
    wg = (0.1 * torch.randn(g, h, l, device=cuda)).to(torch.bfloat16)
    wu = (0.1 * torch.randn(g, h, l, device=cuda)).to(torch.bfloat16)
    off_t = torch.tensor(offs, device=cuda, dtype=torch.int32)
    out, = _C().tc_gemm_grouped(1, dgu, wg, wu, False, True, off_t, r, l, 2 * h, 0, None, False, 4.0, 25.0, None,
                                None, h, 128)
    for i, c in enumerate(counts):
        x = dgu[offs[i]:offs[i] + c].float()
        ref = x[:, :h] @ wg[i].float() + x[:, h:] @ wu[i].float()
        _close(out[offs[i]:offs[i] + c], ref)


def test_grouped_k_weight_grad(cuda):
    """dW[g] = A_seg^T B_seg over 64-aligned row segments (one empty)."""
    torch.manual_seed(4)
    counts = [64, 0, 200, 30]
    offs = _segments(counts, 64)
    r, m, n = offs[-1], 640, 320
    a = torch.zeros(r, m, device=cuda, dtype=torch.bfloat16)
    b = torch.zeros(r, n, device=cuda, dtype=torch.bfloat16)
    for i, c in enumerate(counts):
        a[offs[i]:offs[i] + c] = torch.randn(c, m, device=cuda).to(torch.bfloat16)
        b[offs[i]:offs[i] + c] = torch.randn(c, n, device=cuda).to(torch.bfloat16)
    off_t = torch.tensor(offs, device=cuda, dtype=torch.int32)
    out, = _C().tc_gemm_grouped(2, a, b, None, True, True, off_t, m, n, r, 0, None, True, 4.0, 25.0, None, None, 0,
                                128)
    for i, c in enumerate(counts):
        ref = a[offs[i]:offs[i] + c].float().t() @ b[offs[i]:offs[i] + c].float()
        if c == 0:
            assert out[i].abs().max().item() == 0.0
        else:
            _close(out[i], ref, 1e-3)


def test_moe_grouped_experts_vs_torch(cuda):
    """Routed-expert forward and backward through the grouped GEMMs vs the per-expert PyTorch loop."""
    from kimi_k3_b200.models.moe import GroupedRoutedExperts, vectorized_sparse_dispatch
    from kimi_k3_b200.ops.functional import moe_grouped_experts
    torch.manual_seed(5)
    m, l, h, e, k = 700, 320, 640, 12, 2
    experts = GroupedRoutedExperts(e, l, h, 4.0, 25.0, 0.02).to(cuda)
    latent = torch.randn(m, l, device=cuda).to(torch.bfloat16).requires_grad_()
    logits = torch.randn(m, e, device=cuda)
    sel = torch.topk(logits, k, -1).indices
    w = torch.softmax(torch.randn(m, k, device=cuda), -1).requires_grad_()
    out1 = moe_grouped_experts(latent, sel, w, experts.gate_proj, experts.up_proj, experts.down_proj, 4.0, 25.0)
    go = torch.randn_like(out1)
    out1.backward(go)
    g1 = [latent.grad.clone(), w.grad.clone(), experts.gate_proj.grad.clone(), experts.up_proj.grad.clone(),
          experts.down_proj.grad.clone()]
    for t in (latent, w, experts.gate_proj, experts.up_proj, experts.down_proj):
        t.grad = None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out2 = vectorized_sparse_dispatch(latent, experts, sel, w, accumulation_dtype=torch.float32)
    out2.backward(go)
    g2 = [latent.grad, w.grad, experts.gate_proj.grad, experts.up_proj.grad, experts.down_proj.grad]
    _close(out1, out2, 3e-2)
    for a, b in zip(g1, g2):
        _close(a, b, 5e-2)


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True)])
def test_dense_strided_ragged(cuda, a_mn, b_mn):
    """Row-strided views with ragged M, N, K (the LM-head shapes: vocab 50257 padded to a 64 stride)."""
    torch.manual_seed(11)
    m, n, k = 300, 1001, 333
    def view(rows, cols):
        base = torch.randn(rows, (cols + 63) // 64 * 64, device=cuda).to(torch.bfloat16)
        return base[:, :cols]
    a = view(k, m) if a_mn else view(m, k)
    b = view(k, n) if b_mn else view(n, k)
    ref = (a.float().t() if a_mn else a.float()) @ (b.float() if b_mn else b.float().t())
    out = torch.full((m, (n + 63) // 64 * 64), 7.0, device=cuda)
    _C().tc_gemm_dense(a, b, a_mn, b_mn, True, 128, out[:, :n])
    _close(out[:, :n], ref, 1e-3)
    assert (out[:, n:] == 7.0).all()  # nothing written past the logical edge
    out16 = _C().tc_gemm_dense(a, b, a_mn, b_mn, False, 256, None)
    _close(out16, ref)


def test_pipeline_wait_gives_up_and_context_survives(cuda):
    """A pipeline wait shortened to a single poll gives up inside the kernel: the launch reports the
    failure through the status word, the kernel drains its copies and MMAs and exits, and the next
    GEMM on the same context is correct."""
    import time
    C = _C()
    torch.manual_seed(3)
    a = torch.randn(512, 1024, device=cuda).to(torch.bfloat16)
    b = torch.randn(384, 1024, device=cuda).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    C.tc_gemm_dense(a, b, False, False, False, 256, None, status=status, spin_limit=1)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(status.item()) in (1, 2, 3, 4), int(status.item())
    status.zero_()
    out = C.tc_gemm_dense(a, b, False, False, False, 256, None, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    _close(out, ref)
    # the default (per-device) status word saw nothing
    assert C.tc_gemm_status(False) == 0


@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("shape", [(512, 384, 512), (200, 136, 72), (1000, 640, 640), (384, 1920, 128)])
@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("pair", [0, 1])
def test_dense_cta_pair(cuda, a_mn, b_mn, shape, bn, pair):
    """256-row tiles on CTA pairs (tcgen05.mma.cta_group::2) against the single-CTA kernel and fp32."""
    m, n, k = shape
    torch.manual_seed(m + 3 * n + k)
    a = torch.randn(m, k, device=cuda).to(torch.bfloat16)
    b = torch.randn(n, k, device=cuda).to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    a_in = a.t().contiguous() if a_mn else a
    b_in = b.t().contiguous() if b_mn else b
    out = _C().tc_gemm_dense(a_in, b_in, a_mn, b_mn, True, bn, None, pair=pair)
    _close(out, ref, 1e-3)
    out16 = _C().tc_gemm_dense(a_in, b_in, a_mn, b_mn, False, bn, None, pair=pair)
    _close(out16, ref)


@pytest.mark.parametrize("pair", [0, 1])
def test_dense_bias_residual_epilogue(cuda, pair):
    torch.manual_seed(7)
    m, n, k = 700, 640, 320
    a = torch.randn(m, k, device=cuda).to(torch.bfloat16)
    b = torch.randn(n, k, device=cuda).to(torch.bfloat16)
    bias = torch.randn(n, device=cuda)
    res = torch.randn(m, n, device=cuda).to(torch.bfloat16)
    out = _C().tc_gemm_dense(a, b, False, False, False, 128, None, bias=bias, residual=res, pair=pair)
    _close(out, a.float() @ b.float().t() + bias + res.float())


@pytest.mark.parametrize("ksplit", [1, 3, 8])
@pytest.mark.parametrize("pair", [0, 1])
def test_dense_accumulate_split_k(cuda, ksplit, pair):
    """Weight-gradient form dW += dY^T X (both operands MN-major) with the K range split over work units
    whose fp32 partial tiles are added into the existing gradient."""
    torch.manual_seed(11)
    t, n_out, k_in = 4096, 640, 320
    dy = torch.randn(t, n_out, device=cuda).to(torch.bfloat16)
    x = torch.randn(t, k_in, device=cuda).to(torch.bfloat16)
    g0 = torch.randn(n_out, k_in, device=cuda)
    out = g0.clone()
    _C().tc_gemm_dense(dy, x, True, True, True, 128, out, accumulate=True, ksplit=ksplit, pair=pair)
    _close(out, g0 + dy.float().t() @ x.float(), 1e-3)
