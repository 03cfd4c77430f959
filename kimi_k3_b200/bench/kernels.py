"""Device microbenchmarks of the hand-written sm_100a kernels, with roofline fractions.

Each case times one op (forward, or forward + backward) with CUDA events after
warm-up, flushing L2 between repeats, and prints one JSON line with the median
and the achieved FLOP/s or bytes/s as fractions of the measured peaks. The same
entry points are the small, self-terminating workloads used for Nsight Compute
captures of one kernel, e.g.::

    python -m kimi_k3_b200.bench kernels kda --batch 2 --tokens 1024 --heads 10 --repeats 3

Cases: ``gemm`` (tcgen05 dense GEMM vs cuBLAS), ``kda`` (chunked KDA forward /
backward), ``moe`` (grouped routed experts), ``linear_ce`` (LM head + CE),
``attention`` (causal flash attention), ``attnres`` (depth softmax mix).
"""
from __future__ import annotations

import argparse
import json
import math

import torch
import torch.nn.functional as F

from .timing import roofline, time_fn


def _emit(row: dict) -> dict:
    print(json.dumps(row), flush=True)
    return row


def _require_cuda():
    if not torch.cuda.is_available():
        raise SystemExit("kernel benchmarks need a CUDA device")
    from ..ops import _loader
    return _loader.require(), torch.device("cuda")


def kda_flops_per_chunk_head(c: int = 64, dk: int = 64, dv: int = 64) -> float:
    """Chunked KDA forward FLOPs for one 64-token chunk of one head: the two intra-chunk
    score products, the unit-triangular solve, the two UT products, the state read
    (``w S``, ``q S``), the intra output and the state update."""
    return 2.0 * (2 * c * c * dk + c ** 3 / 3 + c * c * dk + c * c * dv + 2 * c * dk * dv + c * c * dv + c * dk * dv)


def bench_gemm(args) -> list:
    C, dev = _require_cuda()
    torch.manual_seed(0)
    m, n, k = args.m, args.n, args.k
    a = torch.randn(m, k, device=dev).bfloat16()
    b = torch.randn(n, k, device=dev).bfloat16()
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    rows = []
    flops = 2.0 * m * n * k
    for bn in (128, 256):
        t = time_fn(lambda: C.tc_gemm_dense(a, b, False, False, False, bn, out), device=dev,
                    warmup=args.warmup, repeats=args.repeats)
        rows.append(_emit({"case": "gemm", "impl": f"tcgen05_bn{bn}", "m": m, "n": n, "k": k, **t.as_dict(),
                           **roofline(t.median_ms, flops=flops)}))
    ref = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    t = time_fn(lambda: torch.mm(a, b.t(), out=ref), device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "gemm", "impl": "cublas", "m": m, "n": n, "k": k, **t.as_dict(),
                       **roofline(t.median_ms, flops=flops)}))
    err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
    rows.append(_emit({"case": "gemm", "check": "rel_err_vs_cublas", "value": err}))
    return rows


def bench_gemm_variants(args) -> list:
    """Dense GEMM ``[m,k] x [n,k]^T``: every tile variant of the tcgen05 kernel (one CTA with 128 or 256
    output columns, CTA pairs with 256-row tiles) against cuBLAS (``torch.mm``)."""
    C, dev = _require_cuda()
    torch.manual_seed(0)
    m, n, k = args.m, args.n, args.k
    a = torch.randn(m, k, device=dev).bfloat16()
    b = torch.randn(n, k, device=dev).bfloat16()
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    flops = 2.0 * m * n * k
    rows = []
    for pair in (0, 1):
        for bn in (128, 256):
            t = time_fn(lambda: C.tc_gemm_dense(a, b, False, False, False, bn, out, pair=pair), device=dev,
                        warmup=args.warmup, repeats=args.repeats)
            rows.append(_emit({"case": "gemm", "impl": f"tcgen05_bn{bn}_{'pair' if pair else 'single'}", "m": m,
                               "n": n, "k": k, **t.as_dict(), **roofline(t.median_ms, flops=flops)}))
    ref = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    t = time_fn(lambda: torch.mm(a, b.t(), out=ref), device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "gemm", "impl": "cublas", "m": m, "n": n, "k": k, **t.as_dict(),
                       **roofline(t.median_ms, flops=flops)}))
    C.tc_gemm_dense(a, b, False, False, False, 256, out, pair=1)
    err = ((out.float() - ref.float()).norm() / ref.float().norm()).item()
    rows.append(_emit({"case": "gemm", "check": "rel_err_vs_cublas", "value": err}))
    return rows


# (name, output features, input features) of the flagship model's dense projections
PROJECTION_SHAPES = [
    ("attn_640x640", 640, 640), ("qkv_fused", 1920, 640), ("shared_gate_up", 1920, 640),
    ("shared_down", 640, 960), ("moe_down", 320, 640), ("moe_up", 640, 320), ("mtp_fusion", 640, 1280),
]


def bench_projections(args) -> list:
    """Forward ``y = x W^T``, input gradient ``dX = dY W`` and weight gradient ``dW = dY^T X`` of every
    projection shape of the flagship model at ``--tokens`` rows: the tcgen05 kernel (best tile variant,
    split-K fp32 weight gradient) against cuBLAS (``torch.mm`` on bf16, bf16 output)."""
    C, dev = _require_cuda()
    torch.manual_seed(0)
    t = args.tokens
    rows = []
    for name, n_out, k_in in PROJECTION_SHAPES:
        x = torch.randn(t, k_in, device=dev).bfloat16()
        w = (torch.randn(n_out, k_in, device=dev) / k_in ** 0.5).bfloat16()
        dy = torch.randn(t, n_out, device=dev).bfloat16()
        y = torch.empty(t, n_out, device=dev, dtype=torch.bfloat16)
        dx = torch.empty(t, k_in, device=dev, dtype=torch.bfloat16)
        dw = torch.zeros(n_out, k_in, device=dev)
        flops = 2.0 * t * n_out * k_in
        ksplit = max(1, min(16, (2 * 148) // max(1, ((n_out + 255) // 256) * ((k_in + 127) // 128))))
        cases = {
            "fwd": [(f"ours_bn{bn}_p{p}", (lambda bn=bn, p=p: C.tc_gemm_dense(x, w, False, False, False, bn, y, pair=p)))
                    for bn in (128, 256) for p in (0, 1)],
            "dgrad": [(f"ours_bn{bn}_p{p}", (lambda bn=bn, p=p: C.tc_gemm_dense(dy, w, False, True, False, bn, dx,
                                                                                pair=p)))
                      for bn in (128, 256) for p in (0, 1)],
            "wgrad": [(f"ours_bn{bn}_p{p}_k{ks}", (lambda bn=bn, p=p, ks=ks: C.tc_gemm_dense(
                dy, x, True, True, True, bn, dw, accumulate=True, ksplit=ks, pair=p)))
                      for bn in (128, 256) for p in (0, 1) for ks in sorted({1, ksplit})],
        }
        ref = {"fwd": lambda: torch.mm(x, w.t(), out=y), "dgrad": lambda: torch.mm(dy, w, out=dx),
               "wgrad": lambda: torch.mm(dy.t(), x)}
        for kind, variants in cases.items():
            best = None
            for label, fn in variants:
                tm = time_fn(fn, device=dev, warmup=args.warmup, repeats=args.repeats)
                if best is None or tm.median_ms < best[1].median_ms:
                    best = (label, tm)
            tr = time_fn(ref[kind], device=dev, warmup=args.warmup, repeats=args.repeats)
            rows.append(_emit({"case": "projection", "shape": name, "pass": kind, "tokens": t, "n_out": n_out,
                               "k_in": k_in, "ours": best[0], "ours_ms": round(best[1].median_ms, 4),
                               "cublas_ms": round(tr.median_ms, 4),
                               "speedup": round(tr.median_ms / best[1].median_ms, 3),
                               **roofline(best[1].median_ms, flops=flops)}))
    return rows


def bench_kda(args) -> list:
    from ..ops import kda_chunk
    _, dev = _require_cuda()
    torch.manual_seed(0)
    b, t, h = args.batch, args.tokens, args.heads
    q = F.normalize(torch.randn(b, t, h, 64, device=dev), dim=-1).bfloat16().requires_grad_()
    k = F.normalize(torch.randn(b, t, h, 64, device=dev), dim=-1).bfloat16().requires_grad_()
    v = torch.randn(b, t, h, 64, device=dev).bfloat16().requires_grad_()
    g = (-5 * torch.sigmoid(torch.randn(b, t, h, 64, device=dev) - 2)).requires_grad_()
    beta = torch.sigmoid(torch.randn(b, t, h, device=dev)).requires_grad_()
    do = torch.randn(b, t, h, 64, device=dev).bfloat16()
    chunks = b * h * math.ceil(t / 64)
    fwd_flops = chunks * kda_flops_per_chunk_head()
    io_bytes = b * t * h * (64 * 2 * 4 + 64 * 4 + 4)  # q k v o bf16, g fp32, beta fp32

    def fwd():
        with torch.no_grad():
            kda_chunk(q, k, v, g, beta, None, False)

    def fwd_bwd():
        o, _ = kda_chunk(q, k, v, g, beta, None, False)
        o.backward(do)

    rows = []
    tf = time_fn(fwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "kda", "pass": "forward", "batch": b, "tokens": t, "heads": h, **tf.as_dict(),
                       **roofline(tf.median_ms, flops=fwd_flops, bytes_moved=io_bytes)}))
    tb = time_fn(fwd_bwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    # backward ~ 2x the forward products plus the recomputed forward
    rows.append(_emit({"case": "kda", "pass": "forward+backward", "batch": b, "tokens": t, "heads": h,
                       **tb.as_dict(), **roofline(tb.median_ms, flops=3 * fwd_flops, bytes_moved=3 * io_bytes)}))
    return rows


def bench_moe(args) -> list:
    from ..ops import moe_grouped_experts
    _, dev = _require_cuda()
    torch.manual_seed(0)
    m, lat, hid, e, topk = args.tokens, args.latent, args.hidden, args.experts, args.topk
    x = torch.randn(m, lat, device=dev).bfloat16().requires_grad_()
    wg = (torch.randn(e, hid, lat, device=dev) / lat ** 0.5).bfloat16().requires_grad_()
    wu = (torch.randn(e, hid, lat, device=dev) / lat ** 0.5).bfloat16().requires_grad_()
    wd = (torch.randn(e, lat, hid, device=dev) / hid ** 0.5).bfloat16().requires_grad_()
    scores = torch.randn(m, e, device=dev)
    w, sel = scores.sigmoid().topk(topk, dim=-1)
    w = (w / w.sum(-1, keepdim=True)).requires_grad_()
    flops = 2.0 * m * topk * (2 * hid * lat + hid * lat)

    def fwd():
        with torch.no_grad():
            moe_grouped_experts(x, sel, w, wg, wu, wd, 4.0, 25.0)

    def fwd_bwd():
        moe_grouped_experts(x, sel, w, wg, wu, wd, 4.0, 25.0).sum().backward()

    rows = []
    tf = time_fn(fwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "moe", "pass": "forward", "tokens": m, "latent": lat, "hidden": hid, "experts": e,
                       "top_k": topk, **tf.as_dict(), **roofline(tf.median_ms, flops=flops)}))
    tb = time_fn(fwd_bwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "moe", "pass": "forward+backward", "tokens": m, "latent": lat, "hidden": hid,
                       "experts": e, "top_k": topk, **tb.as_dict(), **roofline(tb.median_ms, flops=4 * flops)}))
    return rows


def bench_linear_ce(args) -> list:
    from ..ops import linear_cross_entropy
    _, dev = _require_cuda()
    torch.manual_seed(0)
    n, d, v = args.rows, args.dim, args.vocab
    hdn = torch.randn(n, d, device=dev).bfloat16().requires_grad_()
    wt = (torch.randn(v, d, device=dev) / d ** 0.5).requires_grad_()
    tgt = torch.randint(0, v, (n,), device=dev)
    valid = torch.ones(n, dtype=torch.bool, device=dev)

    def fwd_bwd():
        linear_cross_entropy(hdn, wt, tgt, valid).backward()

    t = time_fn(fwd_bwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    return [_emit({"case": "linear_ce", "pass": "forward+backward", "rows": n, "dim": d, "vocab": v, **t.as_dict(),
                   **roofline(t.median_ms, flops=6.0 * n * d * v)})]


def bench_attention(args) -> list:
    from ..ops import flash_attention
    _, dev = _require_cuda()
    torch.manual_seed(0)
    b, t, h = args.batch, args.tokens, args.heads
    q, k, v = (torch.randn(b, t, h, 64, device=dev).bfloat16().requires_grad_() for _ in range(3))
    flops = 4.0 * b * h * t * t * 64 / 2  # causal

    def fwd():
        with torch.no_grad():
            flash_attention(q, k, v, causal=True)

    def fwd_bwd():
        flash_attention(q, k, v, causal=True).sum().backward()

    rows = []
    tf = time_fn(fwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "attention", "pass": "forward", "batch": b, "tokens": t, "heads": h, **tf.as_dict(),
                       **roofline(tf.median_ms, flops=flops)}))
    tb = time_fn(fwd_bwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "attention", "pass": "forward+backward", "batch": b, "tokens": t, "heads": h,
                       **tb.as_dict(), **roofline(tb.median_ms, flops=3.5 * flops)}))
    return rows


def bench_attnres(args) -> list:
    from ..ops import attnres_mix
    _, dev = _require_cuda()
    torch.manual_seed(0)
    srcs = [torch.randn(args.batch, args.tokens, args.dim, device=dev).bfloat16().requires_grad_()
            for _ in range(args.sources)]
    q = torch.randn(args.dim, device=dev).requires_grad_()
    w = torch.ones(args.dim, device=dev).requires_grad_()
    per = args.batch * args.tokens * args.dim * 2

    def fwd():
        with torch.no_grad():
            attnres_mix(srcs, q, w, 1e-6)

    def fwd_bwd():
        attnres_mix(srcs, q, w, 1e-6).float().sum().backward()

    rows = []
    tf = time_fn(fwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "attnres", "pass": "forward", "sources": args.sources, **tf.as_dict(),
                       **roofline(tf.median_ms, bytes_moved=(args.sources + 1) * per)}))
    tb = time_fn(fwd_bwd, device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "attnres", "pass": "forward+backward", "sources": args.sources, **tb.as_dict(),
                       **roofline(tb.median_ms, bytes_moved=(3 * args.sources + 2) * per)}))
    return rows


def bench_kda_phases(args) -> list:
    """Per-phase cycles of the tcgen05 KDA intra backward (block 0, its first chunk) from the
    kernel's optional clock64 probes."""
    C, dev = _require_cuda()
    from ..ops import kda_chunk
    torch.manual_seed(0)
    b, t, h = args.batch, args.tokens, args.heads
    q = F.normalize(torch.randn(b, t, h, 64, device=dev), dim=-1).bfloat16().requires_grad_()
    k = F.normalize(torch.randn(b, t, h, 64, device=dev), dim=-1).bfloat16().requires_grad_()
    v = torch.randn(b, t, h, 64, device=dev).bfloat16().requires_grad_()
    g = (-5 * torch.sigmoid(torch.randn(b, t, h, 64, device=dev) - 2)).requires_grad_()
    beta = torch.sigmoid(torch.randn(b, t, h, device=dev)).requires_grad_()
    for it in range(3):
        C.kda_phase_profile(it == 2)
        o, _ = kda_chunk(q, k, v, g, beta, None, False)
        o.float().sum().backward()
        torch.cuda.synchronize()
    ph = C.kda_phase_profile(False)
    names = ["loads", "cumsum+operands", "MMA-1/2 wait", "read MMA-1/2", "solve | W,U,Kown", "MMA-3 wait",
             "dL->dA | Kq,Qq", "dA^T|dP^T transpose", "MMA-4/5 wait", "row+column side", "stores+dg"]
    clock_khz = torch.cuda.get_device_properties(dev).clock_rate
    total = ph[11] - ph[0]
    rows = []
    for i, n in enumerate(names):
        cyc = ph[i + 1] - ph[i]
        rows.append(_emit({"case": "kda_phases", "phase": n, "cycles": cyc, "us": round(cyc / clock_khz * 1e3, 2),
                           "share": round(cyc / max(total, 1), 3)}))
    return rows


def bench_decode(args) -> list:
    """One decode step's device kernels at serving shapes: MLA latent flash-decode over a
    ``[batch, tokens, dim]`` cache (``--heads`` query heads), KDA recurrent token, fused sampling."""
    C, dev = _require_cuda()
    torch.manual_seed(0)
    b, t, l, h = args.batch, args.tokens, args.dim, args.heads
    rows = []
    qlat = torch.randn(b, h, l, device=dev)
    latent = torch.randn(b, t, l, device=dev).bfloat16()
    lengths = torch.full((b,), t, dtype=torch.int32, device=dev)
    tm = time_fn(lambda: C.mla_decode(qlat, latent, lengths), device=dev, warmup=args.warmup, repeats=args.repeats)
    rows.append(_emit({"case": "decode", "kernel": "mla_decode", "batch": b, "cache_tokens": t, "latent": l,
                       "heads": h, **tm.as_dict(), **roofline(tm.median_ms, bytes_moved=latent.numel() * 2)}))
    q = torch.randn(b, h, 64, device=dev).bfloat16()
    g = -torch.rand(b, h, 64, device=dev)
    beta = torch.rand(b, h, device=dev)
    st = torch.randn(b, h, 64, 64, device=dev)
    tk = time_fn(lambda: C.kda_decode(q, q, q, g, beta, st, st), device=dev, warmup=args.warmup,
                 repeats=args.repeats)
    rows.append(_emit({"case": "decode", "kernel": "kda_decode", "batch": b, "heads": h, **tk.as_dict(),
                       **roofline(tk.median_ms, bytes_moved=2 * st.numel() * 4)}))
    logits = torch.randn(b, args.vocab, device=dev).bfloat16()
    so = torch.tensor([0, 0], dtype=torch.long, device=dev)
    for name, kw in (("greedy", (1.0, 1.0, 0, 1.0, False)), ("top_k_top_p", (1.0, 0.8, 50, 0.9, True))):
        ts = time_fn(lambda: C.sample_tokens(logits, None, *kw, so), device=dev, warmup=args.warmup,
                     repeats=args.repeats)
        rows.append(_emit({"case": "decode", "kernel": f"sample_{name}", "batch": b, "vocab": args.vocab,
                           **ts.as_dict(), **roofline(ts.median_ms, bytes_moved=logits.numel() * 2)}))
    return rows


def bench_newton_schulz(args) -> list:
    """Five Newton-Schulz iterations per Muon bucket of the t4_wikitext model (vocab 50,257): the
    batched library GEMMs (the training default) against the grouped tcgen05 path."""
    from ..config.profiles import profile_model_config
    from ..models import KimiK3
    from ..train import optimizer as O
    C, dev = _require_cuda()
    del C
    model = KimiK3(profile_model_config("t4_wikitext", vocab_size=50257))
    opt, _ = O.build_kimi_optimizer(model, O.KimiOptimizerConfig(kind="per_head_muon_adamw", per_head_qkv=True))
    rows = []
    for (_, r, c, _, mom, _) in opt.muon._ensure_buckets():
        e = mom.shape[0]
        x = torch.randn(e, r, c, device=dev).to(torch.bfloat16)
        tr = r > c
        w = x.transpose(-2, -1) if tr else x
        for name, tc in (("batched_gemm", False), ("tcgen05_grouped", True)):
            tm = time_fn(lambda: O.newton_schulz_iterations(w, 5, transpose_out=tr, tensor_cores=tc), device=dev,
                         warmup=args.warmup, repeats=args.repeats)
            m, n = min(r, c), max(r, c)
            flops = 5 * e * (2 * m * m * n * 2 + 2 * m * m * m)
            rows.append(_emit({"case": "ns", "path": name, "matrices": e, "rows": r, "cols": c, **tm.as_dict(),
                               **roofline(tm.median_ms, flops=flops)}))
    return rows


CASES = {"kda_phases": bench_kda_phases, "gemm": bench_gemm, "gemm_variants": bench_gemm_variants,
         "projections": bench_projections, "kda": bench_kda, "moe": bench_moe, "linear_ce": bench_linear_ce,
         "attention": bench_attention, "attnres": bench_attnres, "decode": bench_decode,
         "ns": bench_newton_schulz}


def build_parser(parser: argparse.ArgumentParser | None = None) -> argparse.ArgumentParser:
    p = parser or argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("case", choices=sorted(CASES))
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--repeats", type=int, default=10)
    p.add_argument("--m", type=int, default=4096)
    p.add_argument("--n", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--batch", type=int, default=16)
    p.add_argument("--tokens", type=int, default=1024)
    p.add_argument("--heads", type=int, default=10)
    p.add_argument("--dim", type=int, default=640)
    p.add_argument("--sources", type=int, default=4)
    p.add_argument("--latent", type=int, default=320)
    p.add_argument("--hidden", type=int, default=640)
    p.add_argument("--experts", type=int, default=12)
    p.add_argument("--topk", type=int, default=2)
    p.add_argument("--rows", type=int, default=16384)
    p.add_argument("--vocab", type=int, default=50257)
    return p


def main(argv=None) -> list:
    args = build_parser().parse_args(argv)
    if args.case in ("moe", "projections") and args.tokens == 1024:
        args.tokens = 16384  # one micro-batch of the flagship config
    return CASES[args.case](args)


if __name__ == "__main__":
    main()
