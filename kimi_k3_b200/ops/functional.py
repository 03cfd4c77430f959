"""Autograd functions over the sm_100a kernels (CUDA tensors only).

Numerics contract (checked by ``tests/test_kernels_gpu.py`` against fp32 PyTorch):
activations may be bf16/fp16/fp32; all reductions and recurrences run in fp32; outputs
are rounded to the activation dtype once.  Gradients of fp32 parameters are returned in
fp32.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _loader


def _C():
    return _loader.require()


def _act_dtype(x: torch.Tensor) -> torch.dtype:
    if torch.is_autocast_enabled("cuda") and x.dtype == torch.float32:
        return torch.get_autocast_dtype("cuda")
    return x.dtype


# --------------------------------------------------------------------------- projections
def _tma_rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` as a row-major matrix whose rows start on 16-byte boundaries (copy only when needed)."""
    if t.stride(-1) != 1 or (t.stride(0) * t.element_size()) % 16 or t.data_ptr() % 16 or t.stride(0) < t.shape[1]:
        t = t.contiguous()
    return t


def gemm_tiles(n: int) -> int:
    """Output columns per tile for an ``n``-wide product: 256 (with CTA pairs, 256 x 256 tiles) unless
    the width is so narrow that most of a 256-wide tile would be padding."""
    return 256 if n >= 320 or n % 256 == 0 else 128


def wgrad_splits(rows: int, cols: int, k: int, bn: int, sms: int = 148) -> int:
    """K slices of a weight-gradient product ``[rows, cols]`` with reduction length ``k``: about one
    work unit per SM (every extra slice adds a tile of fp32 reduce-adds in L2), at most 8, and every
    slice keeps at least four 64-wide K blocks (measured on B200 at the model's shapes)."""
    tiles = -(-rows // 128) * -(-cols // bn)
    want = max(1, round(sms / tiles))
    return int(max(1, min(want, 8, max(1, (k // 64) // 4))))


_SMALL_M = 128  # rows up to one tile: decode steps and short prompts
_SM_COUNT: dict = {}


def _sm_count(device) -> int:
    n = _SM_COUNT.get(device)
    if n is None:
        n = _SM_COUNT[device] = torch.cuda.get_device_properties(device).multi_processor_count
    return n


def _split_k_product(x2: torch.Tensor, w: torch.Tensor):
    """``x2 @ w^T`` in fp32 for at most one tile of rows, or None when one pass already fills the GPU.

    With a handful of rows a product has only ``ceil(n / 128)`` output tiles, so a plain launch keeps
    a few SMs busy streaming the whole weight.  Here the reduction is split so that about one work
    unit runs per SM (at most 8 slices, each at least four 64-wide K blocks) and the slices add into
    one zeroed fp32 buffer with TMA reduce-adds."""
    m, k = x2.shape
    n = w.shape[0]
    tiles = -(-n // 128)
    splits = int(min(_sm_count(x2.device) // tiles, 8, k // 256))
    if splits < 2 or n % 4:
        return None
    acc = torch.zeros(m, _pad8(n), device=x2.device, dtype=torch.float32)[:, :n]  # row stride: 8 elements
    _C().tc_gemm_dense(x2, w, False, False, True, 128, acc, accumulate=True, ksplit=splits)
    return acc


class _Linear(torch.autograd.Function):
    """``y = x W^T (+ b)`` on the tcgen05 GEMM with bf16 operands and fp32 accumulation.

    Forward reads the weight's persistent bf16 mirror (``ops.mirror``) and adds the bias in the
    epilogue.  Backward: ``dX = dY W`` (the mirror read MN-major, no transpose copy) and
    ``dW = dY^T X`` written in fp32 by split-K work units that add their slices into one zeroed
    buffer, so the fp32 master's gradient needs no cast.  Reference: ``nn.Linear`` under bf16
    autocast (``src/kda/projections.py:164-215``, ``src/mla/latent_kv.py:22-79``,
    ``src/kimi_primitives/output_gate.py:9-74``, ``src/stable_latent_moe/module.py:198-230``).
    """

    @staticmethod
    def forward(ctx, x, weight, bias, wb):
        shape = x.shape
        k, n = shape[-1], wb.shape[0]
        x2 = x.reshape(-1, k)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = _tma_rows(x2)
        acc = _split_k_product(x2, wb) if x2.shape[0] <= _SMALL_M else None
        if acc is not None:
            if bias is not None:
                acc.add_(bias)
            y = acc.to(torch.bfloat16)
        else:
            y = _C().tc_gemm_dense(x2, wb, False, False, False, gemm_tiles(n), None, bias=bias)
        ctx.save_for_backward(x2, wb)
        ctx.meta = (shape, x.dtype, bias is not None)
        return y.view(*shape[:-1], n) if y.is_contiguous() else y.reshape(*shape[:-1], n)

    @staticmethod
    def backward(ctx, dy):
        x2, wb = ctx.saved_tensors
        shape, xdt, has_bias = ctx.meta
        n, k = wb.shape
        dy2 = dy.reshape(-1, n)
        if dy2.dtype != torch.bfloat16:
            dy2 = dy2.to(torch.bfloat16)
        n8 = -(-n // 8) * 8
        if n8 != n:
            # a narrow projection (router, beta): dY is both the K-major A of dX and the MN-major A
            # of dW, so its rows must be 16-byte aligned: pad the width with zero columns (and the
            # weight with zero rows); the zeros add nothing to either product
            dy2 = F.pad(dy2, (0, n8 - n))
            wb = F.pad(wb, (0, 0, 0, n8 - n))
        dy2 = _tma_rows(dy2)
        C = _C()
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = C.tc_gemm_dense(dy2, wb, False, True, xdt == torch.float32, gemm_tiles(k), None)
            dx = dx.reshape(shape)
        if ctx.needs_input_grad[1]:
            bn = gemm_tiles(k)
            dw = torch.zeros(n8, k, device=dy.device, dtype=torch.float32)
            C.tc_gemm_dense(dy2, x2, True, True, True, bn, dw, accumulate=True,
                            ksplit=wgrad_splits(n8, k, dy2.shape[0], bn), pair=0)
            dw = dw[:n]
        if has_bias and ctx.needs_input_grad[2]:
            db = dy2[:, :n].float().sum(0)
        return dx, dw, db, None


def _pad8(n: int) -> int:
    return -(-n // 8) * 8


class _LinearGroup(torch.autograd.Function):
    """Several projections of one input as one GEMM per pass (forward, input gradient, weight
    gradients) over the group's concatenated bf16 weight ``W_cat``.

    Forward writes each projection's output straight into its own tensor (per-column-segment output
    maps); backward reads every output gradient in place as one K-segmented operand, so
    ``dX = sum_i dY_i W_i`` is a single product with no concatenation copy and no gradient adds,
    and all weight gradients come out of one split-K product into one fp32 buffer whose row slices
    are the parameters' gradients."""

    @staticmethod
    def forward(ctx, x, wcat, widths, *weights):
        shape = x.shape
        k = shape[-1]
        x2 = x.reshape(-1, k)
        if x2.dtype != torch.bfloat16:
            x2 = x2.to(torch.bfloat16)
        x2 = _tma_rows(x2)
        m = x2.shape[0]
        acc = _split_k_product(x2, wcat) if m <= _SMALL_M else None
        if acc is not None:  # few rows: one split-K product over W_cat, outputs are column slices
            y = acc.to(torch.bfloat16)
            offs = [0]
            for w in widths:
                offs.append(offs[-1] + w)
            outs = [y[:, a:b] for a, b in zip(offs[:-1], offs[1:])]
        else:
            outs = [torch.empty(m, _pad8(w), device=x.device, dtype=torch.bfloat16)[:, :w] for w in widths]
            _C().tc_gemm_group(1, outs, x2, wcat, None, 256, 1, -1)
        ctx.save_for_backward(x2, wcat)
        ctx.meta = (shape, x.dtype, tuple(widths))
        return tuple(o.view(*shape[:-1], w) for o, w in zip(outs, widths))

    @staticmethod
    def backward(ctx, *grads):
        x2, wcat = ctx.saved_tensors
        shape, xdt, widths = ctx.meta
        m, k = x2.shape
        segs = []
        for g, w in zip(grads, widths):
            if g is None:
                g2 = torch.zeros(m, _pad8(w), device=x2.device, dtype=torch.bfloat16)
            else:
                g2 = g.reshape(m, w)
                if g2.dtype != torch.bfloat16:
                    g2 = g2.to(torch.bfloat16)
                if w % 8:
                    g2 = F.pad(g2, (0, _pad8(w) - w))
                g2 = _tma_rows(g2)
            segs.append(g2)
        C = _C()
        dx = dws = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty(m, k, device=x2.device, dtype=torch.float32 if xdt == torch.float32 else torch.bfloat16)
            C.tc_gemm_group(2, segs, x2, wcat, dx, gemm_tiles(k), 1, -1)
            dx = dx.view(shape)
        if any(ctx.needs_input_grad[3:]):
            n = wcat.shape[0]
            dwcat = torch.zeros(n, k, device=x2.device, dtype=torch.float32)
            bn = gemm_tiles(k)
            C.tc_gemm_group(3, segs, x2, wcat, dwcat, bn, wgrad_splits(n, k, m, bn), 0)
            dws, row = [], 0
            for w in widths:
                dws.append(dwcat[row:row + w])
                row += w
        return (dx, None, None, *(dws if dws is not None else [None] * len(widths)))


def linear_group_supported(x: torch.Tensor, weights) -> bool:
    """Every width but the last a multiple of 64, every weight reading the same ``K``, bf16 compute."""
    if len(weights) < 2 or len(weights) > 8 or _act_dtype(x) != torch.bfloat16:
        return False
    k = x.shape[-1]
    if k % 8 or any(w.ndim != 2 or w.shape[1] != k for w in weights):
        return False
    return all(w.shape[0] % 64 == 0 for w in weights[:-1])


def linear_group(x: torch.Tensor, weights) -> tuple:
    """``tuple(x @ W_i^T for W_i in weights)`` as one tcgen05 GEMM per pass (see :class:`_LinearGroup`)."""
    from .mirror import group_weight
    return _LinearGroup.apply(x, group_weight(weights), [int(w.shape[0]) for w in weights], *weights)


def linear_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """The tcgen05 path applies: bf16 compute (autocast or bf16 input), widths multiples of 8."""
    if _act_dtype(x) != torch.bfloat16 or weight.ndim != 2:
        return False
    return x.shape[-1] % 8 == 0 and weight.shape[1] == x.shape[-1] and x.numel() > 0


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight^T + bias`` with bf16 operands on the tcgen05 GEMM (see :class:`_Linear`)."""
    from .mirror import bf16_weight
    return _Linear.apply(x, weight, bias, bf16_weight(weight))


# --------------------------------------------------------------------------- RMSNorm
class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, period):
        xc = x.contiguous()
        y, rstd = _C().rms_norm_fwd(xc, w, float(eps), int(period))
        ctx.save_for_backward(xc, w, rstd)
        ctx.period = int(period)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, rstd = ctx.saved_tensors
        dx, dw = _C().rms_norm_bwd(dy, x, w, rstd, ctx.period, ctx.needs_input_grad[1])
        return dx, (dw.to(w.dtype) if dw is not None and ctx.needs_input_grad[1] else None), None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, per_row_weight_period: int | None = None):
    """RMSNorm over the last axis; ``weight`` is ``[D]`` or ``[P, D]`` applied to row ``r % P``."""
    dim = x.shape[-1]
    vec = 16 // x.element_size()
    if dim % vec:
        from ..models.primitives import rms_norm_reference
        return rms_norm_reference(x, weight, eps)
    period = per_row_weight_period or 1
    shape = x.shape
    y = _RMSNorm.apply(x.reshape(-1, dim), weight, eps, period)
    return y.reshape(shape)


# --------------------------------------------------------------------------- SiTU / gates
class _SiTU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, g, u, bg, bu):
        g, u = g.contiguous(), u.contiguous()
        ctx.save_for_backward(g, u)
        ctx.b = (float(bg), float(bu))
        return _C().situ_fwd(g, u, *ctx.b)

    @staticmethod
    def backward(ctx, dy):
        g, u = ctx.saved_tensors
        dg, du = _C().situ_bwd(dy, g, u, *ctx.b)
        return dg, du, None, None


def situ_glu(gate, up, beta_gate, beta_up):
    if up.dtype != gate.dtype:
        up = up.to(gate.dtype)
    return _SiTU.apply(gate, up, beta_gate, beta_up)


class _SigMul(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, x):
        z, x = z.contiguous(), x.contiguous()
        ctx.save_for_backward(z, x)
        return _C().sigmul_fwd(z, x)

    @staticmethod
    def backward(ctx, dy):
        z, x = ctx.saved_tensors
        dz, dx = _C().sigmul_bwd(dy, z, x)
        return dz, dx


def sigmoid_mul(logits, x):
    """``sigmoid(logits) * x`` (both in the activation dtype)."""
    if x.dtype != logits.dtype:
        x = x.to(logits.dtype)
    return _SigMul.apply(logits, x)


# --------------------------------------------------------------------------- KDA prep
class _KdaDecay(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, a_log, g_min, ceps):
        z = z.contiguous()
        ctx.save_for_backward(z, a_log)
        ctx.c = (float(g_min), float(ceps))
        return _C().decay_fwd(z, a_log, *ctx.c)

    @staticmethod
    def backward(ctx, dg):
        z, a_log = ctx.saved_tensors
        dz, da = _C().decay_bwd(dg, z, a_log, *ctx.c)
        return dz, da.to(a_log.dtype), None, None


def kda_decay(logits, a_log, g_min):
    """``g_min * clamp(sigmoid(exp(A_log) z), eps, 1-eps)`` in fp32 (eps of the input dtype)."""
    return _KdaDecay.apply(logits, a_log, g_min, torch.finfo(logits.dtype).eps)


class _ConvSiluNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, head_dim, eps, normalize):
        x = x.contiguous()
        ctx.save_for_backward(x, w)
        ctx.c = (int(head_dim), float(eps), bool(normalize))
        return _C().conv_fwd(x, w, *ctx.c)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx, dw = _C().conv_bwd(dy, x, w, *ctx.c)
        return dx, dw.to(w.dtype), None, None, None


def conv_silu_norm(x, conv_weight, head_dim, eps, normalize):
    """Causal depthwise conv (zero history) + SiLU (+ per-head L2 normalisation)."""
    return _ConvSiluNorm.apply(x, conv_weight, head_dim, eps, normalize)


# --------------------------------------------------------------------------- KDA chunk core
class _KdaChunk(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, h0, want_final):
        out = _C().kda_fwd(q, k, v, g, beta, h0, bool(want_final))
        o, ht, saved = out[0], out[1], out[2:]
        ctx.save_for_backward(q, k, v, g, beta, *saved)
        ctx.has_h0 = h0 is not None
        if want_final:
            return o, ht
        return o, None

    @staticmethod
    def backward(ctx, do, dht):
        q, k, v, g, beta, *saved = ctx.saved_tensors
        dq, dk, dv, dg, dbeta, dh0 = _C().kda_bwd(q, k, v, g, beta, list(saved), do, dht, ctx.has_h0)
        return (dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dg, dbeta, dh0 if ctx.has_h0 else None, None)


def kda_chunk(q, k, v, g, beta, initial_state, output_final_state, chunk_size=64):
    """Chunked KDA on ``[B,T,H,64]``; returns ``(o, final_state or None)``.

    ``g`` and ``beta`` are promoted to fp32; the token axis is zero-padded to a multiple
    of 64 (padded tokens have g = 0 and beta = 0, so they neither decay nor write).
    """
    if chunk_size != 64 or q.shape[-1] != 64 or v.shape[-1] != 64:
        raise NotImplementedError("the sm_100a KDA kernel implements chunk 64 and head dims 64")
    b, t, h, _ = q.shape
    dt = _act_dtype(v)
    q, k, v = (x.to(dt).contiguous() for x in (q, k, v))
    g = g.float().contiguous()
    beta = beta.float().contiguous()
    pad = (-t) % 64
    if pad:
        q, k, v, g = (F.pad(x, (0, 0, 0, 0, 0, pad)) for x in (q, k, v, g))
        beta = F.pad(beta, (0, 0, 0, pad))
    h0 = None if initial_state is None else initial_state.float().contiguous()
    o, ht = _KdaChunk.apply(q, k, v, g, beta, h0, bool(output_final_state))
    if pad:
        o = o[:, :t]
    return o, ht


def kda_decode_step(q, k, v, g, beta, state, out_state=None):
    """One recurrent KDA token for ``[B,1,H,64]`` inputs with fp32 state ``[B,H,64,64]``.

    The kernel reads ``state`` and writes the updated state to ``out_state`` (a new tensor when
    None; ``out_state=state`` advances a serving cache in place).  Returns ``(o [B,1,H,64], state')``."""
    b, _, h, _ = q.shape
    o, ns = _C().kda_decode(q.reshape(b, h, 64), k.reshape(b, h, 64), v.reshape(b, h, 64),
                            g.reshape(b, h, 64), beta.reshape(b, h), state.float().contiguous(), out_state)
    return o.view(b, 1, h, 64), ns


def conv_silu_norm_step(xs, histories, weights, biases, head_dims, eps):
    """Advance up to three short-conv streams by one token (one launch).

    ``xs[i]`` ``[B,1,C_i]`` or ``[B,C_i]``; ``histories[i]`` ``[B,K-1,C_i]`` is shifted IN PLACE
    (oldest row first, the new input appended); ``head_dims[i]`` > 0 applies the per-head L2
    norm after the SiLU.  Returns the outputs shaped like ``xs``."""
    ys = _C().conv_step([x.reshape(x.shape[0], -1) for x in xs], list(histories), list(weights), list(biases),
                        [int(d) for d in head_dims], float(eps))
    return [y.view(x.shape) for x, y in zip(xs, ys)]


# --------------------------------------------------------------------------- attention
class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, key_lengths, scale):
        o, lse = _C().fa_fwd(q, k, v, bool(causal), key_lengths, float(scale))
        ctx.save_for_backward(q, k, v, o, lse, key_lengths if key_lengths is not None else torch.empty(0))
        ctx.c = (bool(causal), float(scale), key_lengths is not None)
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse, kl = ctx.saved_tensors
        causal, scale, has_kl = ctx.c
        dq, dk, dv = _C().fa_bwd(q, k, v, o, do, lse, causal, kl if has_kl else None, scale)
        return dq.to(q.dtype), dk, dv, None, None, None


def flash_attention(q, k, v, causal=True, key_padding_mask=None, scale=None):
    """Attention over ``[B,T,H,64]`` tensors (bf16/fp16 compute); returns ``[B,Tq,H,64]``.

    ``key_padding_mask`` ``[B,Tk]`` (True = valid) must be right-padded; it is turned
    into per-row key lengths.
    """
    dt = _act_dtype(q)
    if dt == torch.float32:
        dt = torch.bfloat16
    q, k, v = (x.to(dt).contiguous() for x in (q, k, v))
    kl = None
    if key_padding_mask is not None:
        kl = key_padding_mask.sum(dim=1).to(torch.int32)
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    return _FlashAttn.apply(q, k, v, causal, kl, scale)


def mla_decode_supported(num_heads: int, latent_dim: int) -> bool:
    return bool(_C().mla_decode_supported(int(num_heads), int(latent_dim)))


def mla_absorbed_decode(query, latent_cache, cache_mask, key_up_weight, value_up_weight, lengths=None):
    """Weight-absorbed one-token MLA attention over the latent cache (fp32 math).

    ``query`` ``[B,1,H,Dq]``, ``latent_cache`` ``[B,T,L]`` whose valid rows form a prefix of
    length ``lengths[b]`` (from ``cache_mask`` when not given) -> ``[B,1,H,Dv]`` fp32.  The
    attention over the cache is the split-T flash-decode kernel; the two small per-head
    projections into and out of the latent space are batched GEMMs."""
    b, _, h, dq = query.shape
    l = latent_cache.shape[-1]
    wuk = key_up_weight.float().reshape(h, dq, l)
    wuv = value_up_weight.float().reshape(h, -1, l)
    q_lat = torch.bmm(query[:, 0].float().transpose(0, 1), wuk).transpose(0, 1) / math.sqrt(dq)  # [B,H,L]
    if latent_cache.dtype in (torch.float32, torch.bfloat16, torch.float16) and mla_decode_supported(h, l):
        if lengths is None:
            lengths = (torch.full((b,), latent_cache.shape[1], dtype=torch.int32, device=query.device)
                       if cache_mask is None else cache_mask.sum(dim=1, dtype=torch.int32))
        ctx = _C().mla_decode(q_lat.contiguous(), latent_cache.contiguous(), lengths)
    else:
        scores = torch.einsum("bhl,btl->bht", q_lat, latent_cache.float())
        if lengths is not None:
            cache_mask = torch.arange(latent_cache.shape[1], device=query.device)[None, :] < lengths[:, None]
        if cache_mask is not None:
            scores = scores.masked_fill(~cache_mask[:, None, :], -torch.inf)
        ctx = torch.einsum("bht,btl->bhl", torch.softmax(scores, dim=-1), latent_cache.float())
    out = torch.bmm(ctx.transpose(0, 1), wuv.transpose(1, 2)).transpose(0, 1)  # [B,H,Dv]
    return out[:, None]


# --------------------------------------------------------------------------- sampling
def sample_tokens(logits, seen_bits, config, seed_offset):
    """Fused next-token choice for ``[B,V]`` logits -> ``[B]`` int64 (one launch).

    ``seen_bits`` is an int32 ``[B, ceil(V/32)]`` bitmap of tokens that take the repetition
    penalty (None: no penalty); ``seed_offset`` an int64 CUDA tensor ``{seed, draw counter}``."""
    pen = config.repetition_penalty
    return _C().sample_tokens(logits, seen_bits if pen not in (None, 1) else None, float(pen or 1.0),
                              float(config.temperature), int(config.top_k or 0),
                              float(config.top_p if config.top_p is not None else 1.0), bool(config.do_sample),
                              seed_offset)


def mark_seen(seen_bits, token_ids, vocab):
    """Set the bits of ``token_ids`` ``[B,T]`` in the ``[B, ceil(V/32)]`` bitmap (in place)."""
    _C().seen_mark(seen_bits, token_ids, int(vocab))


# --------------------------------------------------------------------------- router / MoE
class _RouterWeights(torch.autograd.Function):
    """Forward: fused kernel. Backward: gradient of the renormalised weights to the logits."""

    @staticmethod
    def forward(ctx, logits, bias, k, need_cutoff, eps, return_raw):
        sel, raw_sel, weights, cutoff, load, raw = _C().router(logits.contiguous(), bias, int(k), bool(need_cutoff),
                                                               float(eps), bool(return_raw))
        ctx.save_for_backward(sel, raw_sel, weights)
        ctx.shape = logits.shape
        ctx.dtype = logits.dtype
        ctx.eps = float(eps)
        ctx.mark_non_differentiable(sel, raw_sel, cutoff, load)
        if raw is not None and raw.numel():
            ctx.mark_non_differentiable(raw)
        return sel, raw_sel, weights, cutoff, load, raw

    @staticmethod
    def backward(ctx, _dsel, _draw, dw, _dc, _dl, _dr):
        sel, raw_sel, weights = ctx.saved_tensors
        denom = raw_sel.sum(-1, keepdim=True).clamp_min(ctx.eps)
        draw_sel = (dw - (dw * weights).sum(-1, keepdim=True)) / denom
        dlogit_sel = draw_sel * raw_sel * (1.0 - raw_sel)
        dlogits = torch.zeros(ctx.shape, dtype=torch.float32, device=dw.device)
        dlogits.scatter_add_(1, sel, dlogit_sel)
        return dlogits.to(ctx.dtype), None, None, None, None, None


def router_topk(logits, bias, k, need_cutoff, eps, return_raw):
    sel, raw_sel, weights, cutoff, load, raw = _RouterWeights.apply(logits, bias, k, need_cutoff, eps, return_raw)
    return sel, raw_sel, weights, cutoff, load, (raw if return_raw else None)


def qb_histogram(raw_scores, cutoffs, counts, underflow, overflow, min_margin, max_margin):
    e, bins = counts.shape
    margins = raw_scores.float() - cutoffs.float()[:, None]
    underflow.add_((margins < min_margin).sum(0))
    overflow.add_((margins >= max_margin).sum(0))
    width = (max_margin - min_margin) / bins
    idx = torch.floor((margins - min_margin) / width).long().clamp_(0, bins - 1)
    flat = idx + torch.arange(e, device=margins.device)[None, :] * bins
    # scatter_add (atomics) rather than bincount: bincount reads the max index on the host
    counts.view(-1).scatter_add_(0, flat.reshape(-1), torch.ones_like(flat.reshape(-1), dtype=counts.dtype))


class _MoEGrouped(torch.autograd.Function):
    """Routed experts as grouped tcgen05 GEMMs over 128-row aligned expert segments.

    Forward: device routing -> gather -> [gate|up] GEMM with the SiTU-GLU epilogue ->
    down GEMM with a weighted scatter-add epilogue into the fp32 aggregate.
    Backward: recompute Y, dY / d(weight), dH = dY Wd, dWd = dY^T H, SiTU backward,
    dX = [dG|dU] [Wg; Wu], dWg / dWu = [dG|dU]^T X, then the per-token slot sum.
    """

    @staticmethod
    def forward(ctx, latent, weights, selected, gate_w, up_w, down_w, bg, bu):
        C = _C()
        m, l = latent.shape
        k = selected.shape[1]
        e, h, _ = gate_w.shape
        r_max = m * k + e * 128
        bf = torch.bfloat16
        x = latent.to(bf).contiguous()
        from .mirror import bf16_weight
        wg, wu, wd = (bf16_weight(w).contiguous() for w in (gate_w, up_w, down_w))
        _, offsets, row_token, row_weight, row_of = C.moe_route(selected.contiguous(), weights.detach(), e, r_max)
        xs = C.moe_gather(x, row_token)
        hh, gg, uu = C.tc_gemm_grouped(1, xs, wg, wu, False, False, offsets, r_max, h, l, 1, None, False, bg, bu,
                                       None, None, 0, 256)
        agg = torch.zeros(m, l, device=latent.device, dtype=torch.float32)
        C.tc_gemm_grouped(1, hh, wd, None, False, False, offsets, r_max, l, h, 2, agg, True, bg, bu, row_token,
                          row_weight, 0, 128)
        ctx.save_for_backward(xs, gg, uu, hh, wg, wu, wd, offsets, row_token, row_weight, row_of)
        ctx.c = (m, k, e, h, l, r_max, float(bg), float(bu), latent.dtype, gate_w.dtype)
        ctx.mark_non_differentiable()
        return agg

    @staticmethod
    def backward(ctx, dagg):
        C = _C()
        xs, gg, uu, hh, wg, wu, wd, offsets, row_token, row_weight, row_of = ctx.saved_tensors
        m, k, e, h, l, r_max, bg, bu, ldt, wdt = ctx.c
        y, = C.tc_gemm_grouped(1, hh, wd, None, False, False, offsets, r_max, l, h, 0, None, False, bg, bu, None, None,
                               0, 256)
        dy, dw_row = C.moe_dy(dagg, row_token, row_weight, y)
        dh, = C.tc_gemm_grouped(1, dy, wd, None, False, True, offsets, r_max, h, l, 0, None, False, bg, bu, None, None,
                                0, 256)
        dwd, = C.tc_gemm_grouped(2, dy, hh, None, True, True, offsets, l, h, r_max, 0, None, True, bg, bu, None, None,
                                 0, 256)
        dgu = C.situ_bwd_cat(dh, gg, uu, bg, bu)
        dxs, = C.tc_gemm_grouped(1, dgu, wg, wu, False, True, offsets, r_max, l, 2 * h, 0, None, False, bg, bu, None,
                                 None, h, 256)
        dwg, = C.tc_gemm_grouped(2, dgu[:, :h], xs, None, True, True, offsets, h, l, r_max, 0, None, True, bg, bu,
                                 None, None, 0, 256)
        dwu, = C.tc_gemm_grouped(2, dgu[:, h:], xs, None, True, True, offsets, h, l, r_max, 0, None, True, bg, bu,
                                 None, None, 0, 256)
        dlat = C.moe_slot_sum(dxs, row_of, m, k, ldt == torch.float32)
        dweights = dw_row.index_select(0, row_of.long().clamp_min(0)).view(m, k)
        return dlat.to(ldt), dweights, None, dwg.to(wdt), dwu.to(wdt), dwd.to(wdt), None, None


def moe_grouped_experts(latent, selected, weights, gate_w, up_w, down_w, beta_gate, beta_up):
    """``sum_k w_k E_{sel_k}(latent)`` in fp32 (routed experts, grouped tcgen05 GEMMs)."""
    l, h = latent.shape[1], gate_w.shape[1]
    if l % 64 or h % 128:
        raise NotImplementedError("grouped expert GEMMs need latent % 64 == 0 and hidden % 128 == 0")
    return _MoEGrouped.apply(latent, weights, selected, gate_w, up_w, down_w, float(beta_gate), float(beta_up))


# --------------------------------------------------------------------------- AttnRes
class _AttnResMix(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, w, eps, *sources):
        srcs = [s.contiguous() for s in sources]
        out, probs, rstd = _C().attnres_fwd(srcs, q, w, float(eps))
        ctx.save_for_backward(q, w, probs, rstd, *srcs)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, w, probs, rstd, *srcs = ctx.saved_tensors
        grads = _C().attnres_bwd(list(srcs), q, w, dout, probs, rstd)
        dsrc, dq, dw = grads[:-2], grads[-2], grads[-1]
        return (dq.to(q.dtype), dw.to(w.dtype), None, *dsrc)


def attnres_mix(sources, pseudo_query, key_norm_weight, eps):
    """Depth softmax mix of ``S`` same-shape ``[B,T,D]`` sources (one fused pass)."""
    dt = sources[0].dtype
    srcs = [s if s.dtype == dt else s.to(dt) for s in sources]
    return _AttnResMix.apply(pseudo_query, key_norm_weight, eps, *srcs)


# --------------------------------------------------------------------------- LM head + CE
class _LinearCE(torch.autograd.Function):
    """``sum_valid CE(h @ W^T, t)``; gradients are formed in forward on the tcgen05 GEMM.

    Per row chunk (up to ``chunk_rows``): logits = h_c W^T in bf16 with a 64-aligned row stride,
    the fused row kernel writes the loss and (softmax - onehot) in place, then dh_c = G W and
    dW (+)= G^T h_c in fp32. The [N, V] fp32 probability tensor never exists; backward only
    scales by the incoming scalar gradient. Reference: ``src/loss/common/cross_entropy.py:41-46``
    (logits materialised in fp32, CE through ``F.cross_entropy``).
    """

    @staticmethod
    def forward(ctx, h, w, targets, valid, chunk_rows):
        n, d = h.shape
        v = w.shape[0]
        from .mirror import bf16_weight
        wd = bf16_weight(w).contiguous()
        vpad = (v + 63) // 64 * 64
        loss = torch.zeros((), device=h.device, dtype=torch.float32)
        dh = torch.empty_like(h)
        dw = None
        rows_per = min(chunk_rows, n)
        buf = torch.empty(rows_per, vpad, device=h.device, dtype=torch.bfloat16)
        C = _C()
        for s in range(0, n, rows_per):
            e = min(n, s + rows_per)
            hc = h[s:e]
            lg = buf[: e - s, :v]
            C.tc_gemm_dense(hc, wd, False, False, False, 256, lg)
            loss += C.ce_rows(lg, v, targets[s:e], valid[s:e], 1.0).sum()
            # BN = 256 for all three products: 1.08 / 1.05 ms vs 1.52 / 1.46 ms with BN = 128 for dh / dW
            # at 16384 x 50257 x 640 on B200
            C.tc_gemm_dense(lg, wd, False, True, False, 256, dh[s:e])
            part = C.tc_gemm_dense(lg, hc, True, True, True, 256, None)
            dw = part if dw is None else dw.add_(part)
        ctx.save_for_backward(dh, dw)
        ctx.w_dtype = w.dtype
        return loss

    @staticmethod
    def backward(ctx, gl):
        dh, dw = ctx.saved_tensors
        return dh * gl.to(dh.dtype), (dw * gl).to(ctx.w_dtype), None, None, None


def linear_cross_entropy(hidden, weight, targets, valid, chunk_rows: int = 16384):
    """Sum of token CE losses of ``hidden @ weight^T`` over valid rows (fp32 scalar)."""
    if hidden.shape[-1] % 8:
        raise ValueError("linear_cross_entropy needs a hidden width that is a multiple of 8")
    h = hidden.to(torch.bfloat16).contiguous()
    return _LinearCE.apply(h, weight, targets.contiguous(), valid.contiguous(), int(chunk_rows))


__all__ = [
    "linear", "linear_supported", "linear_group", "linear_group_supported", "gemm_tiles", "wgrad_splits", "rms_norm", "situ_glu", "sigmoid_mul", "kda_decay", "conv_silu_norm", "kda_chunk", "kda_decode_step",
    "conv_silu_norm_step", "mla_decode_supported", "sample_tokens", "mark_seen",
    "flash_attention", "mla_absorbed_decode", "router_topk", "qb_histogram", "moe_grouped_experts",
    "attnres_mix", "linear_cross_entropy",
]
