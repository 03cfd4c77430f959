"""Decode-step kernels against plain fp32 PyTorch references, and the CUDA-graph serving decoder
against its own eager replay and against the reference-style generation loop."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    scale = max(b.abs().max().item(), 1e-6)
    assert err <= tol * scale, f"max err {err:.3e} vs scale {scale:.3e} (tol {tol})"


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("ksize,bias", [(4, False), (3, True)])
def test_conv_step(cuda, dtype, ksize, bias):
    from kimi_k3_b200 import ops
    torch.manual_seed(0)
    b, widths, hds = 3, (640, 640, 384), (64, 64, 0)
    xs = [torch.randn(b, 1, c, device=cuda).to(dtype) for c in widths]
    hists = [torch.randn(b, ksize - 1, c, device=cuda).to(dtype) for c in widths]
    ws = [0.3 * torch.randn(c, ksize, device=cuda) for c in widths]
    bs = [0.1 * torch.randn(c, device=cuda) if bias else None for c in widths]
    refs, ref_hist = [], []
    for x, h, w, bb, hd in zip(xs, hists, ws, bs, hds):
        comb = torch.cat((h.float(), x.float()), 1)  # oldest first
        pre = F.conv1d(comb.transpose(1, 2), w.flip(-1).unsqueeze(1), bb, groups=w.shape[0]).transpose(1, 2)
        s = F.silu(pre)
        if hd:
            s = F.normalize(s.reshape(b, 1, -1, hd), dim=-1, eps=1e-6).reshape(b, 1, -1)
        refs.append(s)
        ref_hist.append(comb[:, 1:].to(dtype))
    hs = [h.clone() for h in hists]
    ys = ops.conv_silu_norm_step(xs, hs, ws, bs, hds, 1e-6)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for y, r, h, rh in zip(ys, refs, hs, ref_hist):
        _close(y, r, tol)
        assert torch.equal(h, rh)  # the history shifted in place


@pytest.mark.parametrize("inplace", [False, True])
def test_kda_decode_step(cuda, inplace):
    from kimi_k3_b200 import ops
    torch.manual_seed(1)
    b, h = 3, 10
    q = F.normalize(torch.randn(b, 1, h, 64, device=cuda), dim=-1).bfloat16()
    k = F.normalize(torch.randn(b, 1, h, 64, device=cuda), dim=-1).bfloat16()
    v = torch.randn(b, 1, h, 64, device=cuda).bfloat16()
    g = -torch.rand(b, 1, h, 64, device=cuda)
    beta = torch.rand(b, 1, h, device=cuda)
    s0 = torch.randn(b, h, 64, 64, device=cuda)
    st = s0.clone()
    o, ns = ops.kda_decode_step(q, k, v, g, beta, st, out_state=st if inplace else None)
    qf, kf, vf, gf, bf = (x[:, 0].float() for x in (q, k, v, g, beta))
    s = s0 * torch.exp(gf)[..., None]
    err = vf - torch.einsum("bhkv,bhk->bhv", s, kf)
    s = s + torch.einsum("bhk,bhv->bhkv", bf[..., None] * kf, err)
    ro = torch.einsum("bhkv,bhk->bhv", s, qf)
    _close(ns, s, 1e-5)
    _close(o[:, 0], ro, 1e-2)
    if inplace:
        assert ns.data_ptr() == st.data_ptr()
    else:
        assert torch.equal(st, s0)


@pytest.mark.parametrize("heads,ldim,dtype", [(10, 640, torch.bfloat16), (12, 768, torch.bfloat16),
                                               (24, 512, torch.float32), (16, 1024, torch.bfloat16),
                                               (3, 1536, torch.bfloat16), (12, 1536, torch.bfloat16),
                                               (6, 1536, torch.float32), (2, 64, torch.bfloat16),
                                               (16, 512, torch.bfloat16), (1, 768, torch.bfloat16)])
def test_mla_absorbed_decode(cuda, heads, ldim, dtype):
    from kimi_k3_b200 import ops
    torch.manual_seed(2)
    b, tmax, dq = 3, 301, 64
    lengths = torch.tensor([301, 77, 1], dtype=torch.int32, device=cuda)
    query = torch.randn(b, 1, heads, dq, device=cuda)
    latent = torch.randn(b, tmax, ldim, device=cuda).to(dtype)
    wuk = torch.randn(heads * dq, ldim, device=cuda) / math.sqrt(ldim)
    wuv = torch.randn(heads * 64, ldim, device=cuda) / math.sqrt(ldim)
    out = ops.mla_absorbed_decode(query, latent, None, wuk, wuv, lengths=lengths)
    mask = torch.arange(tmax, device=cuda)[None, :] < lengths[:, None].long()
    q_lat = torch.einsum("bhd,hdl->bhl", query[:, 0], wuk.reshape(heads, dq, ldim)) / math.sqrt(dq)
    sc = torch.einsum("bhl,btl->bht", q_lat, latent.float()).masked_fill(~mask[:, None], -torch.inf)
    ctx = torch.einsum("bht,btl->bhl", torch.softmax(sc, -1), latent.float())
    ref_out = torch.einsum("bhl,hvl->bhv", ctx, wuv.reshape(heads, 64, ldim))[:, None]
    assert ops.mla_decode_supported(heads, ldim)
    _close(out, ref_out, 2e-4)


def test_sample_greedy_and_penalty(cuda):
    from kimi_k3_b200 import ops
    from kimi_k3_b200.infer import GenerationConfig, apply_repetition_penalty, sample_next_token
    torch.manual_seed(3)
    b, vocab = 6, 50257
    logits = torch.randn(b, vocab, device=cuda) * 3
    logits[1, 17] = float("nan")
    logits[2, 5] = float("inf")
    logits[3] = float("-inf")
    logits[3, 9000] = 0.5
    logits[4, 100] = logits[4, 200] = 50.0  # tie: the first index wins
    hist = torch.randint(0, vocab, (b, 40), device=cuda)
    seen = torch.zeros(b, (vocab + 31) // 32, dtype=torch.int32, device=cuda)
    ops.mark_seen(seen, hist, vocab)
    so = torch.tensor([0, 0], dtype=torch.long, device=cuda)
    for pen in (None, 1.7):
        cfg = GenerationConfig(repetition_penalty=pen)
        got = ops.sample_tokens(logits, seen, cfg, so)
        ref = sample_next_token(logits, cfg, previous_token_ids=hist)[:, 0]
        assert torch.equal(got, ref), (got, ref)
    # top-k = 1 and a tiny nucleus reduce sampling to the greedy choice of the penalised logits
    fin = torch.randn(b, vocab, device=cuda)
    target = apply_repetition_penalty(fin, hist, 1.7).argmax(-1)
    for cfg in (GenerationConfig(do_sample=True, top_k=1, repetition_penalty=1.7),
                GenerationConfig(do_sample=True, top_p=1e-6, repetition_penalty=1.7, temperature=0.5)):
        assert torch.equal(ops.sample_tokens(fin, seen, cfg, so), target)


def test_sample_distribution(cuda):
    """Many rows with the same logits: the empirical frequencies follow the top-k / top-p
    filtered, tempered softmax, and nothing outside the kept set is drawn."""
    from kimi_k3_b200 import ops
    from kimi_k3_b200.infer import GenerationConfig, top_k_filter, top_p_filter
    torch.manual_seed(4)
    rows, vocab = 16384, 1000
    base = torch.randn(vocab, device=cuda) * 2  # fp32: no ties at the top-k / top-p boundaries
    logits = base[None].expand(rows, vocab).contiguous()
    cfg = GenerationConfig(do_sample=True, top_k=50, top_p=0.8, temperature=0.7)
    filt = top_p_filter(top_k_filter(logits[:1] / 0.7, 50), 0.8)
    probs = torch.softmax(filt, -1)[0]
    counts = torch.zeros(vocab, device=cuda)
    so = torch.tensor([1234, 0], dtype=torch.long, device=cuda)
    for _ in range(4):
        tok = ops.sample_tokens(logits, None, cfg, so)
        so[1] += 1
        counts += torch.bincount(tok, minlength=vocab).float()
    freq = counts / counts.sum()
    assert float(freq[probs == 0].sum()) == 0.0
    tv = 0.5 * float((freq - probs).abs().sum())
    assert tv < 0.03, tv
    # the draw counter changes the draws
    a = ops.sample_tokens(logits, None, cfg, torch.tensor([5, 0], dtype=torch.long, device=cuda))
    c = ops.sample_tokens(logits, None, cfg, torch.tensor([5, 1], dtype=torch.long, device=cuda))
    assert not torch.equal(a, c)


def _small_model(cuda):
    from kimi_k3_b200.config.model_yaml import build_model_config_from_mapping
    from kimi_k3_b200.config.profiles import profile_model_mapping
    from kimi_k3_b200.models import KimiK3
    m = profile_model_mapping("t4_wikitext")
    m["model"].update(d_model=128, num_heads=2, num_hybrid_groups=1, vocab_size=1000)
    m["model"]["moe"].update(latent_dim=64, shared_expert_hidden_dim=96, routed_expert_hidden_dim=128)
    m["model"]["mla"]["kv_latent_dim"] = 128
    torch.manual_seed(5)
    return KimiK3(build_model_config_from_mapping(m)).to(cuda).eval()


def test_graph_decoder(cuda):
    from kimi_k3_b200.infer import GenerationConfig, GraphDecoder, generate_tokens
    model = _small_model(cuda)
    ids = torch.randint(5, 1000, (4, 37), device=cuda)
    mask = torch.ones_like(ids, dtype=torch.bool)
    mask[2, 20:] = False
    for cfg in (GenerationConfig(max_new_tokens=12),
                GenerationConfig(max_new_tokens=12, do_sample=True, top_k=40, top_p=0.9, temperature=0.8,
                                 repetition_penalty=1.2, seed=11)):
        graph = GraphDecoder(model, max_length=64, generation_config=cfg).generate(ids, mask)
        eager = GraphDecoder(model, max_length=64, generation_config=cfg, use_graph=False).generate(ids, mask)
        assert graph.generated_tokens == 12
        assert torch.equal(graph.generated_ids, eager.generated_ids)
    # fp32 graph decoding follows the reference-style loop (same greedy tokens)
    cfg = GenerationConfig(max_new_tokens=8)
    ref_out = generate_tokens(model, ids, generation_config=cfg, attention_mask=mask)
    dec = GraphDecoder(model, max_length=64, generation_config=cfg, autocast_dtype=None)
    out = dec.generate(ids, mask)
    assert dec.replays == 7
    assert torch.equal(out.generated_ids, ref_out.generated_ids), (out.generated_ids, ref_out.generated_ids)
    # a second generation with the same batch shape refills the buffers and replays the same graph
    graph = dec.graph
    ids2 = torch.randint(5, 1000, (4, 30), device=cuda)
    again = dec.generate(ids2)
    assert dec.graph is graph and dec.replays == 14
    fresh = GraphDecoder(model, max_length=64, generation_config=cfg, autocast_dtype=None).generate(ids2)
    assert torch.equal(again.generated_ids, fresh.generated_ids)
