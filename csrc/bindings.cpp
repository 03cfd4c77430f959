// PyTorch bindings for the kimi_k3_b200 sm_100a kernels. Each binding validates shapes,
// dtypes and contiguity, allocates outputs with the caching allocator and launches on the
// current CUDA stream. Launch errors raise immediately.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include "kernels.h"

namespace {

int dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return 0;
    case at::kBFloat16: return 1;
    case at::kHalf: return 2;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void check(cudaError_t e, const char* what) {
  TORCH_CHECK(e == cudaSuccess, what, " failed: ", cudaGetErrorString(e));
}

#define CHECK_CUDA_CONTIG(x) TORCH_CHECK((x).is_cuda() && (x).is_contiguous(), #x " must be a contiguous CUDA tensor")

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream(); }

// ---------------------------------------------------------------- RMSNorm
std::vector<at::Tensor> rms_norm_fwd(at::Tensor x, at::Tensor w, double eps, int64_t period) {
  CHECK_CUDA_CONTIG(x);
  const at::cuda::CUDAGuard g(x.device());
  const int dim = x.size(-1);
  const int64_t rows = x.numel() / dim;
  auto y = at::empty_like(x);
  auto rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  const float* wp = nullptr;
  at::Tensor wf;
  if (w.defined() && w.numel()) {
    wf = w.to(at::kFloat).contiguous();
    wp = wf.data_ptr<float>();
  }
  check(kimi::rms_norm_fwd(dtype_code(x), x.data_ptr(), wp, y.data_ptr(), rstd.data_ptr<float>(), rows, dim,
                           (int)period, (float)eps, stream()), "rms_norm_fwd");
  return {y, rstd};
}

std::vector<at::Tensor> rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, int64_t period,
                                     bool need_dw) {
  CHECK_CUDA_CONTIG(x);
  dy = dy.contiguous();
  const at::cuda::CUDAGuard g(x.device());
  const int dim = x.size(-1);
  const int64_t rows = x.numel() / dim;
  auto dx = at::empty_like(x);
  at::Tensor wf, dw;
  const float* wp = nullptr;
  float* dwp = nullptr;
  if (w.defined() && w.numel()) {
    wf = w.to(at::kFloat).contiguous();
    wp = wf.data_ptr<float>();
    if (need_dw) {
      dw = at::zeros({wf.numel()}, x.options().dtype(at::kFloat));
      dwp = dw.data_ptr<float>();
    }
  }
  check(kimi::rms_norm_bwd(dtype_code(x), dy.data_ptr(), x.data_ptr(), wp, rstd.data_ptr<float>(), dx.data_ptr(),
                           dwp, rows, dim, (int)period, stream()), "rms_norm_bwd");
  return {dx, dw.defined() ? dw.view(w.sizes()) : dw};
}

// ---------------------------------------------------------------- elementwise
at::Tensor situ_fwd(at::Tensor g, at::Tensor u, double bg, double bu) {
  CHECK_CUDA_CONTIG(g);
  CHECK_CUDA_CONTIG(u);
  const at::cuda::CUDAGuard gd(g.device());
  auto y = at::empty_like(g);
  check(kimi::situ_glu_fwd(dtype_code(g), g.data_ptr(), u.data_ptr(), y.data_ptr(), g.numel(), (float)bg, (float)bu,
                           stream()), "situ_glu_fwd");
  return y;
}

std::vector<at::Tensor> situ_bwd(at::Tensor dy, at::Tensor g, at::Tensor u, double bg, double bu) {
  dy = dy.contiguous();
  const at::cuda::CUDAGuard gd(g.device());
  auto dg = at::empty_like(g), du = at::empty_like(u);
  check(kimi::situ_glu_bwd(dtype_code(g), dy.data_ptr(), g.data_ptr(), u.data_ptr(), dg.data_ptr(), du.data_ptr(),
                           g.numel(), (float)bg, (float)bu, stream()), "situ_glu_bwd");
  return {dg, du};
}

at::Tensor sigmul_fwd(at::Tensor z, at::Tensor x) {
  CHECK_CUDA_CONTIG(z);
  CHECK_CUDA_CONTIG(x);
  const at::cuda::CUDAGuard gd(z.device());
  auto y = at::empty_like(x);
  check(kimi::sigmoid_mul_fwd(dtype_code(x), z.data_ptr(), x.data_ptr(), y.data_ptr(), x.numel(), stream()),
        "sigmoid_mul_fwd");
  return y;
}

std::vector<at::Tensor> sigmul_bwd(at::Tensor dy, at::Tensor z, at::Tensor x) {
  dy = dy.contiguous();
  const at::cuda::CUDAGuard gd(z.device());
  auto dz = at::empty_like(z), dx = at::empty_like(x);
  check(kimi::sigmoid_mul_bwd(dtype_code(x), dy.data_ptr(), z.data_ptr(), x.data_ptr(), dz.data_ptr(), dx.data_ptr(),
                              x.numel(), stream()), "sigmoid_mul_bwd");
  return {dz, dx};
}

at::Tensor decay_fwd(at::Tensor z, at::Tensor a_log, double g_min, double ceps) {
  CHECK_CUDA_CONTIG(z);
  const at::cuda::CUDAGuard gd(z.device());
  const int heads = z.size(-2), kdim = z.size(-1);
  const int64_t rows = z.numel() / (heads * kdim);
  auto g = at::empty(z.sizes(), z.options().dtype(at::kFloat));
  auto af = a_log.to(at::kFloat).contiguous();
  check(kimi::kda_decay_fwd(dtype_code(z), z.data_ptr(), af.data_ptr<float>(), g.data_ptr<float>(), rows, heads, kdim,
                            (float)g_min, (float)ceps, stream()), "kda_decay_fwd");
  return g;
}

std::vector<at::Tensor> decay_bwd(at::Tensor dg, at::Tensor z, at::Tensor a_log, double g_min, double ceps) {
  dg = dg.to(at::kFloat).contiguous();
  const at::cuda::CUDAGuard gd(z.device());
  const int heads = z.size(-2), kdim = z.size(-1);
  const int64_t rows = z.numel() / (heads * kdim);
  auto dz = at::empty_like(z);
  auto af = a_log.to(at::kFloat).contiguous();
  auto da = at::zeros({heads}, z.options().dtype(at::kFloat));
  check(kimi::kda_decay_bwd(dtype_code(z), dg.data_ptr<float>(), z.data_ptr(), af.data_ptr<float>(), dz.data_ptr(),
                            da.data_ptr<float>(), rows, heads, kdim, (float)g_min, (float)ceps, stream()),
        "kda_decay_bwd");
  return {dz, da};
}

at::Tensor conv_fwd(at::Tensor x, at::Tensor w, int64_t head_dim, double eps, bool normalize) {
  CHECK_CUDA_CONTIG(x);
  const at::cuda::CUDAGuard gd(x.device());
  auto wf = w.to(at::kFloat).contiguous();
  auto y = at::empty_like(x);
  check(kimi::conv_silu_norm_fwd(dtype_code(x), x.data_ptr(), wf.data_ptr<float>(), y.data_ptr(), x.size(0),
                                 x.size(1), x.size(2), wf.size(1), (int)head_dim, (float)eps, normalize, stream()),
        "conv_silu_norm_fwd");
  return y;
}

std::vector<at::Tensor> conv_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, int64_t head_dim, double eps,
                                 bool normalize) {
  dy = dy.contiguous();
  const at::cuda::CUDAGuard gd(x.device());
  auto wf = w.to(at::kFloat).contiguous();
  auto dpre = at::empty(x.sizes(), x.options().dtype(at::kFloat));
  auto dx = at::empty_like(x);
  auto dw = at::zeros(wf.sizes(), wf.options());
  check(kimi::conv_silu_norm_bwd(dtype_code(x), dy.data_ptr(), x.data_ptr(), wf.data_ptr<float>(),
                                 dpre.data_ptr<float>(), dx.data_ptr(), dw.data_ptr<float>(), x.size(0), x.size(1),
                                 x.size(2), wf.size(1), (int)head_dim, (float)eps, normalize, stream()),
        "conv_silu_norm_bwd");
  return {dx, dw};
}

// ---------------------------------------------------------------- AttnRes
std::vector<at::Tensor> attnres_fwd(std::vector<at::Tensor> sources, at::Tensor q, at::Tensor w, double eps) {
  const auto& s0 = sources.at(0);
  const at::cuda::CUDAGuard gd(s0.device());
  std::vector<const void*> ptrs;
  for (auto& s : sources) {
    CHECK_CUDA_CONTIG(s);
    TORCH_CHECK(s.sizes() == s0.sizes() && s.scalar_type() == s0.scalar_type(), "sources must match");
    ptrs.push_back(s.data_ptr());
  }
  const int dim = s0.size(-1);
  const int64_t tokens = s0.numel() / dim;
  const int S = (int)sources.size();
  auto out = at::empty_like(s0);
  auto probs = at::empty({tokens, S}, s0.options().dtype(at::kFloat));
  auto rstd = at::empty({tokens, S}, s0.options().dtype(at::kFloat));
  auto qf = q.to(at::kFloat).contiguous(), wf = w.to(at::kFloat).contiguous();
  check(kimi::attnres_mix_fwd(dtype_code(s0), ptrs.data(), S, qf.data_ptr<float>(), wf.data_ptr<float>(),
                              out.data_ptr(), probs.data_ptr<float>(), rstd.data_ptr<float>(), tokens, dim,
                              (float)eps, stream()), "attnres_mix_fwd");
  return {out, probs, rstd};
}

std::vector<at::Tensor> attnres_bwd(std::vector<at::Tensor> sources, at::Tensor q, at::Tensor w, at::Tensor dout,
                                    at::Tensor probs, at::Tensor rstd) {
  const auto& s0 = sources.at(0);
  const at::cuda::CUDAGuard gd(s0.device());
  dout = dout.contiguous();
  std::vector<const void*> ptrs;
  std::vector<void*> dptrs;
  std::vector<at::Tensor> grads;
  for (auto& s : sources) {
    ptrs.push_back(s.data_ptr());
    grads.push_back(at::empty_like(s));
    dptrs.push_back(grads.back().data_ptr());
  }
  const int dim = s0.size(-1);
  const int64_t tokens = s0.numel() / dim;
  auto qf = q.to(at::kFloat).contiguous(), wf = w.to(at::kFloat).contiguous();
  auto dq = at::zeros({dim}, s0.options().dtype(at::kFloat));
  auto dw = at::zeros({dim}, s0.options().dtype(at::kFloat));
  check(kimi::attnres_mix_bwd(dtype_code(s0), ptrs.data(), (int)sources.size(), qf.data_ptr<float>(),
                              wf.data_ptr<float>(), dout.data_ptr(), probs.data_ptr<float>(), rstd.data_ptr<float>(),
                              dptrs.data(), dq.data_ptr<float>(), dw.data_ptr<float>(), tokens, dim, stream()),
        "attnres_mix_bwd");
  grads.push_back(dq);
  grads.push_back(dw);
  return grads;
}

// ---------------------------------------------------------------- CE rows (in place)
at::Tensor ce_rows(at::Tensor logits, int64_t vocab, at::Tensor targets, at::Tensor valid, double grad_scale) {
  TORCH_CHECK(logits.is_cuda() && logits.stride(1) == 1, "logits rows must be unit-stride");
  const at::cuda::CUDAGuard gd(logits.device());
  const int64_t rows = logits.size(0);
  auto loss = at::empty({rows}, logits.options().dtype(at::kFloat));
  auto t = targets.to(at::kLong).contiguous();
  auto v = valid.to(at::kBool).contiguous();
  check(kimi::ce_rows_fwd_bwd(dtype_code(logits), logits.data_ptr(), logits.stride(0), rows, (int)vocab,
                              t.data_ptr<int64_t>(), v.data_ptr<bool>(), loss.data_ptr<float>(), (float)grad_scale,
                              stream()), "ce_rows_fwd_bwd");
  return loss;
}

// ---------------------------------------------------------------- router
std::vector<at::Tensor> router(at::Tensor logits, at::Tensor bias, int64_t k, bool need_cutoff, double eps,
                               bool return_raw) {
  CHECK_CUDA_CONTIG(logits);
  const at::cuda::CUDAGuard gd(logits.device());
  const int64_t rows = logits.size(0);
  const int experts = logits.size(1);
  auto f = logits.options().dtype(at::kFloat);
  auto sel = at::empty({rows, k}, logits.options().dtype(at::kLong));
  auto raw_sel = at::empty({rows, k}, f), weights = at::empty({rows, k}, f);
  auto cutoff = at::empty({rows}, f);
  auto load = at::zeros({experts}, logits.options().dtype(at::kLong));
  at::Tensor raw = return_raw ? at::empty({rows, experts}, f) : at::Tensor();
  auto bf = bias.to(at::kFloat).contiguous();
  check(kimi::router_topk(dtype_code(logits), logits.data_ptr(), bf.data_ptr<float>(), rows, experts, (int)k,
                          need_cutoff, (float)eps, sel.data_ptr<int64_t>(), raw_sel.data_ptr<float>(),
                          weights.data_ptr<float>(), cutoff.data_ptr<float>(), load.data_ptr<int64_t>(),
                          return_raw ? raw.data_ptr<float>() : nullptr, stream()), "router_topk");
  return {sel, raw_sel, weights, cutoff, load, raw};
}

// ---------------------------------------------------------------- KDA chunk
std::vector<at::Tensor> kda_fwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                                c10::optional<at::Tensor> h0, bool want_final) {
  CHECK_CUDA_CONTIG(q);
  CHECK_CUDA_CONTIG(k);
  CHECK_CUDA_CONTIG(v);
  CHECK_CUDA_CONTIG(g);
  CHECK_CUDA_CONTIG(beta);
  TORCH_CHECK(g.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat, "g and beta must be float32");
  TORCH_CHECK(q.size(3) == 64 && v.size(3) == 64, "KDA kernel supports head dims of 64");
  const at::cuda::CUDAGuard gd(q.device());
  const int B = q.size(0), Tp = q.size(1), H = q.size(2);
  TORCH_CHECK(Tp % 64 == 0, "tokens must be padded to a multiple of 64");
  const int NC = Tp / 64;
  auto f = q.options().dtype(at::kFloat);
  auto W = at::empty({B * H, NC, 64, 64}, f), U = at::empty_like(W), P = at::empty_like(W), Qg = at::empty_like(W),
       Kend = at::empty_like(W), states = at::empty_like(W), Vp = at::empty_like(W);
  auto eGC = at::empty({B * H, NC, 64}, f);
  auto o = at::empty_like(v);
  at::Tensor ht = want_final ? at::empty({B, H, 64, 64}, f) : at::Tensor();
  at::Tensor h0c;
  if (h0.has_value() && h0->defined()) h0c = h0->to(at::kFloat).contiguous();
  kimi::KdaBuffers buf{W.data_ptr<float>(), U.data_ptr<float>(), P.data_ptr<float>(), Qg.data_ptr<float>(),
                       Kend.data_ptr<float>(), eGC.data_ptr<float>(), states.data_ptr<float>(), Vp.data_ptr<float>()};
  check(kimi::kda_chunk_fwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(),
                            beta.data_ptr<float>(), h0c.defined() ? h0c.data_ptr<float>() : nullptr, o.data_ptr(),
                            want_final ? ht.data_ptr<float>() : nullptr, buf, B, Tp, H, stream()), "kda_chunk_fwd");
  return {o, ht, W, U, P, Qg, Kend, eGC, states, Vp};
}

std::vector<at::Tensor> kda_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                                std::vector<at::Tensor> saved, at::Tensor dout, c10::optional<at::Tensor> dht,
                                bool want_dh0) {
  const at::cuda::CUDAGuard gd(q.device());
  dout = dout.contiguous();
  const int B = q.size(0), Tp = q.size(1), H = q.size(2);
  auto f = q.options().dtype(at::kFloat);
  auto& W = saved.at(0);
  kimi::KdaBuffers buf{saved[0].data_ptr<float>(), saved[1].data_ptr<float>(), saved[2].data_ptr<float>(),
                       saved[3].data_ptr<float>(), saved[4].data_ptr<float>(), saved[5].data_ptr<float>(),
                       saved[6].data_ptr<float>(), saved[7].data_ptr<float>()};
  auto dVp = at::empty_like(W), dSn = at::empty_like(W);
  auto dq = at::empty(q.sizes(), f), dk = at::empty(k.sizes(), f), dv = at::empty(v.sizes(), f),
       dg = at::empty(g.sizes(), f), dbeta = at::empty(beta.sizes(), f);
  at::Tensor dh0 = want_dh0 ? at::empty({B, H, 64, 64}, f) : at::Tensor();
  at::Tensor dhtc;
  if (dht.has_value() && dht->defined()) dhtc = dht->to(at::kFloat).contiguous();
  check(kimi::kda_chunk_bwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(),
                            beta.data_ptr<float>(), buf, dout.data_ptr(),
                            dhtc.defined() ? dhtc.data_ptr<float>() : nullptr, dVp.data_ptr<float>(),
                            dSn.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr<float>(), dv.data_ptr<float>(),
                            dg.data_ptr<float>(), dbeta.data_ptr<float>(),
                            want_dh0 ? dh0.data_ptr<float>() : nullptr, B, Tp, H, stream()), "kda_chunk_bwd");
  return {dq, dk, dv, dg, dbeta, dh0};
}

// ---------------------------------------------------------------- flash attention
std::vector<at::Tensor> fa_fwd(at::Tensor q, at::Tensor k, at::Tensor v, bool causal,
                               c10::optional<at::Tensor> key_lengths, double scale) {
  CHECK_CUDA_CONTIG(q);
  CHECK_CUDA_CONTIG(k);
  CHECK_CUDA_CONTIG(v);
  const at::cuda::CUDAGuard gd(q.device());
  const int B = q.size(0), tq = q.size(1), H = q.size(2), tk = k.size(1);
  auto o = at::empty({B, tq, H, v.size(3)}, q.options());
  auto lse = at::empty({B, H, tq}, q.options().dtype(at::kFloat));
  at::Tensor kl;
  if (key_lengths.has_value() && key_lengths->defined()) kl = key_lengths->to(at::kInt).contiguous();
  check(kimi::flash_attn_fwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                             lse.data_ptr<float>(), B, tq, tk, H, q.size(3), v.size(3), causal,
                             kl.defined() ? kl.data_ptr<int>() : nullptr, (float)scale, stream()), "flash_attn_fwd");
  return {o, lse};
}

std::vector<at::Tensor> fa_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor dout, at::Tensor lse,
                               bool causal, c10::optional<at::Tensor> key_lengths, double scale) {
  const at::cuda::CUDAGuard gd(q.device());
  dout = dout.contiguous();
  const int B = q.size(0), tq = q.size(1), H = q.size(2), tk = k.size(1);
  auto dq = at::zeros(q.sizes(), q.options().dtype(at::kFloat));
  auto dk = at::empty_like(k), dv = at::empty_like(v);
  auto delta = at::empty({B, H, tq}, q.options().dtype(at::kFloat));
  at::Tensor kl;
  if (key_lengths.has_value() && key_lengths->defined()) kl = key_lengths->to(at::kInt).contiguous();
  check(kimi::flash_attn_bwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(),
                             lse.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr(), dv.data_ptr(),
                             delta.data_ptr<float>(), B, tq, tk, H, q.size(3), v.size(3), causal,
                             kl.defined() ? kl.data_ptr<int>() : nullptr, (float)scale, stream()), "flash_attn_bwd");
  return {dq, dk, dv};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "kimi_k3_b200 sm_100a kernels";
  m.def("rms_norm_fwd", &rms_norm_fwd);
  m.def("rms_norm_bwd", &rms_norm_bwd);
  m.def("situ_fwd", &situ_fwd);
  m.def("situ_bwd", &situ_bwd);
  m.def("sigmul_fwd", &sigmul_fwd);
  m.def("sigmul_bwd", &sigmul_bwd);
  m.def("decay_fwd", &decay_fwd);
  m.def("decay_bwd", &decay_bwd);
  m.def("conv_fwd", &conv_fwd);
  m.def("conv_bwd", &conv_bwd);
  m.def("attnres_fwd", &attnres_fwd);
  m.def("attnres_bwd", &attnres_bwd);
  m.def("ce_rows", &ce_rows);
  m.def("router", &router);
  m.def("kda_fwd", &kda_fwd);
  m.def("kda_bwd", &kda_bwd);
  m.def("fa_fwd", &fa_fwd);
  m.def("fa_bwd", &fa_bwd);
}
