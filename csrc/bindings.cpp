// PyTorch bindings for the kimi_k3_b200 sm_100a kernels. Each binding validates shapes,
// dtypes and contiguity, allocates outputs with the caching allocator and launches on the
// current CUDA stream. Launch errors raise immediately.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <vector>

#include <cstdio>
#include <stdexcept>
#include <string>
#include <execinfo.h>
#include <signal.h>
#include <unistd.h>

#include "kernels.h"
#include "tc_gemm.h"
#include "moe_route.h"

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

// Failures are reported with plain std::string concatenation (no stream formatting) and also
// written to stderr before the exception unwinds.
[[noreturn]] void fail(const std::string& msg) {
  fprintf(stderr, "kimi_k3_b200: %s\n", msg.c_str());
  fflush(stderr);
  throw std::runtime_error(msg);
}

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(std::string(what) + " failed: " + cudaGetErrorString(e));
}

// Kernels read and write with 16-byte vector accesses and bulk copies: every tensor they take is
// contiguous and starts on a 16-byte boundary (a misaligned view fails here, loudly).
#define CHECK_CUDA_CONTIG(x)                                                                           \
  TORCH_CHECK((x).is_cuda() && (x).is_contiguous() && (reinterpret_cast<uintptr_t>((x).data_ptr()) & 15) == 0, \
              #x " must be a contiguous CUDA tensor starting on a 16-byte boundary")

// A contiguous copy-if-needed of `t` that starts on a 16-byte boundary.
at::Tensor dense(const at::Tensor& t) {
  at::Tensor c = t.contiguous();
  if (reinterpret_cast<uintptr_t>(c.data_ptr()) & 15) c = c.clone(at::MemoryFormat::Contiguous);
  return c;
}

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
    wf = dense(w.to(at::kFloat));
    wp = wf.data_ptr<float>();
  }
  check(kimi::rms_norm_fwd(dtype_code(x), x.data_ptr(), wp, y.data_ptr(), rstd.data_ptr<float>(), rows, dim,
                           (int)period, (float)eps, stream()), "rms_norm_fwd");
  return {y, rstd};
}

std::vector<at::Tensor> rms_norm_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, at::Tensor rstd, int64_t period,
                                     bool need_dw) {
  CHECK_CUDA_CONTIG(x);
  dy = dense(dy);
  const at::cuda::CUDAGuard g(x.device());
  const int dim = x.size(-1);
  const int64_t rows = x.numel() / dim;
  auto dx = at::empty_like(x);
  at::Tensor wf, dw;
  const float* wp = nullptr;
  float* dwp = nullptr;
  if (w.defined() && w.numel()) {
    wf = dense(w.to(at::kFloat));
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
  dy = dense(dy);
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
  dy = dense(dy);
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
  auto af = dense(a_log.to(at::kFloat));
  check(kimi::kda_decay_fwd(dtype_code(z), z.data_ptr(), af.data_ptr<float>(), g.data_ptr<float>(), rows, heads, kdim,
                            (float)g_min, (float)ceps, stream()), "kda_decay_fwd");
  return g;
}

std::vector<at::Tensor> decay_bwd(at::Tensor dg, at::Tensor z, at::Tensor a_log, double g_min, double ceps) {
  dg = dense(dg.to(at::kFloat));
  const at::cuda::CUDAGuard gd(z.device());
  const int heads = z.size(-2), kdim = z.size(-1);
  const int64_t rows = z.numel() / (heads * kdim);
  auto dz = at::empty_like(z);
  auto af = dense(a_log.to(at::kFloat));
  auto da = at::zeros({heads}, z.options().dtype(at::kFloat));
  check(kimi::kda_decay_bwd(dtype_code(z), dg.data_ptr<float>(), z.data_ptr(), af.data_ptr<float>(), dz.data_ptr(),
                            da.data_ptr<float>(), rows, heads, kdim, (float)g_min, (float)ceps, stream()),
        "kda_decay_bwd");
  return {dz, da};
}

at::Tensor conv_fwd(at::Tensor x, at::Tensor w, int64_t head_dim, double eps, bool normalize) {
  x = dense(x);
  CHECK_CUDA_CONTIG(x);
  const at::cuda::CUDAGuard gd(x.device());
  auto wf = dense(w.to(at::kFloat));
  auto y = at::empty_like(x);
  check(kimi::conv_silu_norm_fwd(dtype_code(x), x.data_ptr(), wf.data_ptr<float>(), y.data_ptr(), x.size(0),
                                 x.size(1), x.size(2), wf.size(1), (int)head_dim, (float)eps, normalize, stream()),
        "conv_silu_norm_fwd");
  return y;
}

std::vector<at::Tensor> conv_bwd(at::Tensor dy, at::Tensor x, at::Tensor w, int64_t head_dim, double eps,
                                 bool normalize) {
  dy = dense(dy);
  x = dense(x);  // the forward's input as autograd saved it: possibly a misaligned view
  const at::cuda::CUDAGuard gd(x.device());
  auto wf = dense(w.to(at::kFloat));
  auto dx = at::empty_like(x);
  auto dw = at::empty(wf.sizes(), wf.options());
  auto part = at::empty({kimi::conv_bwd_partial_rows(x.size(0), x.size(1)), wf.numel()}, wf.options());
  check(kimi::conv_silu_norm_bwd(dtype_code(x), dy.data_ptr(), x.data_ptr(), wf.data_ptr<float>(),
                                 dx.data_ptr(), dw.data_ptr<float>(), part.data_ptr<float>(), x.size(0), x.size(1),
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
  auto qf = dense(q.to(at::kFloat)), wf = dense(w.to(at::kFloat));
  check(kimi::attnres_mix_fwd(dtype_code(s0), ptrs.data(), S, qf.data_ptr<float>(), wf.data_ptr<float>(),
                              out.data_ptr(), probs.data_ptr<float>(), rstd.data_ptr<float>(), tokens, dim,
                              (float)eps, stream()), "attnres_mix_fwd");
  return {out, probs, rstd};
}

std::vector<at::Tensor> attnres_bwd(std::vector<at::Tensor> sources, at::Tensor q, at::Tensor w, at::Tensor dout,
                                    at::Tensor probs, at::Tensor rstd) {
  const auto& s0 = sources.at(0);
  const at::cuda::CUDAGuard gd(s0.device());
  dout = dense(dout);
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
  auto qf = dense(q.to(at::kFloat)), wf = dense(w.to(at::kFloat));
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
  auto t = dense(targets.to(at::kLong));
  auto v = dense(valid.to(at::kBool));
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
  auto bf = dense(bias.to(at::kFloat));
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
  auto Araw = at::empty_like(W);
  auto o = at::empty_like(v);
  at::Tensor ht = want_final ? at::empty({B, H, 64, 64}, f) : at::Tensor();
  at::Tensor h0c;
  if (h0.has_value() && h0->defined()) h0c = dense(h0->to(at::kFloat));
  kimi::KdaBuffers buf{W.data_ptr<float>(), U.data_ptr<float>(), P.data_ptr<float>(), Qg.data_ptr<float>(),
                       Kend.data_ptr<float>(), eGC.data_ptr<float>(), states.data_ptr<float>(), Vp.data_ptr<float>(),
                       Araw.data_ptr<float>()};
  check(kimi::kda_chunk_fwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(),
                            beta.data_ptr<float>(), h0c.defined() ? h0c.data_ptr<float>() : nullptr, o.data_ptr(),
                            want_final ? ht.data_ptr<float>() : nullptr, buf, B, Tp, H, stream()), "kda_chunk_fwd");
  return {o, ht, W, U, P, Qg, Kend, eGC, states, Vp, Araw};
}

std::vector<at::Tensor> kda_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                                std::vector<at::Tensor> saved, at::Tensor dout, c10::optional<at::Tensor> dht,
                                bool want_dh0) {
  const at::cuda::CUDAGuard gd(q.device());
  dout = dense(dout);
  const int B = q.size(0), Tp = q.size(1), H = q.size(2);
  auto f = q.options().dtype(at::kFloat);
  auto& W = saved.at(0);
  kimi::KdaBuffers buf{saved[0].data_ptr<float>(), saved[1].data_ptr<float>(), saved[2].data_ptr<float>(),
                       saved[3].data_ptr<float>(), saved[4].data_ptr<float>(), saved[5].data_ptr<float>(),
                       saved[6].data_ptr<float>(), saved[7].data_ptr<float>(), saved.at(8).data_ptr<float>()};
  auto dVp = at::empty_like(W), dSn = at::empty_like(W);
  auto dq = at::empty(q.sizes(), f), dk = at::empty(k.sizes(), f), dv = at::empty(v.sizes(), f),
       dg = at::empty(g.sizes(), f), dbeta = at::empty(beta.sizes(), f);
  at::Tensor dh0 = want_dh0 ? at::empty({B, H, 64, 64}, f) : at::Tensor();
  at::Tensor dhtc;
  if (dht.has_value() && dht->defined()) dhtc = dense(dht->to(at::kFloat));
  check(kimi::kda_chunk_bwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(),
                            beta.data_ptr<float>(), buf, dout.data_ptr(),
                            dhtc.defined() ? dhtc.data_ptr<float>() : nullptr, dVp.data_ptr<float>(),
                            dSn.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr<float>(), dv.data_ptr<float>(),
                            dg.data_ptr<float>(), dbeta.data_ptr<float>(),
                            want_dh0 ? dh0.data_ptr<float>() : nullptr, B, Tp, H, nullptr, stream()),
        "kda_chunk_bwd");
  return {dq, dk, dv, dg, dbeta, dh0};
}

// ---------------------------------------------------------------- bf16 weight mirrors
// One launch: dst[t] = bf16(src[t]) for every tensor of a table.  `tables` is an int64 CUDA tensor
// [4, T + 1]: rows 0-2 hold the source pointers, destination pointers and element counts (entry T
// unused), row 3 the prefix sums of ceil(numel / 8); `total_vec` = tables[3][T].
void cast_bf16_multi(at::Tensor tables, int64_t tensors, int64_t total_vec) {
  TORCH_CHECK(tables.is_cuda() && tables.scalar_type() == at::kLong && tables.is_contiguous() && tables.dim() == 2 &&
                  tables.size(0) == 4 && tables.size(1) == tensors + 1,
              "tables must be a contiguous int64 CUDA tensor [4, tensors + 1]");
  const at::cuda::CUDAGuard gd(tables.device());
  const int64_t* t = tables.data_ptr<int64_t>();
  const int64_t w = tensors + 1;
  check(kimi::cast_bf16_multi(reinterpret_cast<const float* const*>(t), reinterpret_cast<void* const*>(t + w), t + 2 * w,
                              t + 3 * w, (int)tensors, total_vec, stream()),
        "cast_bf16_multi");
}

// Newton-Schulz polynomial P = c * G2 + b * G + a * I of stacked [m, m] Gram matrices (bf16 [rows, m]).
at::Tensor ns_poly(at::Tensor g, at::Tensor g2, double a, double b, double c) {
  TORCH_CHECK(g.is_cuda() && g.scalar_type() == at::kBFloat16 && g.dim() == 2 && g.is_contiguous() &&
                  g2.sizes() == g.sizes() && g2.scalar_type() == at::kBFloat16 && g2.is_contiguous(),
              "ns_poly: contiguous bf16 [rows, m] Gram matrices");
  const at::cuda::CUDAGuard gd(g.device());
  at::Tensor out = at::empty_like(g);
  check(kimi::ns_poly(g.data_ptr(), g2.data_ptr(), out.data_ptr(), g.size(0), (int)g.size(1), (float)a, (float)b,
                      (float)c, stream()),
        "ns_poly");
  return out;
}

// ---------------------------------------------------------------- fused Muon passes
void muon_momentum(at::Tensor g, at::Tensor mom, at::Tensor x, at::Tensor sumsq, double momentum, bool nesterov,
                   c10::optional<at::Tensor> skip) {
  CHECK_CUDA_CONTIG(g);
  CHECK_CUDA_CONTIG(mom);
  CHECK_CUDA_CONTIG(x);
  CHECK_CUDA_CONTIG(sumsq);
  TORCH_CHECK(g.scalar_type() == at::kFloat && mom.scalar_type() == at::kFloat && x.scalar_type() == at::kBFloat16 &&
                  sumsq.scalar_type() == at::kFloat && g.dim() == 3 && g.sizes() == mom.sizes() &&
                  g.sizes() == x.sizes() && sumsq.numel() == g.size(0),
              "muon_momentum: g, mom fp32 [count, m, n], x bf16 of the same shape, sumsq fp32 [count]");
  const at::cuda::CUDAGuard gd(g.device());
  const bool* sk = (skip.has_value() && skip->defined()) ? skip->data_ptr<bool>() : nullptr;
  check(kimi::muon_momentum(g.data_ptr<float>(), mom.data_ptr<float>(), x.data_ptr(), sumsq.data_ptr<float>(),
                            (int)g.size(0), g.size(1) * g.size(2), (float)momentum, nesterov, sk, stream()),
        "muon_momentum");
}

void muon_normalize(at::Tensor x, at::Tensor sumsq, double eps) {
  CHECK_CUDA_CONTIG(x);
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x.dim() == 3 && sumsq.numel() == x.size(0), "muon_normalize");
  const at::cuda::CUDAGuard gd(x.device());
  check(kimi::muon_normalize(x.data_ptr(), sumsq.data_ptr<float>(), (int)x.size(0), x.size(1) * x.size(2),
                             (float)eps, stream()),
        "muon_normalize");
}

void muon_apply(at::Tensor o, at::Tensor param_ptrs, at::Tensor sumsq, at::Tensor lr, double wd, double scale,
                double eps, c10::optional<at::Tensor> skip, at::Tensor stats) {
  CHECK_CUDA_CONTIG(o);
  TORCH_CHECK(o.scalar_type() == at::kBFloat16 && o.dim() == 3 && param_ptrs.scalar_type() == at::kLong &&
                  param_ptrs.is_cuda() && param_ptrs.numel() == o.size(0) && sumsq.numel() == o.size(0) &&
                  lr.is_cuda() && lr.scalar_type() == at::kFloat && stats.numel() == 3 * o.size(0) &&
                  stats.scalar_type() == at::kFloat,
              "muon_apply: o bf16 [count, m, n], one fp32 parameter pointer per matrix, device lr, stats [count, 3]");
  const at::cuda::CUDAGuard gd(o.device());
  const bool* sk = (skip.has_value() && skip->defined()) ? skip->data_ptr<bool>() : nullptr;
  check(kimi::muon_apply(o.data_ptr(), reinterpret_cast<float* const*>(param_ptrs.data_ptr<int64_t>()),
                         sumsq.data_ptr<float>(), (int)o.size(0), o.size(1) * o.size(2), lr.data_ptr<float>(),
                         (float)wd, (float)scale, (float)eps, sk, stats.data_ptr<float>(), stream()),
        "muon_apply");
}

// ---------------------------------------------------------------- tcgen05 small-matrix self-test
std::vector<at::Tensor> tcs_selftest(at::Tensor a, at::Tensor b, int64_t n, int64_t mode) {
  CHECK_CUDA_CONTIG(a);
  CHECK_CUDA_CONTIG(b);
  TORCH_CHECK(a.scalar_type() == at::kFloat && b.scalar_type() == at::kFloat, "fp32 operands");
  const at::cuda::CUDAGuard gd(a.device());
  const int K = a.size(1);
  const int ncols = mode == 0 ? n : (mode == 1 ? 256 : 64);
  auto out = at::empty({128, ncols}, a.options());
  auto status = at::zeros({1}, a.options().dtype(at::kInt));
  check(kimi::tcs_selftest(a.data_ptr<float>(), b.data_ptr<float>(), out.data_ptr<float>(), K, (int)n, (int)mode,
                           status.data_ptr<int>(), stream()), "tcs_selftest");
  return {out, status};
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
  if (key_lengths.has_value() && key_lengths->defined()) kl = dense(key_lengths->to(at::kInt));
  check(kimi::flash_attn_fwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(),
                             lse.data_ptr<float>(), B, tq, tk, H, q.size(3), v.size(3), causal,
                             kl.defined() ? kl.data_ptr<int>() : nullptr, (float)scale, stream()), "flash_attn_fwd");
  return {o, lse};
}

std::vector<at::Tensor> fa_bwd(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor o, at::Tensor dout, at::Tensor lse,
                               bool causal, c10::optional<at::Tensor> key_lengths, double scale) {
  const at::cuda::CUDAGuard gd(q.device());
  dout = dense(dout);
  const int B = q.size(0), tq = q.size(1), H = q.size(2), tk = k.size(1);
  auto dq = at::zeros(q.sizes(), q.options().dtype(at::kFloat));
  auto dk = at::empty_like(k), dv = at::empty_like(v);
  auto delta = at::empty({B, H, tq}, q.options().dtype(at::kFloat));
  at::Tensor kl;
  if (key_lengths.has_value() && key_lengths->defined()) kl = dense(key_lengths->to(at::kInt));
  check(kimi::flash_attn_bwd(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dout.data_ptr(),
                             lse.data_ptr<float>(), dq.data_ptr<float>(), dk.data_ptr(), dv.data_ptr(),
                             delta.data_ptr<float>(), B, tq, tk, H, q.size(3), v.size(3), causal,
                             kl.defined() ? kl.data_ptr<int>() : nullptr, (float)scale, stream()), "flash_attn_bwd");
  return {dq, dk, dv};
}


// ---------------------------------------------------------------- tcgen05 GEMM
// Logical C[M,N] = A[M,K] B[N,K]^T. a_mn: A given as [K, M]; b_mn: B given as [K, N] (or [G,K,N]).
static void check_tma_matrix(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.dim() == 2 && t.stride(1) == 1 && t.stride(0) % 8 == 0 && t.stride(0) >= t.size(1),
              name, " must be a row-major CUDA matrix with a 16-byte aligned row stride");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0, name, " must start on a 16-byte boundary");
  TORCH_CHECK(t.scalar_type() == at::kBFloat16, name, ": tc_gemm takes bf16 operands");
}

// Dense GEMM out[M,N] = op(a) op(b)^T on the tcgen05 kernel. Operands may be row-strided views
// (any M, N, K; row strides multiples of 8 elements): tiles past the logical edge read zeros.
// `status` (int32 CUDA tensor) receives the code of the first bounded wait that gave up; without it
// the device's default status word does (tc_gemm_status).  `spin_limit` > 0 shortens every
// pipeline wait to that many polls (tests use it to make a wait run out on purpose).
// `accumulate` adds the product into `out` (fp32, given) with vector atomics instead of storing it;
// `ksplit` > 1 splits the K range over that many work units (needs `accumulate`).  `bias` (fp32 [N])
// and `residual` (bf16 [M, N], row-major) are added in the store epilogue.  `pair`: 1 / 0 force or
// forbid CTA-pair (cta_group::2) tiles, -1 uses them whenever M > 128.
at::Tensor tc_gemm_dense(at::Tensor a, at::Tensor b, bool a_mn, bool b_mn, bool out_fp32, int64_t bn,
                         c10::optional<at::Tensor> out_opt, c10::optional<at::Tensor> status_opt,
                         int64_t spin_limit, bool accumulate, int64_t ksplit, c10::optional<at::Tensor> bias,
                         c10::optional<at::Tensor> residual, int64_t pair, int64_t debug,
                         c10::optional<at::Tensor> dbg) {
  check_tma_matrix(a, "a");
  check_tma_matrix(b, "b");
  const at::cuda::CUDAGuard gd(a.device());
  const int64_t M = a_mn ? a.size(1) : a.size(0), K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "inner dimensions differ");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "empty GEMM");
  // A fresh output gets a row stride padded to 8 elements (16 bytes); the result is a view.
  at::Tensor out = out_opt.has_value() && out_opt->defined()
                       ? *out_opt
                       : at::empty({M, (N + 7) / 8 * 8}, a.options().dtype(out_fp32 ? at::kFloat : at::kBFloat16))
                             .narrow(1, 0, N);
  TORCH_CHECK(out.is_cuda() && out.dim() == 2 && out.size(0) == M && out.size(1) == N && out.stride(1) == 1 &&
                  out.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0,
              "out must be an [M,N] row-major matrix with a 16-byte aligned row stride");
  TORCH_CHECK(!accumulate || (out_opt.has_value() && out_opt->defined() && out.scalar_type() == at::kFloat),
              "accumulate needs a given fp32 out");
  TORCH_CHECK(ksplit <= 1 || accumulate, "ksplit > 1 needs accumulate");
  kimi::TcGemmArgs g;
  g.epi = accumulate ? 3 : 0;
  g.ksplit = (int)std::max<int64_t>(1, ksplit);
  g.pair = (int)pair;
  g.debug = (int)debug;
  if (dbg.has_value() && dbg->defined()) {
    TORCH_CHECK(dbg->is_cuda() && dbg->scalar_type() == at::kLong && dbg->numel() >= 16, "dbg: int64 CUDA [16]");
    g.dbg = reinterpret_cast<unsigned long long*>(dbg->data_ptr<int64_t>());
  }
  at::Tensor bias_c, res_c;
  if (bias.has_value() && bias->defined()) {
    bias_c = bias->to(at::kFloat).contiguous();
    TORCH_CHECK(bias_c.is_cuda() && bias_c.numel() == N, "bias must hold N values");
    g.bias = bias_c.data_ptr<float>();
  }
  if (residual.has_value() && residual->defined()) {
    res_c = *residual;
    TORCH_CHECK(res_c.is_cuda() && res_c.scalar_type() == at::kBFloat16 && res_c.dim() == 2 && res_c.size(0) == M &&
                    res_c.size(1) == N && res_c.stride(1) == 1 && res_c.stride(0) % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(res_c.data_ptr()) & 15) == 0,
                "residual must be a bf16 [M, N] row-major matrix with a 16-byte aligned row stride");
    TORCH_CHECK(out.scalar_type() == at::kBFloat16, "a residual needs a bf16 output");
    g.resid = res_c.data_ptr();
    g.ldr = res_c.stride(0);
  }
  g.mode = 0;
  g.bn = (int)bn;
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.a = a.data_ptr();
  g.a_rows = a.size(0);
  g.a_cols = a.size(1);
  g.a_ld = a.stride(0);
  g.b = b.data_ptr();
  g.b_groups = 1;
  g.b_rows = b.size(0);
  g.b_cols = b.size(1);
  g.b_ld = b.stride(0);
  g.b_gstride = b.stride(0) * b.size(0);
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.out = out.data_ptr();
  g.out_fp32 = out.scalar_type() == at::kFloat;
  g.ldc = out.stride(0);
  if (status_opt.has_value() && status_opt->defined()) {
    TORCH_CHECK(status_opt->is_cuda() && status_opt->scalar_type() == at::kInt, "status must be an int32 CUDA tensor");
    g.status = status_opt->data_ptr<int>();
  }
  g.spin_limit = (uint32_t)std::max<int64_t>(0, std::min<int64_t>(spin_limit, 0x7fffffff));
  int dev = a.get_device();
  g.num_sms = at::cuda::getDeviceProperties(dev)->multiProcessorCount;
  check(kimi::tc_gemm(g, stream()), "tc_gemm_dense");
  return out;
}

// Fused projection group: several weights that read one input, as one GEMM over their concatenated
// bf16 weight W_cat [N_total, K] (rows of consecutive segments).
//   kind 1 (forward):      segs[s] (bf16 [M, N_s] outputs) <- x [M, K] W_cat^T
//   kind 2 (input grad):   out [M, K] = sum_s segs[s] ([M, N_s] output grads) W_cat[rows of s]
//   kind 3 (weight grads): out [N_total, K] fp32 += concat_s(segs[s])^T x   (split over `ksplit` K slices)
// Segment widths must be multiples of 32 (kind 1) or 64 (kinds 2, 3) except the last; rows of every
// tensor start on 16-byte boundaries.  Kind 1 stores whole 16-byte units: a segment whose width is
// not a multiple of 8 also gets its columns [width, round_up(width, 8)) written (zeros), so its row
// stride must leave room for them (such an output is a view into a row-padded buffer).
void tc_gemm_group(int64_t kind, std::vector<at::Tensor> segs, at::Tensor x, at::Tensor w,
                   c10::optional<at::Tensor> out_opt, int64_t bn, int64_t ksplit, int64_t pair) {
  TORCH_CHECK(kind >= 1 && kind <= 3, "kind must be 1, 2 or 3");
  TORCH_CHECK(!segs.empty() && segs.size() <= 8, "1 to 8 segments");
  const at::cuda::CUDAGuard gd(x.device());
  kimi::TcGemmArgs g;
  g.mode = 0;
  g.bn = (int)bn;
  g.pair = (int)pair;
  g.seg_kind = (int)kind;
  g.nseg = (int)segs.size();
  int64_t total = 0;
  for (size_t s = 0; s < segs.size(); ++s) {
    check_tma_matrix(segs[s], "segment");
    g.seg_ptr[s] = segs[s].data_ptr();
    g.seg_width[s] = segs[s].size(1);
    g.seg_ld[s] = segs[s].stride(0);
    total += segs[s].size(1);
  }
  if (kind == 1) {  // A = x [M, K] K-major, B = W_cat [N, K] K-major
    for (auto& t : segs)
      TORCH_CHECK(t.stride(0) >= (t.size(1) + 7) / 8 * 8,
                  "a kind-1 segment's row stride must cover its width rounded up to 8 columns");
    check_tma_matrix(x, "x");
    check_tma_matrix(w, "w");
    TORCH_CHECK(w.size(0) == total && w.size(1) == x.size(1), "W_cat must be [sum of widths, K]");
    for (auto& t : segs) TORCH_CHECK(t.size(0) == x.size(0), "outputs must have the rows of x");
    g.a = x.data_ptr();
    g.a_rows = x.size(0);
    g.a_cols = x.size(1);
    g.a_ld = x.stride(0);
    g.b = w.data_ptr();
    g.b_rows = w.size(0);
    g.b_cols = w.size(1);
    g.b_ld = w.stride(0);
    g.b_gstride = w.stride(0) * w.size(0);
    g.M = (int)x.size(0);
    g.N = (int)total;
    g.K = (int)x.size(1);
  } else if (kind == 2) {  // A = segments (K-major), B = W_cat given MN-major [N_total (k), K_in (n)]
    TORCH_CHECK(out_opt.has_value() && out_opt->defined(), "kind 2 needs out [M, K_in]");
    check_tma_matrix(w, "w");
    const at::Tensor& out = *out_opt;
    const int64_t M = segs[0].size(0);
    for (auto& t : segs) TORCH_CHECK(t.size(0) == M, "segments must share their rows");
    TORCH_CHECK(out.is_cuda() && out.dim() == 2 && out.size(0) == M && out.size(1) == w.size(1) && out.stride(1) == 1,
                "out must be [M, K_in]");
    TORCH_CHECK(total >= w.size(0), "segments must cover every row of W_cat");
    g.a = segs[0].data_ptr();
    g.a_rows = M;
    g.a_cols = segs[0].size(1);
    g.a_ld = segs[0].stride(0);
    g.b_mn = true;
    g.b = w.data_ptr();
    g.b_rows = w.size(0);
    g.b_cols = w.size(1);
    g.b_ld = w.stride(0);
    g.b_gstride = w.stride(0) * w.size(0);
    g.M = (int)M;
    g.N = (int)w.size(1);
    g.K = (int)total;
    g.out = out.data_ptr();
    g.out_fp32 = out.scalar_type() == at::kFloat;
    g.ldc = out.stride(0);
  } else {  // A = segments given MN-major [tokens, N_s], B = x given MN-major [tokens, K_in]
    TORCH_CHECK(out_opt.has_value() && out_opt->defined(), "kind 3 needs an fp32 out [N_total, K_in]");
    check_tma_matrix(x, "x");
    const at::Tensor& out = *out_opt;
    const int64_t T = x.size(0);
    for (auto& t : segs) TORCH_CHECK(t.size(0) == T, "segments must share the token rows of x");
    TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.dim() == 2 && out.size(1) == x.size(1) &&
                    out.stride(1) == 1 && out.stride(0) % 4 == 0 && out.size(0) <= total,
                "out must be an fp32 [N_total, K_in] matrix");
    g.a_mn = true;
    g.a = segs[0].data_ptr();
    g.a_rows = T;
    g.a_cols = segs[0].size(1);
    g.a_ld = segs[0].stride(0);
    g.b_mn = true;
    g.b = x.data_ptr();
    g.b_rows = T;
    g.b_cols = x.size(1);
    g.b_ld = x.stride(0);
    g.b_gstride = x.stride(0) * T;
    g.M = (int)out.size(0);
    g.N = (int)x.size(1);
    g.K = (int)T;
    g.out = out.data_ptr();
    g.out_fp32 = true;
    g.ldc = out.stride(0);
    g.epi = 3;
    g.ksplit = (int)std::max<int64_t>(1, ksplit);
  }
  g.num_sms = at::cuda::getDeviceProperties(x.get_device())->multiProcessorCount;
  check(kimi::tc_gemm(g, stream()), "tc_gemm_group");
}

// Fused GEMM + cross-rank reduction (tensor parallelism): every rank computes its partial
// a @ op(b)^T into `part` (its [M, N] slice of a symmetric buffer) and the comm warps of the same
// kernel reduce it over the group (mode 1 all-reduce into out [M, N]; mode 2 reduce-scatter into
// out [M / world, N]).  part_peers / flag_peers are the device addresses of every rank's partial
// buffer and flag words; part_mc is the multicast address of the partial buffer or 0.
at::Tensor tc_gemm_comm(at::Tensor a, at::Tensor b, bool b_mn, int64_t bn, int64_t mode, int64_t rank, int64_t world,
                        at::Tensor part, std::vector<int64_t> part_peers, int64_t part_mc,
                        std::vector<int64_t> flag_peers, int64_t tiles_cap, at::Tensor out, at::Tensor status,
                        int64_t timeout_ns) {
  check_tma_matrix(a, "a");
  check_tma_matrix(b, "b");
  const at::cuda::CUDAGuard gd(a.device());
  const int64_t M = a.size(0), K = a.size(1), N = b_mn ? b.size(1) : b.size(0);
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == K, "inner dimensions differ");
  TORCH_CHECK(N % 8 == 0, "the reduced width must be a multiple of 8");
  TORCH_CHECK(part.is_cuda() && part.scalar_type() == at::kBFloat16 && part.is_contiguous() && part.size(0) == M &&
                  part.size(1) == N,
              "part must be this rank's contiguous bf16 [M, N] symmetric buffer slice");
  TORCH_CHECK(world >= 1 && world <= 8 && (int64_t)part_peers.size() == world && (int64_t)flag_peers.size() == world,
              "one partial and one flag address per rank (world <= 8)");
  TORCH_CHECK(part_peers[rank] == (int64_t)reinterpret_cast<uintptr_t>(part.data_ptr()),
              "part must be this rank's entry of part_peers");
  const int64_t out_rows = mode == 2 ? M / world : M;
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.size(0) == out_rows &&
                  out.size(1) == N && out.stride(1) == 1 && out.stride(0) % 8 == 0,
              "out has the wrong shape or layout");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "status must be an int32 CUDA tensor");
  kimi::TcGemmArgs g;
  g.mode = 0;
  g.bn = (int)bn;
  g.b_mn = b_mn;
  g.a = a.data_ptr();
  g.a_rows = M;
  g.a_cols = K;
  g.a_ld = a.stride(0);
  g.b = b.data_ptr();
  g.b_groups = 1;
  g.b_rows = b.size(0);
  g.b_cols = b.size(1);
  g.b_ld = b.stride(0);
  g.b_gstride = b.stride(0) * b.size(0);
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.out = part.data_ptr();
  g.ldc = N;
  g.status = status.data_ptr<int>();
  g.comm_mode = (int)mode;
  g.comm_rank = (int)rank;
  g.comm_world = (int)world;
  g.comm_rows_per_rank = (int)(M / world);
  for (int64_t q = 0; q < world; ++q) {
    g.part_peer[q] = (uint64_t)part_peers[q];
    g.flags_peer[q] = (uint64_t)flag_peers[q];
  }
  g.part_mc = (uint64_t)part_mc;
  g.tiles_cap = (int)tiles_cap;
  g.comm_out = out.data_ptr();
  g.comm_ldo = out.stride(0);
  g.timeout_ns = timeout_ns;
  g.num_sms = at::cuda::getDeviceProperties(a.get_device())->multiProcessorCount;
  check(kimi::tc_gemm(g, stream()), "tc_gemm_comm");
  return out;
}

// Grouped GEMM. mode 1: rows of `a` ([R, K] K-major) split by offsets (128-aligned); b is [G, N, K]
// (b_mn=False) or [G, K, N] (b_mn=True); epi 0 store / 1 SiTU (b2 = up weights) / 2 scatter-add.
// mode 2: reduction over row segments (64-aligned) of a ([R, M] MN-major) and b ([R, N] MN-major);
// out is [G, M, N].
std::vector<at::Tensor> tc_gemm_grouped(int64_t mode, at::Tensor a, at::Tensor b, c10::optional<at::Tensor> b2,
                                        bool a_mn, bool b_mn, at::Tensor offsets, int64_t M, int64_t N, int64_t K,
                                        int64_t epi, c10::optional<at::Tensor> out_opt, bool out_fp32, double bg,
                                        double bu, c10::optional<at::Tensor> row_token,
                                        c10::optional<at::Tensor> row_weight, int64_t b2_k_split, int64_t bn,
                                        int64_t uniform_rows) {
  TORCH_CHECK(a.is_cuda() && a.dim() == 2 && a.stride(1) == 1 && a.stride(0) % 8 == 0,
              "a must be a row-major CUDA matrix with a 16-byte aligned row stride");
  CHECK_CUDA_CONTIG(b);
  const at::cuda::CUDAGuard gd(a.device());
  TORCH_CHECK(offsets.scalar_type() == at::kInt && offsets.is_cuda(), "offsets must be int32 on device");
  const int G = (int)offsets.numel() - 1;
  kimi::TcGemmArgs g;
  g.mode = (int)mode;
  g.bn = (int)bn;
  g.a_mn = a_mn;
  g.b_mn = b_mn;
  g.a = a.data_ptr();
  g.a_rows = a.size(0);
  g.a_cols = a.size(1);
  g.a_ld = a.stride(0);
  g.b = b.data_ptr();
  at::Tensor b2t;
  if (b2.has_value() && b2->defined()) {
    b2t = dense(*b2);
    g.b2 = b2t.data_ptr();
  }
  if (b.dim() == 3) {
    g.b_groups = b.size(0);
    g.b_rows = b.size(1);
    g.b_cols = b.size(2);
    g.b_ld = b.size(2);
    g.b_gstride = b.size(1) * b.size(2);
  } else {
    g.b_groups = 1;
    g.b_rows = b.size(0);
    g.b_cols = b.size(1);
    g.b_ld = b.size(1);
    g.b_gstride = b.numel();
  }
  g.b2_k_split = (int)b2_k_split;
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.G = G;
  g.offsets = offsets.data_ptr<int>();
  TORCH_CHECK(uniform_rows == 0 || (mode == 1 && uniform_rows % 128 == 0 && uniform_rows * G == a.size(0)),
              "uniform_rows: mode 1 segments of a multiple of 128 rows covering a");
  g.uniform_rows = (int)uniform_rows;
  g.epi = (int)epi;
  g.bg = (float)bg;
  g.bu = (float)bu;
  std::vector<at::Tensor> outs;
  at::Tensor out;
  if (out_opt.has_value() && out_opt->defined()) {
    out = *out_opt;
  } else if (mode == 2) {
    out = at::empty({G, M, N}, a.options().dtype(out_fp32 ? at::kFloat : at::kBFloat16));
  } else {
    out = at::empty({a.size(0), N}, a.options().dtype(out_fp32 ? at::kFloat : at::kBFloat16));
  }
  g.out = out.data_ptr();
  g.out_fp32 = out.scalar_type() == at::kFloat;
  g.ldc = out.size(-1);
  outs.push_back(out);
  at::Tensor og, ou;
  if (epi == 1) {
    og = at::empty({a.size(0), N}, a.options());
    ou = at::empty({a.size(0), N}, a.options());
    g.out_g = og.data_ptr();
    g.out_u = ou.data_ptr();
    outs.push_back(og);
    outs.push_back(ou);
  }
  at::Tensor rt, rw;
  if (epi == 2) {
    rt = dense(*row_token);
    rw = dense(row_weight->to(at::kFloat));
    g.row_token = rt.data_ptr<int>();
    g.row_weight = rw.data_ptr<float>();
    g.ldc = out.size(-1);
  }
  g.num_sms = at::cuda::getDeviceProperties(a.get_device())->multiProcessorCount;
  const cudaError_t err = kimi::tc_gemm(g, stream());
  if (err != cudaSuccess) {
    using std::to_string;
    fail(std::string("tc_gemm_grouped failed: ") + cudaGetErrorString(err) + " (mode " + to_string(mode) + ", epi " +
         to_string(epi) + ", bn " + to_string(bn) + ", M " + to_string(M) + ", N " + to_string(N) + ", K " +
         to_string(K) + ", G " + to_string(G) + ", a " + to_string(a.size(0)) + "x" + to_string(a.size(1)) +
         " ld " + to_string(a.stride(0)) + ", b dim " + to_string(b.dim()) + ", a_mn " + to_string(a_mn) +
         ", b_mn " + to_string(b_mn) + ")");
  }
  return outs;
}


// ---------------------------------------------------------------- MoE routing
std::vector<at::Tensor> moe_route(at::Tensor sel, at::Tensor w, int64_t E, int64_t r_max) {
  CHECK_CUDA_CONTIG(sel);
  const at::cuda::CUDAGuard gd(sel.device());
  auto i32 = sel.options().dtype(at::kInt);
  const int64_t M = sel.size(0), k = sel.size(1);
  auto wf = dense(w.to(at::kFloat));
  auto counts = at::empty({E}, i32), offsets = at::empty({E + 1}, i32), cursor = at::empty({E}, i32);
  auto row_token = at::empty({r_max}, i32), row_of = at::empty({M * k}, i32);
  auto row_weight = at::zeros({r_max}, sel.options().dtype(at::kFloat));
  check(kimi::moe_route_prep(sel.data_ptr<int64_t>(), wf.data_ptr<float>(), M, (int)k, (int)E, r_max,
                             counts.data_ptr<int>(), offsets.data_ptr<int>(), cursor.data_ptr<int>(),
                             row_token.data_ptr<int>(), row_weight.data_ptr<float>(), row_of.data_ptr<int>(),
                             stream()), "moe_route_prep");
  return {counts, offsets, row_token, row_weight, row_of};
}

at::Tensor moe_gather(at::Tensor latent, at::Tensor row_token) {
  CHECK_CUDA_CONTIG(latent);
  const at::cuda::CUDAGuard gd(latent.device());
  auto xs = at::empty({row_token.size(0), latent.size(1)}, latent.options());
  check(kimi::moe_gather(latent.data_ptr(), row_token.data_ptr<int>(), xs.data_ptr(), row_token.size(0),
                         latent.size(1), stream()), "moe_gather");
  return xs;
}

std::vector<at::Tensor> moe_dy(at::Tensor dagg, at::Tensor row_token, at::Tensor row_weight, at::Tensor y) {
  const at::cuda::CUDAGuard gd(y.device());
  dagg = dense(dagg.to(at::kFloat));
  auto dy = at::empty_like(y);
  auto dw_row = at::empty({y.size(0)}, y.options().dtype(at::kFloat));
  check(kimi::moe_dy(dagg.data_ptr<float>(), row_token.data_ptr<int>(), row_weight.data_ptr<float>(), y.data_ptr(),
                     dy.data_ptr(), dw_row.data_ptr<float>(), y.size(0), y.size(1), stream()), "moe_dy");
  return {dy, dw_row};
}

at::Tensor moe_slot_sum(at::Tensor dxs, at::Tensor row_of, int64_t M, int64_t k, bool out_fp32) {
  const at::cuda::CUDAGuard gd(dxs.device());
  auto out = at::empty({M, dxs.size(1)}, dxs.options().dtype(out_fp32 ? at::kFloat : at::kBFloat16));
  check(kimi::moe_slot_sum(dxs.data_ptr(), row_of.data_ptr<int>(), out.data_ptr(), out_fp32, M, (int)k,
                           dxs.size(1), stream()), "moe_slot_sum");
  return out;
}

at::Tensor situ_bwd_cat(at::Tensor dh, at::Tensor g, at::Tensor u, double bg, double bu) {
  const at::cuda::CUDAGuard gd(g.device());
  dh = dense(dh);
  auto dgu = at::empty({g.size(0), 2 * g.size(1)}, g.options());
  check(kimi::situ_bwd_cat(dh.data_ptr(), g.data_ptr(), u.data_ptr(), dgu.data_ptr(), g.size(0), g.size(1),
                           (float)bg, (float)bu, stream()), "situ_bwd_cat");
  return dgu;
}

// ---------------------------------------------------------------- decode step
std::vector<at::Tensor> conv_step(std::vector<at::Tensor> xs, std::vector<at::Tensor> hists,
                                  std::vector<at::Tensor> ws, std::vector<c10::optional<at::Tensor>> biases,
                                  std::vector<int64_t> head_dims, double eps) {
  const size_t n = xs.size();
  TORCH_CHECK(n >= 1 && n <= 3 && hists.size() == n && ws.size() == n && biases.size() == n && head_dims.size() == n,
              "conv_step takes one to three streams");
  const at::cuda::CUDAGuard gd(xs[0].device());
  kimi::ConvStepArgs a{};
  std::vector<at::Tensor> ys, keep;
  const int64_t batch = xs[0].size(0);
  const int64_t ksize = ws[0].size(1);
  for (size_t i = 0; i < n; ++i) {
    auto x = dense(xs[i]);
    CHECK_CUDA_CONTIG(hists[i]);
    TORCH_CHECK(x.scalar_type() == xs[0].scalar_type() && hists[i].scalar_type() == x.scalar_type(),
                "conv_step streams share one dtype");
    const int64_t c = x.size(-1);
    TORCH_CHECK(x.numel() == batch * c && hists[i].size(0) == batch && hists[i].size(1) == ksize - 1 &&
                    hists[i].size(2) == c && ws[i].size(0) == c && ws[i].size(1) == ksize,
                "conv_step shapes: x [B, C], history [B, K-1, C], weight [C, K]");
    auto w = dense(ws[i].to(at::kFloat));
    at::Tensor bias;
    if (biases[i].has_value() && biases[i]->defined()) bias = dense(biases[i]->to(at::kFloat));
    auto y = at::empty_like(x);
    a.x[i] = x.data_ptr();
    a.hist[i] = hists[i].data_ptr();
    a.w[i] = w.data_ptr<float>();
    a.bias[i] = bias.defined() ? bias.data_ptr<float>() : nullptr;
    a.y[i] = y.data_ptr();
    a.channels[i] = (int)c;
    a.head_lanes[i] = (int)(head_dims[i] / 8);
    TORCH_CHECK(head_dims[i] == 0 || (head_dims[i] % 8 == 0 && c % head_dims[i] == 0), "conv_step head_dim");
    keep.insert(keep.end(), {x, w, bias});
    ys.push_back(y);
  }
  check(kimi::conv_step(dtype_code(xs[0]), a, (int)n, (int)batch, (int)ksize, (float)eps, stream()), "conv_step");
  return ys;
}

std::vector<at::Tensor> kda_decode(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor g, at::Tensor beta,
                                   at::Tensor state, c10::optional<at::Tensor> state_out) {
  q = dense(q);
  k = dense(k);
  v = dense(v);
  g = dense(g.to(at::kFloat));
  beta = dense(beta.to(at::kFloat));
  CHECK_CUDA_CONTIG(state);
  TORCH_CHECK(state.scalar_type() == at::kFloat && state.dim() == 4 && state.size(2) == 64 && state.size(3) == 64,
              "kda_decode takes an fp32 state [B, H, 64, 64]");
  const int64_t b = state.size(0), h = state.size(1);
  TORCH_CHECK(q.numel() == b * h * 64 && k.numel() == b * h * 64 && v.numel() == b * h * 64 &&
                  g.numel() == b * h * 64 && beta.numel() == b * h,
              "kda_decode shapes: q/k/v/g [B, H, 64], beta [B, H]");
  const at::cuda::CUDAGuard gd(q.device());
  at::Tensor out_state = state_out.has_value() && state_out->defined() ? *state_out : at::empty_like(state);
  CHECK_CUDA_CONTIG(out_state);
  TORCH_CHECK(out_state.sizes() == state.sizes() && out_state.scalar_type() == at::kFloat, "state_out shape");
  auto o = at::empty({b, h, 64}, q.options());
  check(kimi::kda_decode(dtype_code(q), q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr<float>(),
                         beta.data_ptr<float>(), state.data_ptr<float>(), out_state.data_ptr<float>(), o.data_ptr(),
                         (int)b, (int)h, stream()),
        "kda_decode");
  return {o, out_state};
}

bool mla_decode_supported(int64_t heads, int64_t ldim) { return kimi::mla_decode_supported((int)heads, (int)ldim); }

at::Tensor mla_decode(at::Tensor qlat, at::Tensor latent, at::Tensor lengths) {
  qlat = dense(qlat.to(at::kFloat));
  CHECK_CUDA_CONTIG(latent);
  auto len = dense(lengths.to(at::kInt));
  TORCH_CHECK(latent.dim() == 3 && qlat.dim() == 3 && qlat.size(0) == latent.size(0) && qlat.size(2) == latent.size(2),
              "mla_decode shapes: qlat [B, H, L], latent [B, T, L]");
  const int64_t b = latent.size(0), tmax = latent.size(1), l = latent.size(2), h = qlat.size(1);
  const at::cuda::CUDAGuard gd(latent.device());
  int rps = 0;
  const int splits = kimi::mla_decode_splits((int)b, tmax, &rps);
  auto opts = qlat.options();
  auto part = at::empty({b, splits, h, l}, opts);
  auto ml = at::empty({b, splits, h, 2}, opts);
  auto ctx = at::empty({b, h, l}, opts);
  check(kimi::mla_decode(dtype_code(latent), qlat.data_ptr<float>(), latent.data_ptr(), len.data_ptr<int32_t>(),
                         (int)b, (int)h, (int)l, tmax, part.data_ptr<float>(), ml.data_ptr<float>(), splits, rps,
                         ctx.data_ptr<float>(), stream()),
        "mla_decode");
  return ctx;
}

at::Tensor sample_tokens(at::Tensor logits, c10::optional<at::Tensor> seen, double penalty, double temperature,
                         int64_t top_k, double top_p, bool do_sample, at::Tensor seed_offset) {
  logits = dense(logits);
  TORCH_CHECK(logits.dim() == 2, "logits must be [B, V]");
  TORCH_CHECK(seed_offset.is_cuda() && seed_offset.scalar_type() == at::kLong && seed_offset.numel() >= 2,
              "seed_offset must be a CUDA int64 tensor {seed, offset}");
  const int64_t b = logits.size(0), vocab = logits.size(1);
  const at::cuda::CUDAGuard gd(logits.device());
  const uint32_t* sp = nullptr;
  int words = 0;
  if (seen.has_value() && seen->defined()) {
    CHECK_CUDA_CONTIG((*seen));
    TORCH_CHECK(seen->scalar_type() == at::kInt && seen->size(0) == b && seen->size(1) * 32 >= vocab,
                "seen must be an int32 bitmap [B, ceil(V / 32)]");
    sp = reinterpret_cast<const uint32_t*>(seen->data_ptr());
    words = (int)seen->size(1);
  }
  auto out = at::empty({b}, logits.options().dtype(at::kLong));
  check(kimi::sample_tokens(dtype_code(logits), logits.data_ptr(), (int)b, (int)vocab, sp, words, (float)penalty,
                            (float)temperature, (int)top_k, (float)top_p, do_sample,
                            seed_offset.data_ptr<int64_t>(), out.data_ptr<int64_t>(), stream()),
        "sample_tokens");
  return out;
}

void seen_mark(at::Tensor seen, at::Tensor ids, int64_t vocab) {
  CHECK_CUDA_CONTIG(seen);
  TORCH_CHECK(seen.scalar_type() == at::kInt && ids.dim() == 2 && ids.size(0) == seen.size(0), "seen_mark shapes");
  auto idc = dense(ids.to(at::kLong));
  const at::cuda::CUDAGuard gd(seen.device());
  check(kimi::seen_mark(reinterpret_cast<uint32_t*>(seen.data_ptr()), (int)seen.size(1), idc.data_ptr<int64_t>(),
                        idc.size(0), idc.size(1), idc.size(1), (int)vocab, stream()),
        "seen_mark");
}

// ---------------------------------------------------------------- expert-parallel comm
// `ptrs`: nine regions x world peer addresses, region-major (flags, counts, xs, row_token,
// row_weight, agg, dagg, dxs, dw_row).
kimi::EpPeers make_peers(const std::vector<int64_t>& ptrs, int64_t rank, int64_t world, at::Tensor status,
                         int64_t timeout_ns) {
  TORCH_CHECK(world >= 1 && world <= 8 && (int64_t)ptrs.size() == 9 * world && rank >= 0 && rank < world,
              "expert-parallel peers: 9 regions x world (<= 8) pointers");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "status must be an int32 CUDA tensor");
  kimi::EpPeers p;
  p.rank = (int)rank;
  p.world = (int)world;
  for (int r = 0; r < world; ++r) {
    p.flags[r] = reinterpret_cast<int*>(ptrs[0 * world + r]);
    p.counts[r] = reinterpret_cast<int*>(ptrs[1 * world + r]);
    p.xs[r] = reinterpret_cast<void*>(ptrs[2 * world + r]);
    p.row_token[r] = reinterpret_cast<int*>(ptrs[3 * world + r]);
    p.row_weight[r] = reinterpret_cast<float*>(ptrs[4 * world + r]);
    p.agg[r] = reinterpret_cast<float*>(ptrs[5 * world + r]);
    p.dagg[r] = reinterpret_cast<float*>(ptrs[6 * world + r]);
    p.dxs[r] = reinterpret_cast<void*>(ptrs[7 * world + r]);
    p.dw_row[r] = reinterpret_cast<float*>(ptrs[8 * world + r]);
  }
  p.status = status.data_ptr<int>();
  p.timeout_ns = timeout_ns;
  return p;
}

#define EP_PEER_ARGS std::vector<int64_t> ptrs, int64_t rank, int64_t world, at::Tensor status, int64_t timeout_ns
#define EP_PEERS make_peers(ptrs, rank, world, status, timeout_ns)

void ep_count(at::Tensor sel, int64_t E, at::Tensor cnt, at::Tensor agg) {
  CHECK_CUDA_CONTIG(sel);
  CHECK_CUDA_CONTIG(cnt);
  CHECK_CUDA_CONTIG(agg);
  TORCH_CHECK(sel.scalar_type() == at::kLong && cnt.scalar_type() == at::kInt && cnt.numel() >= E &&
                  agg.scalar_type() == at::kFloat,
              "ep_count: int64 selections, int32 counts, fp32 aggregate");
  const at::cuda::CUDAGuard gd(sel.device());
  check(kimi::ep_count(sel.data_ptr<int64_t>(), sel.numel(), (int)E, cnt.data_ptr<int>(), agg.data_ptr<float>(),
                       agg.numel(), stream()),
        "ep_count");
}

void ep_exchange(EP_PEER_ARGS, at::Tensor cnt, int64_t E, int64_t per, int64_t L, at::Tensor offsets_local,
                 at::Tensor base, at::Tensor cursor) {
  const at::cuda::CUDAGuard gd(cnt.device());
  TORCH_CHECK(offsets_local.numel() == per + 1 && base.numel() >= E && cursor.numel() >= E, "ep_exchange shapes");
  check(kimi::ep_exchange(EP_PEERS, cnt.data_ptr<int>(), (int)E, (int)per, (int)L, offsets_local.data_ptr<int>(),
                          base.data_ptr<int>(), cursor.data_ptr<int>(), stream()),
        "ep_exchange");
}

void ep_dispatch(EP_PEER_ARGS, at::Tensor latent, at::Tensor sel, at::Tensor w, int64_t E, int64_t per,
                 at::Tensor base, at::Tensor cursor, at::Tensor slot_pos) {
  latent = dense(latent);
  auto wf = dense(w.to(at::kFloat));
  CHECK_CUDA_CONTIG(sel);
  TORCH_CHECK(latent.scalar_type() == at::kBFloat16 && latent.dim() == 2 && sel.scalar_type() == at::kLong &&
                  sel.dim() == 2 && sel.size(0) == latent.size(0) && slot_pos.numel() == sel.numel(),
              "ep_dispatch: bf16 latent [M, L], int64 selections [M, k]");
  const at::cuda::CUDAGuard gd(latent.device());
  check(kimi::ep_dispatch(EP_PEERS, latent.data_ptr(), sel.data_ptr<int64_t>(), wf.data_ptr<float>(),
                          (int)latent.size(0), (int)sel.size(1), (int)E, (int)per, (int)latent.size(1),
                          base.data_ptr<int>(), cursor.data_ptr<int>(), slot_pos.data_ptr<int>(), stream()),
        "ep_dispatch");
}

int64_t ep_dispatch_grid(int64_t slots) { return kimi::ep_dispatch_grid(slots); }

void ep_wait(EP_PEER_ARGS, int64_t kind, int64_t target) {
  const at::cuda::CUDAGuard gd(status.device());
  check(kimi::ep_wait(EP_PEERS, (int)kind, (uint32_t)target, stream()), "ep_wait");
}

void ep_signal_wait(EP_PEER_ARGS, int64_t kind) {
  const at::cuda::CUDAGuard gd(status.device());
  check(kimi::ep_signal_wait(EP_PEERS, (int)kind, stream()), "ep_signal_wait");
}

at::Tensor ep_dy(EP_PEER_ARGS, at::Tensor offsets_local, int64_t M, at::Tensor y) {
  CHECK_CUDA_CONTIG(y);
  TORCH_CHECK(y.scalar_type() == at::kBFloat16 && y.dim() == 2, "ep_dy: bf16 y [r_max, L]");
  const at::cuda::CUDAGuard gd(y.device());
  auto dy = at::empty_like(y);
  const int per = (int)offsets_local.numel() - 1;
  check(kimi::ep_dy(EP_PEERS, offsets_local.data_ptr<int>() + per, y.size(0), (int)M, (int)y.size(1), y.data_ptr(),
                    dy.data_ptr(), stream()),
        "ep_dy");
  return dy;
}

std::vector<at::Tensor> ep_slot_sum(EP_PEER_ARGS, at::Tensor sel, at::Tensor slot_pos, int64_t E, int64_t per,
                                    int64_t L, bool out_fp32) {
  CHECK_CUDA_CONTIG(sel);
  const at::cuda::CUDAGuard gd(sel.device());
  const int64_t M = sel.size(0), k = sel.size(1);
  auto dlat = at::empty({M, L}, sel.options().dtype(out_fp32 ? at::kFloat : at::kBFloat16));
  auto dweights = at::empty({M, k}, sel.options().dtype(at::kFloat));
  check(kimi::ep_slot_sum(EP_PEERS, sel.data_ptr<int64_t>(), slot_pos.data_ptr<int>(), (int)M, (int)k, (int)E,
                          (int)per, (int)L, dlat.data_ptr(), out_fp32, dweights.data_ptr<float>(), stream()),
        "ep_slot_sum");
  return {dlat, dweights};
}

// Down-projection of the routed experts with the combine fused into the epilogue: row r adds
// row_weight[r] * (a[r] @ b[g]^T) into agg_peers[row_token[r] / tokens_per_rank] at token
// row_token[r] % tokens_per_rank (a peer's fp32 [tokens, N] aggregate, over NVLink).
void tc_gemm_grouped_remote(at::Tensor a, at::Tensor b, at::Tensor offsets, int64_t M, int64_t N, int64_t K,
                            at::Tensor row_token, at::Tensor row_weight, std::vector<int64_t> agg_peers,
                            int64_t tokens_per_rank, int64_t bn) {
  TORCH_CHECK(a.is_cuda() && a.dim() == 2 && a.stride(1) == 1 && a.stride(0) % 8 == 0, "a must be row-major");
  CHECK_CUDA_CONTIG(b);
  CHECK_CUDA_CONTIG(row_token);
  CHECK_CUDA_CONTIG(row_weight);
  TORCH_CHECK(!agg_peers.empty() && agg_peers.size() <= 8 && tokens_per_rank > 0, "agg_peers: 1..8 pointers");
  const at::cuda::CUDAGuard gd(a.device());
  kimi::TcGemmArgs g;
  g.mode = 1;
  g.bn = (int)bn;
  g.a = a.data_ptr();
  g.a_rows = a.size(0);
  g.a_cols = a.size(1);
  g.a_ld = a.stride(0);
  g.b = b.data_ptr();
  g.b_groups = b.size(0);
  g.b_rows = b.size(1);
  g.b_cols = b.size(2);
  g.b_ld = b.size(2);
  g.b_gstride = b.size(1) * b.size(2);
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.G = (int)offsets.numel() - 1;
  g.offsets = offsets.data_ptr<int>();
  g.epi = 2;
  g.out = reinterpret_cast<void*>(agg_peers[0]);
  g.out_fp32 = true;
  g.ldc = N;
  g.row_token = row_token.data_ptr<int>();
  g.row_weight = row_weight.data_ptr<float>();
  for (size_t r = 0; r < agg_peers.size(); ++r) g.agg_peer[r] = (uint64_t)agg_peers[r];
  g.agg_tokens = (int)tokens_per_rank;
  check(kimi::tc_gemm(g, stream()), "tc_gemm_grouped_remote");
}

// Y [world * rows, N] = all-gather(x shards) @ w^T in one kernel.  `buf` is this rank's [M, K]
// symmetric gather buffer (its own shard already in rows [rank * rows, ...)); `peers` every rank's
// buffer base.  The kernel's comm warps copy each remote block once over NVLink into `buf`.
at::Tensor tc_gemm_allgather(at::Tensor buf, at::Tensor w, std::vector<int64_t> peers, int64_t rank, int64_t rows,
                             at::Tensor flags, at::Tensor epoch, at::Tensor status, at::Tensor out, int64_t bn) {
  TORCH_CHECK(buf.is_cuda() && buf.scalar_type() == at::kBFloat16 && buf.dim() == 2 && buf.is_contiguous(),
              "buf must be a contiguous bf16 [M, K] gather buffer");
  CHECK_CUDA_CONTIG(w);
  CHECK_CUDA_CONTIG(out);
  CHECK_CUDA_CONTIG(flags);
  const int64_t world = (int64_t)peers.size();
  TORCH_CHECK(world >= 1 && world <= 8 && buf.size(0) == world * rows && w.scalar_type() == at::kBFloat16 &&
                  w.size(1) == buf.size(1) && out.size(0) == buf.size(0) && out.size(1) == w.size(0) &&
                  out.scalar_type() == at::kBFloat16 && flags.scalar_type() == at::kInt &&
                  flags.numel() >= buf.size(0) / 128 && epoch.scalar_type() == at::kInt &&
                  status.scalar_type() == at::kInt,
              "tc_gemm_allgather shapes");
  const at::cuda::CUDAGuard gd(buf.device());
  kimi::TcGemmArgs g;
  g.mode = 0;
  g.bn = (int)bn;
  g.a = buf.data_ptr();
  g.a_rows = buf.size(0);
  g.a_cols = buf.size(1);
  g.a_ld = buf.size(1);
  g.b = w.data_ptr();
  g.b_groups = 1;
  g.b_rows = w.size(0);
  g.b_cols = w.size(1);
  g.b_ld = w.size(1);
  g.b_gstride = w.numel();
  g.M = (int)buf.size(0);
  g.N = (int)w.size(0);
  g.K = (int)w.size(1);
  g.G = 1;
  g.out = out.data_ptr();
  g.out_fp32 = false;
  g.ldc = out.size(1);
  g.ag_world = (int)world;
  g.ag_rows = (int)rows;
  g.ag_rank = (int)rank;
  g.ag_flags = reinterpret_cast<uint32_t*>(flags.data_ptr());
  g.ag_epoch = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  g.status = status.data_ptr<int>();
  for (int64_t r = 0; r < world; ++r) g.ag_peer[r] = (uint64_t)peers[r];
  g.num_sms = at::cuda::getDeviceProperties(buf.get_device())->multiProcessorCount;
  check(kimi::tc_gemm(g, stream()), "tc_gemm_allgather");
  return out;
}

}  // namespace

namespace {
// KIMI_K3_SEGV_TRACE=1: print the native stack of a segmentation fault (diagnostics only).
void segv_trace(int sig) {
  void* frames[64];
  const int n = backtrace(frames, 64);
  backtrace_symbols_fd(frames, n, 2);
  signal(sig, SIG_DFL);
  raise(sig);
}
}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "kimi_k3_b200 sm_100a kernels";
  if (getenv("KIMI_K3_SEGV_TRACE")) signal(SIGSEGV, segv_trace);
  m.def("rms_norm_fwd", &rms_norm_fwd);
  m.def("conv_step", &conv_step);
  m.def("ep_count", &ep_count);
  m.def("ep_exchange", &ep_exchange);
  m.def("ep_dispatch", &ep_dispatch);
  m.def("ep_dispatch_grid", &ep_dispatch_grid);
  m.def("ep_wait", &ep_wait);
  m.def("ep_signal_wait", &ep_signal_wait);
  m.def("ep_dy", &ep_dy);
  m.def("ep_slot_sum", &ep_slot_sum);
  m.def("tc_gemm_grouped_remote", &tc_gemm_grouped_remote);
  m.def("tc_gemm_allgather", &tc_gemm_allgather);
  m.def("kda_decode", &kda_decode);
  m.def("mla_decode_supported", &mla_decode_supported);
  m.def("mla_decode", &mla_decode);
  m.def("sample_tokens", &sample_tokens);
  m.def("seen_mark", &seen_mark);
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
  m.def("tcs_selftest", &tcs_selftest);
  m.def("muon_momentum", &muon_momentum);
  m.def("cast_bf16_multi", &cast_bf16_multi);
  m.def("ns_poly", &ns_poly);
  m.def("muon_normalize", &muon_normalize);
  m.def("muon_apply", &muon_apply);
  m.def("kda_phase_profile", &kimi::kda_phase_profile);
  m.def("kda_tc_status", [](bool clear) { return kimi::kda_tc_status(clear); });
  m.def("kda_fwd", &kda_fwd);
  m.def("kda_bwd", &kda_bwd);
  m.def("fa_fwd", &fa_fwd);
  m.def("fa_bwd", &fa_bwd);
  m.def("tc_gemm_dense", &tc_gemm_dense, py::arg("a"), py::arg("b"), py::arg("a_mn"), py::arg("b_mn"),
        py::arg("out_fp32"), py::arg("bn"), py::arg("out") = py::none(), py::arg("status") = py::none(),
        py::arg("spin_limit") = 0, py::arg("accumulate") = false, py::arg("ksplit") = 1,
        py::arg("bias") = py::none(), py::arg("residual") = py::none(), py::arg("pair") = -1, py::arg("debug") = 0,
        py::arg("dbg") = py::none());
  // Views of the current device's default status words of the GEMM and the KDA kernels (int32
  // [1] each, not owned): a training step copies them to pinned host memory with its other
  // per-step flags, so a bounded wait that gave up inside a kernel surfaces at the next step.
  m.def("status_words", []() {
    const int dev = c10::cuda::current_device();
    auto opts = at::TensorOptions().dtype(at::kInt).device(at::kCUDA, dev);
    int* g = kimi::tc_gemm_default_status();
    int* k = kimi::kda_tc_default_status();
    TORCH_CHECK(g && k, "status words unavailable on this device");
    return std::vector<at::Tensor>{at::from_blob(g, {1}, opts), at::from_blob(k, {1}, opts)};
  });
  m.def("tc_gemm_status", [](bool clear) {
    const int v = kimi::tc_gemm_status(clear);
    TORCH_CHECK(v >= 0, "reading the GEMM status word failed");
    return v;
  });
  m.def("tc_gemm_grouped", &tc_gemm_grouped, py::arg("mode"), py::arg("a"), py::arg("b"), py::arg("b2"),
        py::arg("a_mn"), py::arg("b_mn"), py::arg("offsets"), py::arg("M"), py::arg("N"), py::arg("K"), py::arg("epi"),
        py::arg("out"), py::arg("out_fp32"), py::arg("bg"), py::arg("bu"), py::arg("row_token"), py::arg("row_weight"),
        py::arg("b2_k_split"), py::arg("bn"), py::arg("uniform_rows") = 0);
  m.def("tc_gemm_group", &tc_gemm_group, py::arg("kind"), py::arg("segs"), py::arg("x"), py::arg("w"),
        py::arg("out") = py::none(), py::arg("bn") = 256, py::arg("ksplit") = 1, py::arg("pair") = -1);
  m.def("tc_gemm_comm", &tc_gemm_comm);
  m.def("tc_gemm_tiles", [](int64_t m, int64_t n, int64_t bn) { return kimi::tc_gemm_tiles((int)m, (int)n, (int)bn); });
  m.def("moe_route", &moe_route);
  m.def("moe_gather", &moe_gather);
  m.def("moe_dy", &moe_dy);
  m.def("moe_slot_sum", &moe_slot_sum);
  m.def("situ_bwd_cat", &situ_bwd_cat);
}
