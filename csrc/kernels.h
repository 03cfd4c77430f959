// Host-side launch entry points of the kimi_k3_b200 CUDA kernels.
// Each launcher takes raw device pointers and a stream and returns the launch status.
// dtype codes: 0 = float32, 1 = bfloat16, 2 = float16.
#pragma once
#include <vector>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kimi {

// ---- norms / gates / activations (elementwise.cu)
cudaError_t rms_norm_fwd(int dtype, const void* x, const float* w, void* y, float* rstd, int64_t rows, int dim,
                         int weight_period, float eps, cudaStream_t s);
cudaError_t rms_norm_bwd(int dtype, const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                         float* dw, int64_t rows, int dim, int weight_period, cudaStream_t s);
cudaError_t situ_glu_fwd(int dtype, const void* g, const void* u, void* y, int64_t n, float bg, float bu,
                         cudaStream_t s);
cudaError_t situ_glu_bwd(int dtype, const void* dy, const void* g, const void* u, void* dg, void* du, int64_t n,
                         float bg, float bu, cudaStream_t s);
cudaError_t sigmoid_mul_fwd(int dtype, const void* z, const void* x, void* y, int64_t n, cudaStream_t s);
cudaError_t sigmoid_mul_bwd(int dtype, const void* dy, const void* z, const void* x, void* dz, void* dx, int64_t n,
                            cudaStream_t s);
cudaError_t kda_decay_fwd(int dtype, const void* z, const float* a_log, float* g, int64_t rows, int heads,
                          int kdim, float g_min, float clamp_eps, cudaStream_t s);
cudaError_t kda_decay_bwd(int dtype, const float* dg, const void* z, const float* a_log, void* dz, float* da_log,
                          int64_t rows, int heads, int kdim, float g_min, float clamp_eps, cudaStream_t s);
cudaError_t conv_silu_norm_fwd(int dtype, const void* x, const float* w, void* y, int batch, int tokens,
                               int channels, int ksize, int head_dim, float eps, bool normalize, cudaStream_t s);
cudaError_t conv_silu_norm_bwd(int dtype, const void* dy, const void* x, const float* w, void* dx, float* dw,
                               float* dw_part, int batch, int tokens, int channels, int ksize, int head_dim, float eps,
                               bool normalize, cudaStream_t s);
// Rows of the dw scratch conv_silu_norm_bwd needs ([rows, channels * ksize] fp32).
int conv_bwd_partial_rows(int batch, int tokens);

// ---- attention residual depth mix (attnres.cu); sources: device array of S pointers
cudaError_t attnres_mix_fwd(int dtype, const void* const* sources, int num_sources, const float* q, const float* w,
                            void* out, float* probs, float* rstd, int64_t tokens, int dim, float eps,
                            cudaStream_t s);
cudaError_t attnres_mix_bwd(int dtype, const void* const* sources, int num_sources, const float* q, const float* w,
                            const void* dout, const float* probs, const float* rstd, void* const* dsources,
                            float* dq, float* dw, int64_t tokens, int dim, cudaStream_t s);

// ---- cross-entropy rows (ce.cu): logits rows with leading dimension ld (elements)
cudaError_t ce_rows_fwd_bwd(int dtype, void* logits, int64_t ld, int64_t rows, int vocab, const int64_t* targets,
                            const bool* valid, float* loss_rows, float grad_scale, cudaStream_t s);

// ---- router (router.cu)
cudaError_t router_topk(int dtype, const void* logits, const float* bias, int64_t rows, int experts, int k,
                        bool need_cutoff, float eps, int64_t* sel, float* raw_sel, float* weights, float* cutoff,
                        int64_t* load, float* raw_out, cudaStream_t s);

// ---- KDA chunk (kda_chunk.cu); head dims 64, chunk 64, tokens padded to a multiple of 64.
// Intermediates are fp32 [B*H, NC, 64, 64] (eGC: [B*H, NC, 64]) and are kept for backward.
struct KdaBuffers {
  float* W;       // M (k e^G)            rows = chunk tokens, cols = key dim
  float* U;       // M v
  float* P;       // lower((q e^G)(k e^-G)^T)
  float* Qg;      // q e^G
  float* Kend;    // k e^(G_C - G)
  float* eGC;     // e^(G_C)
  float* states;  // S at the start of each chunk  [K x V]
  float* Vp;      // U - W S
  float* Araw = nullptr;  // strict_lower(sum_d k_i k_j e^(G_i - G_j)), kept for the backward
};
cudaError_t kda_chunk_fwd(int dtype, const void* q, const void* k, const void* v, const float* g, const float* beta,
                          const float* h0, void* o, float* ht, KdaBuffers buf, int batch, int tokens_padded,
                          int heads, cudaStream_t s, int* status = nullptr);
cudaError_t kda_chunk_bwd(int dtype, const void* q, const void* k, const void* v, const float* g, const float* beta,
                          KdaBuffers buf, const void* dout, const float* dht, float* dVp, float* dSn, float* dq,
                          float* dk, float* dv, float* dg, float* dbeta, float* dh0, int batch, int tokens_padded,
                          int heads, int* status, cudaStream_t s);

// Intra-chunk backward on tcgen05 (kda_tc.cu); needs buf.Araw from the forward and dV', dS_next
// from the state backward.  Mbarrier timeouts are reported through `status` (0 = ok).
cudaError_t kda_intra_bwd_tc(int dtype, const void* q, const void* k, const void* v, const float* g,
                             const float* beta, KdaBuffers buf, const float* araw, const void* dout, const float* dVp,
                             const float* dSn, float* dq, float* dk, float* dv, float* dg, float* dbeta, int batch,
                             int tokens_padded, int heads, int* status, cudaStream_t s);
// Intra-chunk forward on tcgen05 (kda_tc.cu): W, U, P, Qg, Kend, eGC and Araw of every chunk.
cudaError_t kda_intra_fwd_tc(int dtype, const void* q, const void* k, const void* v, const float* g,
                             const float* beta, KdaBuffers buf, int batch, int tokens_padded, int heads, int* status,
                             cudaStream_t s);
// Sequential state passes on tcgen05 (kda_tc.cu): forward fills buf.states / buf.Vp and writes o
// (and ht); backward writes dV' and dS_next per chunk (and dh0).
cudaError_t kda_state_fwd_tc(int dtype, KdaBuffers buf, const float* h0, void* o, float* ht, int batch,
                             int tokens_padded, int heads, int* status, cudaStream_t s);
cudaError_t kda_state_bwd_tc(int dtype, KdaBuffers buf, const void* dout, const float* dht, float* dVp, float* dSn,
                             float* dh0, int batch, int tokens_padded, int heads, int* status, cudaStream_t s);
// Phase timestamps (clock64) of the intra backward's first chunk on block 0 from the last launch
// made while enabled; enable / disable recording for later launches.
std::vector<long long> kda_phase_profile(bool enable);
// Device status word shared by the tcgen05 KDA kernels (read and cleared by the host).
int kda_tc_status(bool clear);

// ---- bf16 mirrors of fp32 tensors (optim.cu): device tables of source / destination pointers,
// element counts and the prefix sums of ceil(numel / 8) (tensors + 1 entries); 16-byte aligned tensors.
cudaError_t cast_bf16_multi(const float* const* src, void* const* dst, const int64_t* numel, const int64_t* vec_off,
                            int tensors, int64_t total_vec, cudaStream_t s);
// Newton-Schulz polynomial c * G2 + b * G + a * I over a batch of [m, m] matrices stacked as
// [rows, m] (bf16, m a multiple of 8, 16-byte aligned).
cudaError_t ns_poly(const void* g, const void* g2, void* out, int64_t rows, int m, float a, float b, float c,
                    cudaStream_t s);
// Device address of the current device's default KDA status word (for stream-ordered reads).
int* kda_tc_default_status();

// ---- flash attention (flash_attn.cu); q/k/v/o are [B,T,H,D] contiguous
cudaError_t flash_attn_fwd(int dtype, const void* q, const void* k, const void* v, void* o, float* lse, int batch,
                           int tq, int tk, int heads, int dqk, int dv, bool causal, const int* key_lengths,
                           float scale, cudaStream_t s);
cudaError_t flash_attn_bwd(int dtype, const void* q, const void* k, const void* v, const void* o, const void* dout,
                           const float* lse, float* dq_acc, void* dk, void* dv, float* delta, int batch, int tq,
                           int tk, int heads, int dqk, int dv_dim, bool causal, const int* key_lengths, float scale,
                           cudaStream_t s);

// ---- fused Muon passes around the Newton-Schulz GEMMs (optim.cu); one bucket of `count`
// equal-shape matrices of `mn` elements, contiguous
cudaError_t muon_momentum(const float* g, float* mom, void* x_bf16, float* sumsq, int count, int64_t mn,
                          float momentum, bool nesterov, const bool* skip, cudaStream_t s);
cudaError_t muon_normalize(void* x_bf16, const float* sumsq, int count, int64_t mn, float eps, cudaStream_t s);
cudaError_t muon_apply(const void* o_bf16, float* const* params, const float* sumsq, int count, int64_t mn,
                       const float* lr, float wd, float scale, float eps, const bool* skip, float* stats,
                       cudaStream_t s);

// ---- self-test of the small-matrix tcgen05 path (tc_small_selftest.cu)
cudaError_t tcs_selftest(const float* A, const float* B, float* out, int K, int n, int mode, int* status,
                         cudaStream_t s);

// ---------------------------------------------------------------- decode step (decode.cu)
// Up to three short-conv streams advanced by one token in one launch; head_lanes = head_dim / 8
// for a per-head L2 norm after the SiLU, 0 for none.  bias[i] may be nullptr.
struct ConvStepArgs {
  const void* x[3];
  void* hist[3];
  const float* w[3];
  const float* bias[3];
  void* y[3];
  int channels[3];
  int head_lanes[3];
};
cudaError_t conv_step(int dtype, const ConvStepArgs& args, int streams, int batch, int ksize, float eps,
                      cudaStream_t s);
cudaError_t kda_decode(int dtype, const void* q, const void* k, const void* v, const float* g, const float* beta,
                       const float* state_in, float* state_out, void* o, int batch, int heads, cudaStream_t s);
bool mla_decode_supported(int heads, int ldim);
int mla_decode_splits(int batch, int64_t tmax, int* rows_per_split);
cudaError_t mla_decode(int dtype, const float* qlat, const void* latent, const int32_t* lengths, int batch,
                       int heads, int ldim, int64_t tmax, float* part_acc, float* part_ml, int splits,
                       int rows_per_split, float* ctx, cudaStream_t s);
cudaError_t sample_tokens(int dtype, const void* logits, int batch, int vocab, const uint32_t* seen, int seen_words,
                          float penalty, float temperature, int top_k, float top_p, bool do_sample,
                          const int64_t* seed_offset, int64_t* out, cudaStream_t s);
cudaError_t seen_mark(uint32_t* seen, int seen_words, const int64_t* ids, int64_t rows, int64_t cols, int64_t ld,
                      int vocab, cudaStream_t s);

// ---------------------------------------------------------------- expert-parallel comm (ep_comm.cu)
// Pointers into every rank's symmetric buffer (index = rank in the expert group).
struct EpPeers {
  int rank = 0, world = 1;
  int* flags[8] = {};       // [kinds][8] counting semaphores
  int* counts[8] = {};      // [world, E]
  void* xs[8] = {};         // [r_max, L] bf16 expert-input rows
  int* row_token[8] = {};   // [r_max]
  float* row_weight[8] = {};
  float* agg[8] = {};       // [M, L] fp32
  float* dagg[8] = {};      // [M, L] fp32
  void* dxs[8] = {};        // [r_max, L] bf16
  float* dw_row[8] = {};    // [r_max]
  int* status = nullptr;    // local
  int64_t timeout_ns = 10000000000LL;
};
int ep_dispatch_grid(int64_t slots);
cudaError_t ep_count(const int64_t* sel, int64_t n, int E, int* cnt, float* agg, int64_t agg_elems, cudaStream_t s);
cudaError_t ep_exchange(const EpPeers& p, const int* cnt, int E, int per, int L, int* offsets_local, int* base,
                        int* cursor, cudaStream_t s);
cudaError_t ep_dispatch(const EpPeers& p, const void* latent, const int64_t* sel, const float* w, int M, int k, int E,
                        int per, int L, const int* base, int* cursor, int* slot_pos, cudaStream_t s);
cudaError_t ep_wait(const EpPeers& p, int kind, uint32_t target, cudaStream_t s);
cudaError_t ep_signal_wait(const EpPeers& p, int kind, cudaStream_t s);
cudaError_t ep_dy(const EpPeers& p, const int* offsets_total, int64_t r_max, int M, int L, const void* y, void* dy,
                  cudaStream_t s);
cudaError_t ep_slot_sum(const EpPeers& p, const int64_t* sel, const int* slot_pos, int M, int k, int E, int per, int L,
                        void* dlat, bool out_fp32, float* dweights, cudaStream_t s);

}  // namespace kimi
