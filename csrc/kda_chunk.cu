// Kimi Delta Attention chunk kernels (forward + backward), head dims 64, chunk 64.
//
// Per chunk of C = 64 tokens with G = cumsum(g) (per key channel):
//   A   = diag(beta) * strict_lower(Kq Kd^T)             (A_ij = sum_k k_ik k_jk e^{G_ik - G_jk})
//   L   = I + A,   [W | U] = L^-1 diag(beta) [k e^G | v]
//   P   = lower((q e^G)(k e^-G)^T)                       (computed with rebased factors)
//   V'  = U - W S,   O = (q e^G) S + P V',   S <- e^{G_C} S + (k e^{G_C - G})^T V'
//
// Work split (chunk-parallel; only the state pass is sequential):
//   kda_intra_fwd  grid (NC, B*H): A, the triangular solve, P, Qg, Kend, e^{G_C}  -> global fp32
//   kda_state_fwd  grid (B*H, V/VB): sequential over chunks: V', O, S (S_c saved per chunk)
//   kda_state_bwd  grid (B*H, V/VB): reverse: dV' = P^T dO + Kend dS ; dS <- Qg^T dO + e^{G_C} dS - W^T dV'
//   kda_intra_bwd  grid (NC, B*H): every remaining gradient of the chunk (derivation below)
//
// Pairwise factors e^{G_i - G_j} (j <= i) are evaluated per 16-row tile I with a reference
// r = G at the first row of I: e^{G_i - r} <= 1 for i in I, e^{r - G_j} <= 1 for j before I and
// <= e^{-15 g_min} inside I, so nothing overflows in fp32 for g >= -5.8.
//
// Backward of the intra-chunk algebra (X = [W|U], R = [k e^G | v], Y = L^-T [dW | dU]):
//   dQg = dO S^T,   dP = lower(dO V'^T),   dW = -dV' S^T,   dU = dV',   dKend = V' dSn^T
//   d(k e^G) = beta * Y_K,  dv = beta * Y_V,  dbeta_i = sum_c R_ic Y_ic + sum_{j<i} A_ij dL_ij
//   dL = -Y X^T (strict lower),  dA = diag(beta) dL
//   A / P pair grads: dk_i += (dA Kd)_i e^{G_i - r},  dk_j += (dA^T Kq)_j e^{r - G_j},
//                     dG_i += Kq_i (dA Kd)_i,  dG_j -= Kd_j (dA^T Kq)_j   (same with q for P)
//   dG_C += e^{G_C} rowsum(S * dSn) + sum_j Kend_j dKend_j;  dg = reverse cumsum of dG.
#include "common.cuh"
#include "kernels.h"

namespace kimi {
namespace {

constexpr int C = 64;     // chunk
constexpr int D = 64;     // key and value head dim
constexpr int LD = 65;    // padded smem row stride
constexpr int LDX = 129;  // [kg | v] rows
constexpr int NT = 256;   // threads per block
constexpr int VB = 32;    // value columns per state block

KIMI_D int64_t tok_off(int b, int t, int h, int T, int H) { return (((int64_t)b * T + t) * H + h) * D; }
KIMI_D int64_t blk_off(int bh, int c, int NC) { return ((int64_t)bh * NC + c) * C * D; }

// Γ = cumsum over rows of g (per column), in place.
KIMI_D void cumsum_rows(float* sG) {
  if (threadIdx.x < D) {
    float acc = 0.f;
    for (int i = 0; i < C; ++i) {
      acc += sG[i * LD + threadIdx.x];
      sG[i * LD + threadIdx.x] = acc;
    }
  }
}

// Build the rebased tile operands for row tile I (rows s0..s0+15):
//   sKd[j][d] = k_jd e^{G_s0,d - G_jd} for j < s0+16 (0 otherwise),  sE[i][d] = e^{G_id - G_s0,d},
//   sKq[i][d] = k_id sE[i][d],  sQq[i][d] = q_id sE[i][d]  (sQq optional)
KIMI_D void build_tile(int s0, const float* sG, const float* sK, const float* sQ, float* sKd, float* sE, float* sKq,
                       float* sQq) {
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int j = idx / D, d = idx % D;
    sKd[j * LD + d] = (j < s0 + 16) ? sK[j * LD + d] * expf(sG[s0 * LD + d] - sG[j * LD + d]) : 0.f;
  }
  for (int idx = threadIdx.x; idx < 16 * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D, i = s0 + r;
    const float e = expf(sG[i * LD + d] - sG[s0 * LD + d]);
    sE[r * LD + d] = e;
    sKq[r * LD + d] = sK[i * LD + d] * e;
    if (sQq) sQq[r * LD + d] = sQ[i * LD + d] * e;
  }
}

// ------------------------------------------------------------------ intra forward
template <typename T>
__global__ void __launch_bounds__(NT) kda_intra_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                           const T* __restrict__ v, const float* __restrict__ g,
                                                           const float* __restrict__ beta, KdaBuffers buf, int Tp,
                                                           int H) {
  extern __shared__ float sm[];
  float* sG = sm;
  float* sK = sG + C * LD;
  float* sQ = sK + C * LD;
  float* sA = sQ + C * LD;
  float* sKd = sA + C * LD;
  float* sX = sKd + C * LD;       // [C][LDX]
  float* sE = sX + C * LDX;       // [16][LD]
  float* sKq = sE + 16 * LD;
  float* sQq = sKq + 16 * LD;
  float* sB = sQq + 16 * LD;      // [C]
  const int c = blockIdx.x, NC = gridDim.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int t0 = c * C;
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    const int64_t off = tok_off(b, t0 + i, h, Tp, H) + d;
    sK[i * LD + d] = to_f<T>(k[off]);
    sQ[i * LD + d] = to_f<T>(q[off]);
    sG[i * LD + d] = g[off];
    sX[i * LDX + D + d] = to_f<T>(v[off]);
  }
  for (int i = threadIdx.x; i < C; i += blockDim.x) sB[i] = beta[((int64_t)b * Tp + t0 + i) * H + h];
  __syncthreads();
  cumsum_rows(sG);
  __syncthreads();
  const int64_t bo = blk_off(bh, c, NC);
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    const float G = sG[i * LD + d], e = expf(G);
    sX[i * LDX + d] = sK[i * LD + d] * e;
    buf.Qg[bo + i * D + d] = sQ[i * LD + d] * e;
    buf.Kend[bo + i * D + d] = sK[i * LD + d] * expf(sG[(C - 1) * LD + d] - G);
  }
  if (threadIdx.x < D) buf.eGC[((int64_t)bh * NC + c) * D + threadIdx.x] = expf(sG[(C - 1) * LD + threadIdx.x]);
  // A (strict lower) and P (lower incl. diagonal), tile by tile.
  for (int I = 0; I < 4; ++I) {
    const int s0 = I * 16;
    __syncthreads();
    build_tile(s0, sG, sK, sQ, sKd, sE, sKq, sQq);
    __syncthreads();
    for (int o = threadIdx.x; o < 16 * C; o += blockDim.x) {
      const int r = o / C, j = o % C, i = s0 + r;
      float aa = 0.f, pp = 0.f;
      if (j <= i) {
#pragma unroll 8
        for (int d = 0; d < D; ++d) {
          const float kd = sKd[j * LD + d];
          aa += sKq[r * LD + d] * kd;
          pp += sQq[r * LD + d] * kd;
        }
      }
      sA[i * LD + j] = (j < i) ? aa : 0.f;
      buf.P[bo + i * C + j] = pp;
    }
  }
  __syncthreads();
  // Forward substitution: X_i = beta_i (R_i - sum_{j<i} A_ij X_j), 128 columns.
  for (int i = 0; i < C; ++i) {
    if (threadIdx.x < 2 * D) {
      const int col = threadIdx.x;
      float acc = sX[i * LDX + col];
      for (int j = 0; j < i; ++j) acc -= sA[i * LD + j] * sX[j * LDX + col];
      sX[i * LDX + col] = sB[i] * acc;
    }
    __syncthreads();
  }
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    buf.W[bo + i * D + d] = sX[i * LDX + d];
    buf.U[bo + i * D + d] = sX[i * LDX + D + d];
  }
}

// ------------------------------------------------------------------ state forward (sequential)
template <typename T>
__global__ void __launch_bounds__(NT) kda_state_fwd_kernel(KdaBuffers buf, const float* __restrict__ h0,
                                                           T* __restrict__ o, float* __restrict__ ht, int NC, int Tp,
                                                           int H) {
  extern __shared__ float sm[];
  constexpr int LV = VB + 1;
  float* sW = sm;
  float* sQg = sW + C * LD;
  float* sP = sQg + C * LD;
  float* sKe = sP + C * LD;
  float* sS = sKe + C * LD;     // [D][LV]
  float* sU = sS + D * LV;      // [C][LV]
  float* sVp = sU + C * LV;     // [C][LV]
  float* sE = sVp + C * LV;     // [D]
  const int bh = blockIdx.x, b = bh / H, h = bh % H, v0 = blockIdx.y * VB;
  for (int idx = threadIdx.x; idx < D * VB; idx += blockDim.x) {
    const int kk = idx / VB, vv = idx % VB;
    sS[kk * LV + vv] = h0 ? h0[(int64_t)bh * D * D + kk * D + v0 + vv] : 0.f;
  }
  for (int c = 0; c < NC; ++c) {
    const int64_t bo = blk_off(bh, c, NC);
    __syncthreads();
    for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
      const int i = idx / D, d = idx % D;
      sW[i * LD + d] = buf.W[bo + idx];
      sQg[i * LD + d] = buf.Qg[bo + idx];
      sP[i * LD + d] = buf.P[bo + idx];
      sKe[i * LD + d] = buf.Kend[bo + idx];
    }
    for (int idx = threadIdx.x; idx < C * VB; idx += blockDim.x) {
      const int i = idx / VB, vv = idx % VB;
      sU[i * LV + vv] = buf.U[bo + i * D + v0 + vv];
      buf.states[bo + i * D + v0 + vv] = sS[i * LV + vv];  // rows of S are key channels (C == D)
    }
    if (threadIdx.x < D) sE[threadIdx.x] = buf.eGC[((int64_t)bh * NC + c) * D + threadIdx.x];
    __syncthreads();
    // V' = U - W S
    for (int idx = threadIdx.x; idx < C * VB; idx += blockDim.x) {
      const int i = idx / VB, vv = idx % VB;
      float acc = sU[i * LV + vv];
#pragma unroll 8
      for (int kk = 0; kk < D; ++kk) acc -= sW[i * LD + kk] * sS[kk * LV + vv];
      sVp[i * LV + vv] = acc;
      buf.Vp[bo + i * D + v0 + vv] = acc;
    }
    __syncthreads();
    // O = Qg S + P V'
    for (int idx = threadIdx.x; idx < C * VB; idx += blockDim.x) {
      const int i = idx / VB, vv = idx % VB;
      float acc = 0.f;
#pragma unroll 8
      for (int kk = 0; kk < D; ++kk) acc += sQg[i * LD + kk] * sS[kk * LV + vv];
      for (int j = 0; j <= i; ++j) acc += sP[i * LD + j] * sVp[j * LV + vv];
      o[tok_off(b, c * C + i, h, Tp, H) + v0 + vv] = from_f<T>(acc);
    }
    __syncthreads();
    // S <- e^{G_C} S + Kend^T V'  (each thread owns its own S entries: in-place is safe)
    for (int idx = threadIdx.x; idx < D * VB; idx += blockDim.x) {
      const int kk = idx / VB, vv = idx % VB;
      float acc = sE[kk] * sS[kk * LV + vv];
#pragma unroll 8
      for (int j = 0; j < C; ++j) acc += sKe[j * LD + kk] * sVp[j * LV + vv];
      sS[kk * LV + vv] = acc;
    }
  }
  __syncthreads();
  if (ht)
    for (int idx = threadIdx.x; idx < D * VB; idx += blockDim.x) {
      const int kk = idx / VB, vv = idx % VB;
      ht[(int64_t)bh * D * D + kk * D + v0 + vv] = sS[kk * LV + vv];
    }
}

// ------------------------------------------------------------------ state backward (reverse sequential)
template <typename T>
__global__ void __launch_bounds__(NT) kda_state_bwd_kernel(KdaBuffers buf, const T* __restrict__ dout,
                                                           const float* __restrict__ dht, float* __restrict__ dVp,
                                                           float* __restrict__ dSn, float* __restrict__ dh0, int NC,
                                                           int Tp, int H) {
  extern __shared__ float sm[];
  constexpr int LV = VB + 1;
  float* sW = sm;
  float* sQg = sW + C * LD;
  float* sP = sQg + C * LD;
  float* sKe = sP + C * LD;
  float* sdS = sKe + C * LD;    // [D][LV]
  float* sdO = sdS + D * LV;    // [C][LV]
  float* sdV = sdO + C * LV;    // [C][LV]
  float* sE = sdV + C * LV;     // [D]
  const int bh = blockIdx.x, b = bh / H, h = bh % H, v0 = blockIdx.y * VB;
  for (int idx = threadIdx.x; idx < D * VB; idx += blockDim.x) {
    const int kk = idx / VB, vv = idx % VB;
    sdS[kk * LV + vv] = dht ? dht[(int64_t)bh * D * D + kk * D + v0 + vv] : 0.f;
  }
  for (int c = NC - 1; c >= 0; --c) {
    const int64_t bo = blk_off(bh, c, NC);
    __syncthreads();
    for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
      const int i = idx / D, d = idx % D;
      sW[i * LD + d] = buf.W[bo + idx];
      sQg[i * LD + d] = buf.Qg[bo + idx];
      sP[i * LD + d] = buf.P[bo + idx];
      sKe[i * LD + d] = buf.Kend[bo + idx];
    }
    for (int idx = threadIdx.x; idx < C * VB; idx += blockDim.x) {
      const int i = idx / VB, vv = idx % VB;
      sdO[i * LV + vv] = to_f<T>(dout[tok_off(b, c * C + i, h, Tp, H) + v0 + vv]);
      dSn[bo + i * D + v0 + vv] = sdS[i * LV + vv];
    }
    if (threadIdx.x < D) sE[threadIdx.x] = buf.eGC[((int64_t)bh * NC + c) * D + threadIdx.x];
    __syncthreads();
    // dV' = P^T dO + Kend dS
    for (int idx = threadIdx.x; idx < C * VB; idx += blockDim.x) {
      const int j = idx / VB, vv = idx % VB;
      float acc = 0.f;
      for (int i = j; i < C; ++i) acc += sP[i * LD + j] * sdO[i * LV + vv];
#pragma unroll 8
      for (int kk = 0; kk < D; ++kk) acc += sKe[j * LD + kk] * sdS[kk * LV + vv];
      sdV[j * LV + vv] = acc;
      dVp[bo + j * D + v0 + vv] = acc;
    }
    __syncthreads();
    // dS <- Qg^T dO + e^{G_C} dS - W^T dV'
    for (int idx = threadIdx.x; idx < D * VB; idx += blockDim.x) {
      const int kk = idx / VB, vv = idx % VB;
      float acc = sE[kk] * sdS[kk * LV + vv];
#pragma unroll 8
      for (int i = 0; i < C; ++i) acc += sQg[i * LD + kk] * sdO[i * LV + vv] - sW[i * LD + kk] * sdV[i * LV + vv];
      sdS[kk * LV + vv] = acc;
    }
  }
  __syncthreads();
  if (dh0)
    for (int idx = threadIdx.x; idx < D * VB; idx += blockDim.x) {
      const int kk = idx / VB, vv = idx % VB;
      dh0[(int64_t)bh * D * D + kk * D + v0 + vv] = sdS[kk * LV + vv];
    }
}

// ------------------------------------------------------------------ intra backward
template <typename T>
__global__ void __launch_bounds__(NT) kda_intra_bwd_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, KdaBuffers buf, const T* __restrict__ dout, const float* __restrict__ dVp,
    const float* __restrict__ dSn, float* __restrict__ dq, float* __restrict__ dk, float* __restrict__ dv,
    float* __restrict__ dg, float* __restrict__ dbeta, int Tp, int H) {
  extern __shared__ float sm[];
  float* sG = sm;
  float* sK = sG + C * LD;
  float* sQ = sK + C * LD;
  float* sA = sQ + C * LD;   // A, later Kd temp
  float* sB1 = sA + C * LD;
  float* sB2 = sB1 + C * LD;
  float* sB3 = sB2 + C * LD;
  float* sDG = sB3 + C * LD;  // dΓ accumulator
  float* sT1 = sDG + C * LD;  // dL -> dA
  float* sT2 = sT1 + C * LD;  // dP
  float* sE = sT2 + C * LD;   // [16][LD]
  float* sKq = sE + 16 * LD;
  float* sQq = sKq + 16 * LD;
  float* sBeta = sQq + 16 * LD;  // [C]
  float* sDB = sBeta + C;        // dbeta [C]
  float* sDGC = sDB + C;         // dΓ_C [D]
  const int c = blockIdx.x, NC = gridDim.x, bh = blockIdx.y, b = bh / H, h = bh % H, t0 = c * C;
  const int64_t bo = blk_off(bh, c, NC);
  auto goff = [&](int i, int d) { return tok_off(b, t0 + i, h, Tp, H) + d; };

  // phase 0: inputs, zero accumulators
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    const int64_t off = goff(i, d);
    sK[i * LD + d] = to_f<T>(k[off]);
    sQ[i * LD + d] = to_f<T>(q[off]);
    sG[i * LD + d] = g[off];
    sDG[i * LD + d] = 0.f;
    dq[off] = 0.f;
    dk[off] = 0.f;
  }
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    sBeta[i] = beta[((int64_t)b * Tp + t0 + i) * H + h];
    sDB[i] = 0.f;
    sDGC[i] = 0.f;
  }
  __syncthreads();
  cumsum_rows(sG);
  __syncthreads();

  // phase 1: A (strict lower), sB1 used as the Kd tile
  for (int I = 0; I < 4; ++I) {
    const int s0 = I * 16;
    build_tile(s0, sG, sK, sQ, sB1, sE, sKq, nullptr);
    __syncthreads();
    for (int o = threadIdx.x; o < 16 * C; o += blockDim.x) {
      const int r = o / C, j = o % C, i = s0 + r;
      float aa = 0.f;
      if (j < i) {
#pragma unroll 8
        for (int d = 0; d < D; ++d) aa += sKq[r * LD + d] * sB1[j * LD + d];
      }
      sA[i * LD + j] = aa;
    }
    __syncthreads();
  }

  // phase 2: dO -> sB1, V' -> sB2, S -> sB3; dP and dQg
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    sB1[i * LD + d] = to_f<T>(dout[goff(i, d)]);
    sB2[i * LD + d] = buf.Vp[bo + idx];
    sB3[i * LD + d] = buf.states[bo + idx];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < C * C; o += blockDim.x) {
    const int i = o / C, j = o % C;
    float acc = 0.f;
    if (j <= i) {
#pragma unroll 8
      for (int vv = 0; vv < D; ++vv) acc += sB1[i * LD + vv] * sB2[j * LD + vv];
    }
    sT2[i * LD + j] = acc;  // dP
    // dQg[i][kk] with kk = j: sum_v dO[i][v] S[kk][v]
    float dqg = 0.f;
#pragma unroll 8
    for (int vv = 0; vv < D; ++vv) dqg += sB1[i * LD + vv] * sB3[j * LD + vv];
    const float e = expf(sG[i * LD + j]);
    dq[goff(i, j)] += dqg * e;
    sDG[i * LD + j] += dqg * sQ[i * LD + j] * e;
  }
  __syncthreads();

  // phase 3: dSn -> sB1; dKend = V' dSn^T; state-decay term of dΓ_C
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    sB1[i * LD + d] = dSn[bo + idx];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < C * D; o += blockDim.x) {
    const int j = o / D, kk = o % D;
    float acc = 0.f;
#pragma unroll 8
    for (int vv = 0; vv < D; ++vv) acc += sB2[j * LD + vv] * sB1[kk * LD + vv];
    const float f = expf(sG[(C - 1) * LD + kk] - sG[j * LD + kk]);
    const float kend = sK[j * LD + kk] * f;
    dk[goff(j, kk)] += acc * f;
    sDG[j * LD + kk] -= acc * kend;
    atomicAdd(&sDGC[kk], acc * kend);
  }
  if (threadIdx.x < D) {
    const int kk = threadIdx.x;
    float acc = 0.f;
    for (int vv = 0; vv < D; ++vv) acc += sB3[kk * LD + vv] * sB1[kk * LD + vv];
    atomicAdd(&sDGC[kk], expf(sG[(C - 1) * LD + kk]) * acc);
  }
  __syncthreads();

  // phase 4: dV' -> sB2, dW = -dV' S^T -> sB1, then Y = L^-T [dW | dU] in place
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    sB2[i * LD + d] = dVp[bo + idx];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < C * D; o += blockDim.x) {
    const int j = o / D, kk = o % D;
    float acc = 0.f;
#pragma unroll 8
    for (int vv = 0; vv < D; ++vv) acc += sB2[j * LD + vv] * sB3[kk * LD + vv];
    sB1[j * LD + kk] = -acc;
  }
  __syncthreads();
  for (int i = C - 1; i >= 0; --i) {
    if (threadIdx.x < 2 * D) {
      float* col = threadIdx.x < D ? sB1 : sB2;
      const int cc = threadIdx.x % D;
      float acc = col[i * LD + cc];
      for (int j = i + 1; j < C; ++j) acc -= sBeta[j] * sA[j * LD + i] * col[j * LD + cc];
      col[i * LD + cc] = acc;
    }
    __syncthreads();
  }

  // phase 5: v -> sB3; d(k e^G), dv, dbeta (first part)
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    sB3[i * LD + d] = to_f<T>(v[goff(i, d)]);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    const float e = expf(sG[i * LD + d]);
    const float kg = sK[i * LD + d] * e;
    const float yk = sB1[i * LD + d], yv = sB2[i * LD + d];
    const float dkg = sBeta[i] * yk;
    dk[goff(i, d)] += dkg * e;
    sDG[i * LD + d] += dkg * kg;
    dv[goff(i, d)] = sBeta[i] * yv;
    atomicAdd(&sDB[i], kg * yk + sB3[i * LD + d] * yv);
  }
  __syncthreads();

  // phase 6: dL = -(Y_K W^T + Y_V U^T) (strict lower) -> sT1; dbeta += A.dL; dA = beta dL
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    sB3[i * LD + d] = buf.W[bo + idx];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < C * C; o += blockDim.x) {
    const int i = o / C, j = o % C;
    float acc = 0.f;
    if (j < i) {
#pragma unroll 8
      for (int d = 0; d < D; ++d) acc += sB1[i * LD + d] * sB3[j * LD + d];
    }
    sT1[i * LD + j] = -acc;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < C * D; idx += blockDim.x) {
    const int i = idx / D, d = idx % D;
    sB3[i * LD + d] = buf.U[bo + idx];
  }
  __syncthreads();
  for (int o = threadIdx.x; o < C * C; o += blockDim.x) {
    const int i = o / C, j = o % C;
    if (j < i) {
      float acc = 0.f;
#pragma unroll 8
      for (int d = 0; d < D; ++d) acc += sB2[i * LD + d] * sB3[j * LD + d];
      const float dl = sT1[i * LD + j] - acc;
      atomicAdd(&sDB[i], sA[i * LD + j] * dl);
      sT1[i * LD + j] = sBeta[i] * dl;
    } else {
      sT1[i * LD + j] = 0.f;
    }
  }
  __syncthreads();

  // phase 7: pair gradients through A (k,k) and P (q,k); sA is reused as the Kd tile.
  for (int I = 0; I < 4; ++I) {
    const int s0 = I * 16;
    build_tile(s0, sG, sK, sQ, sA, sE, sKq, sQq);
    __syncthreads();
    // row side (rows of tile I)
    for (int o = threadIdx.x; o < 16 * D; o += blockDim.x) {
      const int r = o / D, d = o % D, i = s0 + r;
      float ra = 0.f, rp = 0.f;
      for (int j = 0; j <= i; ++j) {
        const float kd = sA[j * LD + d];
        ra += sT1[i * LD + j] * kd;
        rp += sT2[i * LD + j] * kd;
      }
      const float e = sE[r * LD + d];
      dk[goff(i, d)] += ra * e;
      dq[goff(i, d)] += rp * e;
      sDG[i * LD + d] += ra * sKq[r * LD + d] + rp * sQq[r * LD + d];
    }
    __syncthreads();
    // column side (rows j <= s0+15)
    for (int o = threadIdx.x; o < (s0 + 16) * D; o += blockDim.x) {
      const int j = o / D, d = o % D;
      float gc = 0.f;
      for (int r = 0; r < 16; ++r) {
        const int i = s0 + r;
        if (j <= i) gc += sT1[i * LD + j] * sKq[r * LD + d] + sT2[i * LD + j] * sQq[r * LD + d];
      }
      const float f = expf(sG[s0 * LD + d] - sG[j * LD + d]);
      dk[goff(j, d)] += gc * f;
      sDG[j * LD + d] -= gc * sA[j * LD + d];
    }
    __syncthreads();
  }

  // phase 8: dg = reverse cumsum of dΓ (+ dΓ_C on the last row), dbeta
  if (threadIdx.x < D) {
    const int d = threadIdx.x;
    float acc = sDGC[d];
    for (int i = C - 1; i >= 0; --i) {
      acc += sDG[i * LD + d];
      dg[goff(i, d)] = acc;
    }
  }
  for (int i = threadIdx.x; i < C; i += blockDim.x) dbeta[((int64_t)b * Tp + t0 + i) * H + h] = sDB[i];
}

size_t intra_fwd_smem() { return (size_t)(5 * C * LD + C * LDX + 3 * 16 * LD + C) * sizeof(float); }
size_t state_smem() { return (size_t)(4 * C * LD + 3 * C * (VB + 1) + D) * sizeof(float); }
size_t intra_bwd_smem() { return (size_t)(10 * C * LD + 3 * 16 * LD + 3 * C) * sizeof(float); }

template <typename T>
cudaError_t fwd_impl(const void* q, const void* k, const void* v, const float* g, const float* beta, const float* h0,
                     void* o, float* ht, KdaBuffers buf, int B, int Tp, int H, cudaStream_t s) {
  const int NC = Tp / C;
  static bool configured = false;
  if (!configured) {
    KIMI_CUDA_CHECK(cudaFuncSetAttribute(kda_intra_fwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)intra_fwd_smem()));
    KIMI_CUDA_CHECK(cudaFuncSetAttribute(kda_state_fwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)state_smem()));
    configured = true;
  }
  kda_intra_fwd_kernel<T><<<dim3(NC, B * H), NT, intra_fwd_smem(), s>>>((const T*)q, (const T*)k, (const T*)v, g,
                                                                          beta, buf, Tp, H);
  KIMI_CUDA_CHECK(cudaGetLastError());
  kda_state_fwd_kernel<T><<<dim3(B * H, D / VB), NT, state_smem(), s>>>(buf, h0, (T*)o, ht, NC, Tp, H);
  return cudaGetLastError();
}

template <typename T>
cudaError_t bwd_impl(const void* q, const void* k, const void* v, const float* g, const float* beta, KdaBuffers buf,
                     const void* dout, const float* dht, float* dVp, float* dSn, float* dq, float* dk, float* dv,
                     float* dg, float* dbeta, float* dh0, int B, int Tp, int H, cudaStream_t s) {
  const int NC = Tp / C;
  static bool configured = false;
  if (!configured) {
    KIMI_CUDA_CHECK(cudaFuncSetAttribute(kda_state_bwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)state_smem()));
    KIMI_CUDA_CHECK(cudaFuncSetAttribute(kda_intra_bwd_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)intra_bwd_smem()));
    configured = true;
  }
  kda_state_bwd_kernel<T><<<dim3(B * H, D / VB), NT, state_smem(), s>>>(buf, (const T*)dout, dht, dVp, dSn, dh0, NC,
                                                                        Tp, H);
  KIMI_CUDA_CHECK(cudaGetLastError());
  kda_intra_bwd_kernel<T><<<dim3(NC, B * H), NT, intra_bwd_smem(), s>>>(
      (const T*)q, (const T*)k, (const T*)v, g, beta, buf, (const T*)dout, dVp, dSn, dq, dk, dv, dg, dbeta, Tp, H);
  return cudaGetLastError();
}

}  // namespace

cudaError_t kda_chunk_fwd(int dtype, const void* q, const void* k, const void* v, const float* g, const float* beta,
                          const float* h0, void* o, float* ht, KdaBuffers buf, int B, int Tp, int H, cudaStream_t s) {
  if (Tp % C) return cudaErrorInvalidValue;
  switch (dtype) {
    case 0: return fwd_impl<float>(q, k, v, g, beta, h0, o, ht, buf, B, Tp, H, s);
    case 1: return fwd_impl<__nv_bfloat16>(q, k, v, g, beta, h0, o, ht, buf, B, Tp, H, s);
    case 2: return fwd_impl<__half>(q, k, v, g, beta, h0, o, ht, buf, B, Tp, H, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t kda_chunk_bwd(int dtype, const void* q, const void* k, const void* v, const float* g, const float* beta,
                          KdaBuffers buf, const void* dout, const float* dht, float* dVp, float* dSn, float* dq,
                          float* dk, float* dv, float* dg, float* dbeta, float* dh0, int B, int Tp, int H,
                          cudaStream_t s) {
  if (Tp % C) return cudaErrorInvalidValue;
  switch (dtype) {
    case 0: return bwd_impl<float>(q, k, v, g, beta, buf, dout, dht, dVp, dSn, dq, dk, dv, dg, dbeta, dh0, B, Tp, H, s);
    case 1: return bwd_impl<__nv_bfloat16>(q, k, v, g, beta, buf, dout, dht, dVp, dSn, dq, dk, dv, dg, dbeta, dh0, B,
                                           Tp, H, s);
    case 2: return bwd_impl<__half>(q, k, v, g, beta, buf, dout, dht, dVp, dSn, dq, dk, dv, dg, dbeta, dh0, B, Tp, H,
                                    s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace kimi
