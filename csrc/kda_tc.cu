// Kimi Delta Attention: intra-chunk backward on tcgen05 (sm_100a), head dims 64, chunk 64.
//
// One persistent CTA (256 threads) per SM walks chunks (b, h, c).  Every product of the chunk
// runs as a kind::tf32 MMA with M = 128 (tc_small.cuh); the operands are written by the threads
// (scaled, masked or transposed on the way into shared memory) and the results come back from
// TMEM one accumulator row per thread.  Notation as in kda_chunk.cu (G = cumsum g per channel,
// r_I = G at the first row of 16-row tile I, A = strict_lower(sum_d k_i k_j e^{G_i - G_j})).
//
//   MMA-1  [dO; dV'] x [V'; S]^T          -> dP = lower(dO V'^T), dQg = dO S^T, dW = -dV' S^T
//   MMA-2  [V'; S] x dSn^T                 -> dKend = V' dSn^T, diag(S dSn^T) (the e^{G_C} term)
//   solve  Y = (I + diag(beta) A)^-T [dW | dV']   one column per thread, in registers
//   MMA-3  [Y_K | Y_V] x [W | U]^T         -> dL = -(Y_K W^T + Y_V U^T), dA = beta dL
//   MMA-4  [dA; dP] x Kown, per K tile J   -> row-side pair gradients; Kown_j = k_j e^{r_J - G_j}
//   MMA-5  [dA^T | dP^T] x [Kq | Qq], per K tile I -> column-side pair gradients;
//          Kq_i = k_i e^{G_i - r_I}, Qq_i = q_i e^{G_i - r_I}
//
// The row side uses  k_j e^{r_I - G_j} = e^{r_I - r_J} k_j e^{r_J - G_j}  (j in tile J <= I), so one
// operand per chunk serves every row tile; each tile's partial lands in its own 64 TMEM columns
// and is rescaled by e^{r_I - r_J} <= 1 when read.  The column side keeps one accumulator per row
// tile I and applies e^{r_I - G_j} (only for j <= 16 I + 15, where it is bounded by e^{-15 g_min}).
// Gradients of q and k accumulate in global fp32 (one writer per element per stage); dG
// accumulates in shared memory and becomes dg by a reverse cumulative sum.  Every mbarrier wait
// is bounded and reports through the status word.
#include <mutex>
#include <vector>

#include "kernels.h"
#include "tc_small.cuh"
#include "device_info.h"

namespace kimi {
namespace {

constexpr int C = 64;
constexpr int LDP = 65;                  // plain smem row stride (floats)
constexpr int NTH = 256;
constexpr int KB = 1024;
// operand arena (bytes from the 1024-aligned base)
constexpr int OFF_4A = 0;                // [dA; dP]      R128 K64   (32 KB)
constexpr int OFF_X = 32 * KB;           // [dO; dV']     R128 K64   | later [W | U]   R64 K128
constexpr int OFF_Y = 64 * KB;           // [V'; S]       R128 K64   | later plain RHS, then Kown R64 K64
constexpr int OFF_Z = 96 * KB;           // dSn           R64 K64
constexpr int OFF_5A = 80 * KB;          // [dA^T | dP^T] R64 K128
constexpr int OFF_3A = 112 * KB;         // [Y_K | Y_V]   R64 K128   | later [Kq | Qq] R64 K128
constexpr int ARENA = 152 * KB;          // M = 128 reads of R64 tiles reach 8 KB past their last atom
constexpr int LDT = 68;                  // A^T row stride (16-byte aligned rows)

// Optional phase timing of the intra backward (block 0, its first chunk, thread 0): clock64() at
// each phase boundary, enabled from the host for profiling runs only.
__device__ long long g_kda_phase[16];
__device__ int g_kda_phase_on = 0;
#define KIMI_PHASE(k)                                                          \
  do {                                                                          \
    if (phase_on && blockIdx.x == 0 && ci == 0 && tid == 0) g_kda_phase[k] = clock64(); \
  } while (0)

struct BwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  const void* dout;
  const float* W;
  const float* U;
  const float* S;
  const float* Vp;
  const float* Araw;
  const float* dVp;
  const float* dSn;
  float* dq;
  float* dk;
  float* dv;
  float* dg;
  float* dbeta;
  int B, Tp, H, NC;
  int* status;
};

KIMI_D int64_t tok_off(int b, int t, int h, int Tp, int H) { return (((int64_t)b * Tp + t) * H + h) * 64; }

template <typename T>
KIMI_D void load32(const T* p, float* out) {
#pragma unroll
  for (int i = 0; i < 32; ++i) out[i] = to_f<T>(p[i]);
}
template <>
KIMI_D void load32<float>(const float* p, float* out) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const float4 x = *reinterpret_cast<const float4*>(p + i);
    out[i] = x.x;
    out[i + 1] = x.y;
    out[i + 2] = x.z;
    out[i + 3] = x.w;
  }
}
template <>
KIMI_D void load32<__nv_bfloat16>(const __nv_bfloat16* p, float* out) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const uint4 x = *reinterpret_cast<const uint4*>(p + i);
    const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&x);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h2[j]);
      out[i + 2 * j] = f.x;
      out[i + 2 * j + 1] = f.y;
    }
  }
}

// 64 x 64 fp32 block (row-major, contiguous) -> rows [row0, row0 + 64) of a K-major tile.
KIMI_D void tile_from_f32(float* tile, int R, int row0, const float* src) {
  for (int idx = threadIdx.x; idx < 64 * 16; idx += NTH) {
    const int r = idx >> 4, k4 = (idx & 15) * 4;
    tcs::st4(tile, R, row0 + r, k4, *reinterpret_cast<const float4*>(src + r * 64 + k4));
  }
}
// 64 token rows of a [B,T,H,64] T tensor -> rows [row0, row0 + 64) of a K-major tile.
template <typename T>
KIMI_D void tile_from_tok(float* tile, int R, int row0, const T* base, int H) {
  for (int idx = threadIdx.x; idx < 64 * 16; idx += NTH) {
    const int r = idx >> 4, k4 = (idx & 15) * 4;
    const T* p = base + (int64_t)r * H * 64 + k4;
    tcs::st4(tile, R, row0 + r, k4, make_float4(to_f<T>(p[0]), to_f<T>(p[1]), to_f<T>(p[2]), to_f<T>(p[3])));
  }
}

KIMI_D float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// q / k rows for the row-owner threads: staged in shared memory for 16-bit inputs, read from
// global memory (L1) for fp32 inputs, where staging would not fit.
template <typename T>
struct QKRows {
  static constexpr bool kStaged = sizeof(T) == 2;
  static constexpr int LD = 72;  // elements per staged row (16-byte aligned, bank-staggered)
  const T* gq;
  const T* gk;
  int64_t rs;
  T* sq;
  T* sk;
  KIMI_D void stage(int tid, int nthreads) {
    if constexpr (kStaged) {
      for (int idx = tid; idx < 64 * 8; idx += nthreads) {
        const int i = idx >> 3, c8 = (idx & 7) * 8;
        *reinterpret_cast<uint4*>(sq + i * LD + c8) = *reinterpret_cast<const uint4*>(gq + i * rs + c8);
        *reinterpret_cast<uint4*>(sk + i * LD + c8) = *reinterpret_cast<const uint4*>(gk + i * rs + c8);
      }
    }
  }
  KIMI_D void row32(bool is_q, int i, int c0, float* out) const {
    if (kStaged) {
      const T* p = (is_q ? sq : sk) + i * LD + c0;
#pragma unroll
      for (int u = 0; u < 32; ++u) out[u] = to_f<T>(p[u]);
    } else {
      load32<T>((is_q ? gq : gk) + i * rs + c0, out);
    }
  }
  KIMI_D float at(bool is_q, int i, int d) const {
    return kStaged ? to_f<T>((is_q ? sq : sk)[i * LD + d]) : to_f<T>((is_q ? gq : gk)[i * rs + d]);
  }
};

// 16 warps: thread (TMEM row `row`, column quarter cq) owns columns [16 cq, 16 cq + 16) of each
// 64-wide block of its row, so twice as many warps share each phase's per-row work.
constexpr int NTB = 512;

template <typename T>
__global__ void __launch_bounds__(NTB, 1) kda_intra_bwd_tc_kernel(const __grid_constant__ BwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* arena = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* op4a = reinterpret_cast<float*>(arena + OFF_4A);
  float* opx = reinterpret_cast<float*>(arena + OFF_X);
  float* opy = reinterpret_cast<float*>(arena + OFF_Y);
  float* opz = reinterpret_cast<float*>(arena + OFF_Z);
  float* op5a = reinterpret_cast<float*>(arena + OFF_5A);
  float* op3a = reinterpret_cast<float*>(arena + OFF_3A);
  float* op3b = opx;   // [W | U]                         (after MMA-1/2)
  float* op5b = opx;   // [Kq | Qq]^T                     (after MMA-3)
  float* rhs = op5a;   // plain [64][128] solve workspace (after MMA-1/2)
  float* op4b = opy;   // Kown^T                          (after MMA-1/2)
  float* stage = op3a; // plain [2][64][LDP] dk / dq      (after MMA-4/5)
  float* sG = reinterpret_cast<float*>(arena + ARENA);
  float* sDG = sG + C * LDP;
  float* sAT = sDG + C * LDP;  // A^T: sAT[j][i] = A_ij (the solve reads rows of A^T as float4)
  float* sBeta = sAT + C * LDT;
  float* sDB = sBeta + C;
  float* sDGC = sDB + C;
  T* sQK = reinterpret_cast<T*>(sDGC + C);
  uint64_t* bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sQK) +
                                              (QKRows<T>::kStaged ? 2 * 64 * QKRows<T>::LD * sizeof(T) : 0));
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = (warp & 3) * 32 + lane;  // TMEM lane of this thread
  const int cq = warp >> 2;                // column quarter handled by this thread
  const int c0 = 16 * cq;
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tm = *slot;
  uint32_t phase = 0;
  const int phase_on = g_kda_phase_on;
  const int H = a.H, Tp = a.Tp, NC = a.NC;
  const int total = a.B * H * NC;

  for (int ci = blockIdx.x; ci < total; ci += gridDim.x) {
    const int bh = ci / NC, c = ci % NC, b = bh / H, h = bh % H, t0 = c * C;
    const int64_t bo = ((int64_t)bh * NC + c) * C * 64;
    const int64_t tok0 = tok_off(b, t0, h, Tp, H);
    const int64_t rs = (int64_t)H * 64;  // token stride
    const T* v = reinterpret_cast<const T*>(a.v) + tok0;
    const T* dout = reinterpret_cast<const T*>(a.dout) + tok0;
    const float* g = a.g + tok0;
    QKRows<T> qk{reinterpret_cast<const T*>(a.q) + tok0, reinterpret_cast<const T*>(a.k) + tok0, rs, sQK,
                 sQK + 64 * QKRows<T>::LD};
    // dk for TMEM lanes 0..63 (rows of dV', V', dA), dq for lanes 64..127 (rows of dO, dP)
    float gacc[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) gacc[u] = 0.f;
    const int ri = row & 63;

    KIMI_PHASE(0);
    // ---------------------------------------------------------------- loads (all issued before any use)
    {
      float gv[8], av[8];
      float4 t4[5][2];
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int idx = tid + n * NTB, i = idx >> 6, d = idx & 63;
        gv[n] = g[i * rs + d];
        av[n] = a.Araw[bo + idx];
      }
      const float* srcs[4] = {a.dVp + bo, a.Vp + bo, a.S + bo, a.dSn + bo};
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          const int idx = tid + n * NTB, r = idx >> 4, k4 = (idx & 15) * 4;
          t4[m][n] = *reinterpret_cast<const float4*>(srcs[m] + r * 64 + k4);
        }
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int idx = tid + n * NTB, r = idx >> 4, k4 = (idx & 15) * 4;
        const T* p = dout + (int64_t)r * rs + k4;
        t4[4][n] = make_float4(to_f<T>(p[0]), to_f<T>(p[1]), to_f<T>(p[2]), to_f<T>(p[3]));
      }
      const float bt = tid < C ? a.beta[((int64_t)b * Tp + t0 + tid) * H + h] : 0.f;
      qk.stage(tid, NTB);
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int idx = tid + n * NTB, i = idx >> 6, d = idx & 63;
        sG[i * LDP + d] = gv[n];
        sDG[i * LDP + d] = 0.f;
        sAT[d * LDT + i] = av[n];
      }
#pragma unroll
      for (int n = 0; n < 2; ++n) {
        const int idx = tid + n * NTB, r = idx >> 4, k4 = (idx & 15) * 4;
        tcs::st4(opx, 128, r, k4, t4[0][n]);        // dV'
        tcs::st4(opx, 128, 64 + r, k4, t4[4][n]);   // dO
        tcs::st4(opy, 128, r, k4, t4[1][n]);        // V'
        tcs::st4(opy, 128, 64 + r, k4, t4[2][n]);   // S
        tcs::st4(opz, 64, r, k4, t4[3][n]);         // dSn
      }
      if (tid < C) {
        sBeta[tid] = bt;
        sDB[tid] = 0.f;
        sDGC[tid] = 0.f;
      }
    }
    __syncthreads();
    KIMI_PHASE(1);
    {  // G = cumsum over rows: eight 8-row segments per channel, then the segment offsets
      const int d = tid & 63, part = tid >> 6;
      float run = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        run += sG[(8 * part + r) * LDP + d];
        sG[(8 * part + r) * LDP + d] = run;
      }
      __syncthreads();
      float off = 0.f;
      for (int p2 = 0; p2 < part; ++p2) off += sG[(8 * p2 + 7) * LDP + d];
      __syncthreads();
      if (part > 0) {
#pragma unroll
        for (int r = 0; r < 8; ++r) sG[(8 * part + r) * LDP + d] += off;
      }
    }
    tcs::operands_ready();
    KIMI_PHASE(2);
    if (tid == 0) {
      tcs::mma_rows128(tm, opx, 128, opy, 128, 0, 128, 0, 64, false);      // MMA-1 -> cols [0,128)
      tcs::mma_rows128(tm + 128, opy, 128, opz, 64, 0, 64, 0, 64, false);  // MMA-2 -> cols [128,192)
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 11);
    KIMI_PHASE(3);

    // ---------------------------------------------------------------- read MMA-1 / MMA-2
    {
      float val[16];
      if (row < 64) {
        const int j = ri;
        // dW = -(dV' S^T) -> left half of the solve's right-hand side; dU = dV' -> right half
        tcs::tmem_row16(tm, warp, 64 + c0, val);
#pragma unroll
        for (int u = 0; u < 16; u += 4)
          *reinterpret_cast<float4*>(rhs + j * 128 + c0 + u) = make_float4(-val[u], -val[u + 1], -val[u + 2], -val[u + 3]);
#pragma unroll
        for (int u = 0; u < 16; ++u) rhs[j * 128 + 64 + c0 + u] = tcs::ld(opx, 128, j, c0 + u);
        // dKend = V' dSn^T: dk = dKend e^{G_C - G}, dG -= dKend Kend, dG_C += sum_j dKend Kend
        tcs::tmem_row16(tm + 128, warp, c0, val);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int d = c0 + u;
          const float f = expf(sG[63 * LDP + d] - sG[j * LDP + d]);
          const float kend = qk.at(false, j, d) * f;
          gacc[u] = val[u] * f;
          atomicAdd(&sDG[j * LDP + d], -val[u] * kend);
          const float sum = warp_sum(val[u] * kend);
          if (lane == 0) atomicAdd(&sDGC[d], sum);
        }
      } else {
        const int i = ri;
        // dP = lower(dO V'^T) -> rows 64.. of [dA; dP]
        tcs::tmem_row16(tm, warp, c0, val);
#pragma unroll
        for (int u = 0; u < 16; u += 4) {
          const int j = c0 + u;
          tcs::st4(op4a, 128, 64 + i, j,
                   make_float4(j <= i ? val[u] : 0.f, j + 1 <= i ? val[u + 1] : 0.f, j + 2 <= i ? val[u + 2] : 0.f,
                               j + 3 <= i ? val[u + 3] : 0.f));
        }
        // dQg = dO S^T: dq = dQg e^G, dG += dQg q e^G
        tcs::tmem_row16(tm, warp, 64 + c0, val);
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int d = c0 + u;
          const float e = expf(sG[i * LDP + d]);
          gacc[u] = val[u] * e;
          atomicAdd(&sDG[i * LDP + d], val[u] * qk.at(true, i, d) * e);
        }
        // diag(S dSn^T): the e^{G_C} term of dG_C; the warp of column quarter cq holds channels 16 cq..
        tcs::tmem_row16(tm + 128, warp, c0, val);
        if ((i >> 4) == cq) {
          float mine = 0.f;
#pragma unroll
          for (int u = 0; u < 16; ++u)
            if (u == (i & 15)) mine = val[u];
          atomicAdd(&sDGC[i], expf(sG[63 * LDP + i]) * mine);
        }
      }
    }
    __syncthreads();
    KIMI_PHASE(4);

    // ---------------------------------------------------------------- solve (threads 384..511) | W, U, Kown
    if (tid >= 384) {
      // L^T Y = R with L = I + diag(beta) A, one column per thread, 16-row blocks from the bottom
      const int col = tid - 384;
      for (int J = 3; J >= 0; --J) {
        const int j0 = 16 * J;
        float yb[16], zb[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) yb[u] = rhs[(j0 + u) * 128 + col];
#pragma unroll
        for (int jj = 15; jj >= 0; --jj) {
          zb[jj] = sBeta[j0 + jj] * yb[jj];
#pragma unroll
          for (int ii = 0; ii < jj; ++ii) yb[ii] -= sAT[(j0 + ii) * LDT + j0 + jj] * zb[jj];
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) tcs::st(op3a, 64, j0 + u, col, yb[u]);
        if (col >= 64) {
          float* dv = a.dv + tok0;
#pragma unroll
          for (int u = 0; u < 16; ++u) dv[(j0 + u) * rs + col - 64] = zb[u];
        }
        for (int i = 0; i < j0; ++i) {
          const float4* ap = reinterpret_cast<const float4*>(sAT + i * LDT + j0);
          float acc = rhs[i * 128 + col];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 a4 = ap[q4];
            acc -= a4.x * zb[4 * q4] + a4.y * zb[4 * q4 + 1] + a4.z * zb[4 * q4 + 2] + a4.w * zb[4 * q4 + 3];
          }
          rhs[i * 128 + col] = acc;
        }
      }
    } else {
      for (int idx = tid; idx < 64 * 16; idx += 384) {
        const int r = idx >> 4, k4 = (idx & 15) * 4;
        const float4 w4 = *reinterpret_cast<const float4*>(a.W + bo + r * 64 + k4);
        const float4 u4 = *reinterpret_cast<const float4*>(a.U + bo + r * 64 + k4);
        tcs::st4(op3b, 64, r, k4, w4);
        tcs::st4(op3b, 64, r, 64 + k4, u4);
      }
      // Kown^T: B[d][j] = k_jd e^{r_J(j),d - G_jd}
      for (int idx = tid; idx < 64 * 64; idx += 384) {
        const int jt = idx >> 6, d = idx & 63;
        tcs::st(op4b, 64, d, jt, qk.at(false, jt, d) * expf(sG[(jt & ~15) * LDP + d] - sG[jt * LDP + d]));
      }
    }
    tcs::operands_ready();
    KIMI_PHASE(5);
    if (tid == 0) {
      tcs::mma_rows128(tm, op3a, 64, op3b, 64, 0, 64, 0, 128, false);  // MMA-3 -> cols [0,64)
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 12);
    KIMI_PHASE(6);

    // ---------------------------------------------------------------- dL -> dA, dbeta, Y terms | [Kq | Qq]
    if (row < 64) {
      const int i = ri;
      float val[16];
      tcs::tmem_row16(tm, warp, c0, val);
      float part = 0.f;
      const float bi = sBeta[i];
#pragma unroll
      for (int u = 0; u < 16; u += 4) {
        float da[4];
#pragma unroll
        for (int w4 = 0; w4 < 4; ++w4) {
          const int j = c0 + u + w4;
          const float dl = j < i ? -val[u + w4] : 0.f;
          part += sAT[j * LDT + i] * dl;
          da[w4] = bi * dl;
        }
        tcs::st4(op4a, 128, i, c0 + u, make_float4(da[0], da[1], da[2], da[3]));
      }
      // d(k e^G) = beta Y_K: dk += beta Y_K e^G, dG += beta Y_K k e^G; dbeta += k e^G . Y_K + v . Y_V
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int d = c0 + u;
        const float yk = tcs::ld(op3a, 64, i, d), yv = tcs::ld(op3a, 64, i, 64 + d);
        const float e = expf(sG[i * LDP + d]);
        const float kg = qk.at(false, i, d) * e;
        gacc[u] += bi * yk * e;
        atomicAdd(&sDG[i * LDP + d], bi * yk * kg);
        part += kg * yk + to_f<T>(v[i * rs + d]) * yv;
      }
      atomicAdd(&sDB[i], part);
    } else {
      // [Kq | Qq]^T: B[d][i] = k_id e^{G_id - r_I(i),d}, B[d][64 + i] = q_id e^{G_id - r_I(i),d}
      const int t2 = (warp & 1) * 32 + (warp >> 2) * 64 + lane;  // 0..255 over the warps of lanes 64..127
      for (int idx = t2; idx < 64 * 64; idx += 256) {
        const int t = idx >> 6, d = idx & 63;
        const float e = expf(sG[t * LDP + d] - sG[(t & ~15) * LDP + d]);
        tcs::st(op5b, 64, d, t, qk.at(false, t, d) * e);
        tcs::st(op5b, 64, d, 64 + t, qk.at(true, t, d) * e);
      }
    }
    __syncthreads();
    KIMI_PHASE(7);
    // [dA^T | dP^T]
    for (int idx = tid; idx < 64 * 64; idx += NTB) {
      const int i = idx >> 6, j = idx & 63;
      tcs::st(op5a, 64, j, i, tcs::ld(op4a, 128, i, j));
      tcs::st(op5a, 64, j, 64 + i, tcs::ld(op4a, 128, 64 + i, j));
    }
    tcs::operands_ready();
    KIMI_PHASE(8);
    if (tid == 0) {
#pragma unroll
      for (int J = 0; J < 4; ++J)  // MMA-4: row side, K tile J -> cols [64J, 64J+64)
        tcs::mma_rows128(tm + 64 * J, op4a, 128, op4b, 64, 0, 64, 16 * J, 16, false);
#pragma unroll
      for (int I = 0; I < 4; ++I) {  // MMA-5: column side, K tile I (dA part, then dP part)
        tcs::mma_rows128(tm + 256 + 64 * I, op5a, 64, op5b, 64, 0, 64, 16 * I, 16, false);
        tcs::mma_rows128(tm + 256 + 64 * I, op5a, 64, op5b, 64, 0, 64, 64 + 16 * I, 16, true);
      }
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 13);
    KIMI_PHASE(9);

    // ---------------------------------------------------------------- row side (dk rows: dA, dq rows: dP)
    {
      const bool is_p = row >= 64;
      const int i = ri, I = i >> 4;
      float acc[16], val[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) acc[u] = 0.f;
#pragma unroll
      for (int J = 0; J < 4; ++J) {
        tcs::tmem_row16(tm + 64 * J, warp, c0, val);
        if (J <= I) {
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const int d = c0 + u;
            acc[u] += expf(sG[16 * I * LDP + d] - sG[16 * J * LDP + d]) * val[u];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int d = c0 + u;
        const float e = expf(sG[i * LDP + d] - sG[16 * I * LDP + d]);
        gacc[u] += acc[u] * e;
        atomicAdd(&sDG[i * LDP + d], acc[u] * qk.at(is_p, i, d) * e);
      }
      // column side (lanes 0..63): dk_j += sum_I e^{r_I - G_j} gc_I, dG_j -= k_j (same)
      if (!is_p) {
        const int j = i;
#pragma unroll
        for (int u = 0; u < 16; ++u) acc[u] = 0.f;
#pragma unroll
        for (int I2 = 0; I2 < 4; ++I2) {
          tcs::tmem_row16(tm + 256 + 64 * I2, warp, c0, val);
          if (j <= 16 * I2 + 15) {
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const int d = c0 + u;
              acc[u] += val[u] * expf(sG[16 * I2 * LDP + d] - sG[j * LDP + d]);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          gacc[u] += acc[u];
          atomicAdd(&sDG[j * LDP + c0 + u], -acc[u] * qk.at(false, j, c0 + u));
        }
      }
    }
    // dk / dq rows -> staging tile -> coalesced stores
#pragma unroll
    for (int u = 0; u < 16; ++u) stage[(row >= 64 ? C * LDP : 0) + ri * LDP + c0 + u] = gacc[u];
    __syncthreads();
    KIMI_PHASE(10);
    {
      float* dq = a.dq + tok0;
      float* dk = a.dk + tok0;
      for (int idx = tid; idx < C * 64; idx += NTB) {
        const int i = idx >> 6, d = idx & 63;
        dk[i * rs + d] = stage[i * LDP + d];
        dq[i * rs + d] = stage[C * LDP + i * LDP + d];
      }
      // dg = reverse cumsum of dG (+ dG_C): eight 8-row segments per channel, then the offsets
      const int d = tid & 63, part = tid >> 6;
      float run = 0.f;
#pragma unroll
      for (int r = 7; r >= 0; --r) {
        run += sDG[(8 * part + r) * LDP + d];
        sDG[(8 * part + r) * LDP + d] = run;
      }
      __syncthreads();
      float off = sDGC[d];
      for (int p2 = part + 1; p2 < 8; ++p2) off += sDG[(8 * p2) * LDP + d];
      float* dg = a.dg + tok0;
#pragma unroll
      for (int r = 0; r < 8; ++r) dg[(8 * part + r) * rs + d] = sDG[(8 * part + r) * LDP + d] + off;
      if (tid < C) a.dbeta[((int64_t)b * Tp + t0 + tid) * H + h] = sDB[tid];
    }
    tc::tc_fence_before();
    __syncthreads();
    KIMI_PHASE(11);
    tc::tc_fence_after();
  }
  if (warp == 0) tc::tmem_dealloc(tm, 512);
}

template <typename T>
size_t bwd_smem() {
  return 1024 + ARENA + (size_t)(2 * C * LDP + C * LDT + 3 * C) * sizeof(float) +
         (QKRows<T>::kStaged ? 2 * 64 * QKRows<T>::LD * sizeof(T) : 0) + 16;
}

template <typename T>
cudaError_t launch_bwd(const BwdArgs& args, cudaStream_t s) {
  {
    cudaError_t e = ensure_dynamic_smem(kda_intra_bwd_tc_kernel<T>, (int)bwd_smem<T>());
    if (e != cudaSuccess) return e;
  }
  const int total = args.B * args.H * args.NC;
  const int sms = device_sms();
  const int grid = total < sms ? total : sms;
  kda_intra_bwd_tc_kernel<T><<<grid, NTB, bwd_smem<T>(), s>>>(args);
  return cudaGetLastError();
}

// ======================================================================== intra forward
// One persistent CTA per SM walks chunks.  A single M = 128 MMA gives both pair matrices:
//   [Kq; Qq] x [Kd^(0) | Kd^(1) | Kd^(2) | Kd^(3)]^T   (N = 256)
// with Kq_i = k_i e^{G_i - r_I(i)}, Qq_i = q_i e^{G_i - r_I(i)} and Kd^(I)_j = k_j e^{r_I - G_j} for
// j <= 16 I + 15 (zero beyond, so no exponential overflows); row i keeps column block I(i).
// Then [W | U] = (I + diag(beta) A)^-1 diag(beta) [k e^G | v] by forward substitution (one column
// per thread, 16-row register blocks), and the elementwise outputs Qg, Kend, e^{G_C}.
struct FwdArgs {
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const float* beta;
  KdaBuffers buf;
  int B, Tp, H, NC;
  int* status;
};

template <typename T>
__global__ void __launch_bounds__(NTH, 1) kda_intra_fwd_tc_kernel(const __grid_constant__ FwdArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* tQK = reinterpret_cast<float*>(base);            // R128 K64 [Kq; Qq]
  float* tKd = reinterpret_cast<float*>(base + 32 * KB);  // R256 K64 [Kd^(0..3)]
  float* rhs = reinterpret_cast<float*>(base + 96 * KB);  // plain [64][128]
  float* sG = reinterpret_cast<float*>(base + 128 * KB);
  float* sA = sG + C * LDP;     // A (row-major, stride LDT)
  float* sBeta = sA + C * LDT;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sBeta + C);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = (warp & 3) * 32 + (tid & 31), half = warp >> 2, c0 = 32 * half;
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(slot, 256);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tm = *slot;
  uint32_t phase = 0;
  const int H = a.H, Tp = a.Tp, NC = a.NC;
  const int total = a.B * H * NC;
  const int64_t rs = (int64_t)H * 64;
  // The global inputs of a chunk (g, beta, q, k, v) are loaded into registers one chunk ahead:
  // the loads of chunk ci + gridDim.x are issued before chunk ci's solve and land while it runs.
  float gv[16], kr[16], qr[16], vr[16], bt = 0.f;
  auto load_chunk = [&](int cj) {
    const int bhj = cj / NC, cc = cj % NC, bj = bhj / H, hj = bhj % H;
    const int64_t tj = tok_off(bj, cc * C, hj, Tp, H);
    const float* gj = a.g + tj;
    const T* qj = reinterpret_cast<const T*>(a.q) + tj;
    const T* kj = reinterpret_cast<const T*>(a.k) + tj;
    const T* vj = reinterpret_cast<const T*>(a.v) + tj;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int idx = tid + n * NTH, i = idx >> 6, d = idx & 63;
      gv[n] = gj[i * rs + d];
      kr[n] = to_f<T>(kj[i * rs + d]);
      qr[n] = to_f<T>(qj[i * rs + d]);
      vr[n] = to_f<T>(vj[i * rs + d]);
    }
    bt = tid < C ? a.beta[((int64_t)bj * Tp + cc * C + tid) * H + hj] : 0.f;
  };
  if (blockIdx.x < total) load_chunk(blockIdx.x);
  for (int ci = blockIdx.x; ci < total; ci += gridDim.x) {
    const int bh = ci / NC, c = ci % NC;
    const int64_t bo = ((int64_t)bh * NC + c) * C * 64;
    {
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int idx = tid + n * NTH;
        sG[(idx >> 6) * LDP + (idx & 63)] = gv[n];
      }
      if (tid < C) sBeta[tid] = bt;
    }
    __syncthreads();
    {  // G = cumsum over rows (four 16-row segments, then the segment offsets)
      const int d = tid & 63, part = tid >> 6;
      float run = 0.f;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        run += sG[(16 * part + r) * LDP + d];
        sG[(16 * part + r) * LDP + d] = run;
      }
      __syncthreads();
      float off = 0.f;
      for (int p2 = 0; p2 < part; ++p2) off += sG[(16 * p2 + 15) * LDP + d];
      __syncthreads();
      if (part > 0) {
#pragma unroll
        for (int r = 0; r < 16; ++r) sG[(16 * part + r) * LDP + d] += off;
      }
    }
    __syncthreads();
    // operands, elementwise outputs and the solve's right-hand side [k e^G | v]; every load of the
    // chunk is issued before the first store, so the loads overlap instead of paying one
    // round trip per element group
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int idx = tid + n * NTH;
      const int i = idx >> 6, d = idx & 63;
      const float G = sG[i * LDP + d], r = sG[(i & ~15) * LDP + d], GC = sG[63 * LDP + d];
      const float kv = kr[n], qv = qr[n];
      const float e = expf(G - r);
      tcs::st(tQK, 128, i, d, kv * e);
      tcs::st(tQK, 128, 64 + i, d, qv * e);
#pragma unroll
      for (int I = 0; I < 4; ++I)
        tcs::st(tKd, 256, 64 * I + i, d, i <= 16 * I + 15 ? kv * expf(sG[16 * I * LDP + d] - G) : 0.f);
      const float eG = expf(G);
      a.buf.Qg[bo + idx] = qv * eG;
      a.buf.Kend[bo + idx] = kv * expf(GC - G);
      rhs[i * 128 + d] = kv * eG;
      rhs[i * 128 + 64 + d] = vr[n];
      if (i == 0) a.buf.eGC[((int64_t)bh * NC + c) * 64 + d] = expf(GC);
    }
    tcs::operands_ready();
    if (tid == 0) {
      tcs::mma_rows128(tm, tQK, 128, tKd, 256, 0, 256, 0, 64, false);
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 31);
    {  // row i: A (strict lower) from the k rows, P (lower) from the q rows; column block I(i)
      // tcgen05.ld takes one column address per warp: a warp's 32 rows span two 16-row tiles,
      // so load both column blocks and keep the one of this row's tile.
      const int i = row & 63, I = i >> 4, Ia = 2 * ((warp & 3) & 1);
      float val[32], alt[32];
      tcs::tmem_row32(tm, warp, 64 * Ia + c0, val);
      tcs::tmem_row32(tm, warp, 64 * (Ia + 1) + c0, alt);
      if (I != Ia) {
#pragma unroll
        for (int u = 0; u < 32; ++u) val[u] = alt[u];
      }
      float* dst = (row < 64 ? a.buf.Araw : a.buf.P) + bo + i * 64 + c0;
      const int lim = row < 64 ? i : i + 1;  // columns j < lim are kept
#pragma unroll
      for (int u = 0; u < 32; u += 4) {
        const int j = c0 + u;
        const float4 x = make_float4(j < lim ? val[u] : 0.f, j + 1 < lim ? val[u + 1] : 0.f,
                                     j + 2 < lim ? val[u + 2] : 0.f, j + 3 < lim ? val[u + 3] : 0.f);
        *reinterpret_cast<float4*>(dst + u) = x;
        if (row < 64) *reinterpret_cast<float4*>(sA + i * LDT + j) = x;
      }
    }
    __syncthreads();
    if (ci + (int)gridDim.x < total) load_chunk(ci + gridDim.x);  // lands during the solve
    // forward substitution: X_i = beta_i (R_i - sum_{j<i} A_ij X_j), 16-row blocks from the top
    if (tid < 128) {
      const int col = tid;
      float* wu = (col < 64 ? a.buf.W : a.buf.U) + bo + (col & 63);
      for (int I = 0; I < 4; ++I) {
        const int i0 = 16 * I;
        float xb[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) xb[u] = rhs[(i0 + u) * 128 + col];
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) {
#pragma unroll
          for (int jj = 0; jj < ii; ++jj) xb[ii] -= sA[(i0 + ii) * LDT + i0 + jj] * xb[jj];
          xb[ii] *= sBeta[i0 + ii];
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) wu[(i0 + u) * 64] = xb[u];
        for (int i = i0 + 16; i < 64; ++i) {
          const float4* ap = reinterpret_cast<const float4*>(sA + i * LDT + i0);
          float acc = rhs[i * 128 + col];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const float4 a4 = ap[q4];
            acc -= a4.x * xb[4 * q4] + a4.y * xb[4 * q4 + 1] + a4.z * xb[4 * q4 + 2] + a4.w * xb[4 * q4 + 3];
          }
          rhs[i * 128 + col] = acc;
        }
      }
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
  }
  if (warp == 0) tc::tmem_dealloc(tm, 256);
}

constexpr size_t kFwdSmem = 1024 + 128 * KB + (size_t)(C * LDP + C * LDT + C) * sizeof(float) + 16;

// ======================================================================== state passes
// Sequential over chunks; two (b, h) sequences per CTA stacked along M, so every product is an
// M = 128 MMA whose off-diagonal 64 x 64 blocks are ignored.  The state S (forward) or dS
// (backward) of a sequence lives in the registers of the TMEM row owners: thread (row kk of
// sequence s, column half) holds 32 entries.
//
// forward, per chunk:   V' = U - W S                       MMA-a  [W] x [S^T]^T
//                       O  = Qg S + P V'                   MMA-b  [Qg | P] x [S^T | V'^T]^T
//                       S <- diag(e^{G_C}) S + Kend^T V'   MMA-c  [Kend^T] x [V'^T]^T
// backward, per chunk:  dV' = P^T dO + Kend dS             MMA-a  [P^T | Kend] x [dO^T | dS^T]^T
//                       dS <- diag(e^{G_C}) dS + Qg^T dO - W^T dV'
//                                                          MMA-b  [Qg^T | -W^T] x [dO^T | dV'^T]^T
constexpr int ST_TILE = 64 * KB;  // R128 x K128 fp32 operand

struct StateArgs {
  KdaBuffers buf;
  const void* x;      // forward: h0 (fp32, may be null); backward: dout (T)
  const float* init;  // forward: h0; backward: dht (may be null)
  void* y;            // forward: o (T); backward: unused
  float* fin;         // forward: ht; backward: dh0 (may be null)
  float* dVp;         // backward outputs
  float* dSn;
  int B, Tp, H, NC;
  int* status;
};

// Forward pass: ONE sequence per CTA (grid = B * H), operand tiles of 64 rows (96 KB of shared
// memory, 256 TMEM columns), so two CTAs share an SM and every SM has work.  The M = 128 MMAs read
// 64 rows past each 64-row A tile (the next tile's memory); those accumulator lanes are ignored.
// Threads of warps 0, 1, 4, 5 own rows 0..63 (column halves); warps 2, 3, 6, 7 help with loads.
constexpr size_t kStateFwdSmem = 1024 + 96 * KB + 16;

template <typename T>
__global__ void __launch_bounds__(NTH, 2) kda_state_fwd_tc_kernel(const __grid_constant__ StateArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* tW = reinterpret_cast<float*>(base);                  // R64 K64  [W]
  float* tKT = reinterpret_cast<float*>(base + 16 * KB);       // R64 K64  [Kend^T]
  float* tQP = reinterpret_cast<float*>(base + 32 * KB);       // R64 K128 [Qg | P]
  float* tSV = reinterpret_cast<float*>(base + 64 * KB);       // R64 K128 [S^T | V'^T]
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + 96 * KB);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = (warp & 3) * 32 + (tid & 31), r = row & 63, half = warp >> 2, c0 = 32 * half;
  const int BH = a.B * a.H, NC = a.NC;
  const int my_bh = blockIdx.x;
  const bool valid = my_bh < BH;
  const bool mine = valid && row < 64;
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(slot, 256);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tm = *slot;
  uint32_t phase = 0;
  float S[32];
#pragma unroll
  for (int u = 0; u < 32; ++u)
    S[u] = (mine && a.init) ? a.init[(int64_t)my_bh * 4096 + r * 64 + c0 + u] : 0.f;
  const int b = valid ? my_bh / a.H : 0, h = valid ? my_bh % a.H : 0;
  for (int c = 0; c < NC; ++c) {
    const int64_t bo = ((int64_t)my_bh * NC + c) * 4096;
    // states[c] = S; S^T -> tSV[k 0..63]
    if (mine) {
      float* dst = a.buf.states + bo + r * 64 + c0;
#pragma unroll
      for (int u = 0; u < 32; u += 4) *reinterpret_cast<float4*>(dst + u) = make_float4(S[u], S[u + 1], S[u + 2], S[u + 3]);
#pragma unroll
      for (int u = 0; u < 32; ++u) tcs::st(tSV, 64, c0 + u, r, S[u]);
    }
    {  // W, Qg, P, Kend: 16 float4 loads in flight per thread, then the stores
      float4 ld[4][4];
      const float* srcs[4] = {a.buf.W + bo, a.buf.Qg + bo, a.buf.P + bo, a.buf.Kend + bo};
#pragma unroll
      for (int t4 = 0; t4 < 4; ++t4)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int idx = tid + n * NTH, rr = idx >> 4, cc = (idx & 15) * 4;
          ld[t4][n] = valid ? *reinterpret_cast<const float4*>(srcs[t4] + rr * 64 + cc) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int idx = tid + n * NTH, rr = idx >> 4, cc = (idx & 15) * 4;
        tcs::st4(tW, 64, rr, cc, ld[0][n]);
        tcs::st4(tQP, 64, rr, cc, ld[1][n]);
        tcs::st4(tQP, 64, rr, 64 + cc, ld[2][n]);
        const float4 kt = ld[3][n];  // Kend row rr, columns cc..cc+3 -> transposed rows
        tcs::st(tKT, 64, cc, rr, kt.x);
        tcs::st(tKT, 64, cc + 1, rr, kt.y);
        tcs::st(tKT, 64, cc + 2, rr, kt.z);
        tcs::st(tKT, 64, cc + 3, rr, kt.w);
      }
    }
    tcs::operands_ready();
    if (tid == 0) {
      tcs::mma_rows128(tm, tW, 64, tSV, 64, 0, 64, 0, 64, false);  // W S -> cols [0, 64)
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 21);
    {  // V' = U - W S  (row r)
      float val[32];
      float4 ur[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        ur[u] = mine ? *reinterpret_cast<const float4*>(a.buf.U + bo + r * 64 + c0 + 4 * u) : make_float4(0, 0, 0, 0);
      tcs::tmem_row32(tm, warp, c0, val);
      if (mine) {
#pragma unroll
        for (int u = 0; u < 32; u += 4) {
          const float4 uu = ur[u / 4];
          const float4 vp = make_float4(uu.x - val[u], uu.y - val[u + 1], uu.z - val[u + 2], uu.w - val[u + 3]);
          *reinterpret_cast<float4*>(a.buf.Vp + bo + r * 64 + c0 + u) = vp;
          tcs::st(tSV, 64, c0 + u, 64 + r, vp.x);
          tcs::st(tSV, 64, c0 + u + 1, 64 + r, vp.y);
          tcs::st(tSV, 64, c0 + u + 2, 64 + r, vp.z);
          tcs::st(tSV, 64, c0 + u + 3, 64 + r, vp.w);
        }
      }
    }
    tcs::operands_ready();
    if (tid == 0) {
      tcs::mma_rows128(tm + 64, tQP, 64, tSV, 64, 0, 64, 0, 128, false);           // Qg S + P V' -> [64, 128)
      tcs::mma_rows128_ab(tm + 128, tKT, 64, 0, tSV, 64, 0, 64, 64, 64, false);  // Kend^T V' -> [128, 192)
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 22);
    {
      float val[32];
      tcs::tmem_row32(tm + 64, warp, c0, val);
      if (mine) {
        T* o = reinterpret_cast<T*>(a.y) + (((int64_t)b * a.Tp + c * 64 + r) * a.H + h) * 64 + c0;
        if constexpr (sizeof(T) == 2) {
#pragma unroll
          for (int u = 0; u < 32; u += 8) {
            Vec<T> v8;
#pragma unroll
            for (int e = 0; e < 8; ++e) v8.set(e, val[u + e]);
            v8.store(o + u);
          }
        } else {
#pragma unroll
          for (int u = 0; u < 32; ++u) o[u] = from_f<T>(val[u]);
        }
      }
      tcs::tmem_row32(tm + 128, warp, c0, val);
      const float e = mine ? a.buf.eGC[((int64_t)my_bh * NC + c) * 64 + r] : 0.f;
#pragma unroll
      for (int u = 0; u < 32; ++u) S[u] = e * S[u] + val[u];
    }
  }
  if (mine && a.fin) {
    float* dst = a.fin + (int64_t)my_bh * 4096 + r * 64 + c0;
#pragma unroll
    for (int u = 0; u < 32; ++u) dst[u] = S[u];
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 0) tc::tmem_dealloc(tm, 256);
}

template <typename T>
__global__ void __launch_bounds__(NTH, 2) kda_state_bwd_tc_kernel(const __grid_constant__ StateArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* tA = reinterpret_cast<float*>(base);                // R64 K128 [P^T | Kend]   rows j
  float* tB = reinterpret_cast<float*>(base + 32 * KB);      // R64 K128 [dO^T | dS^T -> dV'^T]  rows v
  float* tC = reinterpret_cast<float*>(base + 64 * KB);      // R64 K128 [Qg^T | -W^T]  rows kk
  // 8 KB after tC: the M = 128 MMA over tC's last atom reads 64 rows past it
  uint64_t* bar = reinterpret_cast<uint64_t*>(base + 104 * KB);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row = (warp & 3) * 32 + (tid & 31), r = row & 63, half = warp >> 2, c0 = 32 * half;
  const int BH = a.B * a.H, NC = a.NC;
  const int my_bh = blockIdx.x;
  const bool valid = my_bh < BH;
  const bool mine = valid && row < 64;
  if (tid == 0) {
    tc::mbar_init(bar, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(slot, 128);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tm = *slot;
  uint32_t phase = 0;
  float dS[32];
#pragma unroll
  for (int u = 0; u < 32; ++u)
    dS[u] = (mine && a.init) ? a.init[(int64_t)my_bh * 4096 + r * 64 + c0 + u] : 0.f;
  const int64_t rs = (int64_t)a.H * 64;
  const T* dout = reinterpret_cast<const T*>(a.x);
  for (int c = NC - 1; c >= 0; --c) {
    if (mine) {
      float* dst = a.dSn + ((int64_t)my_bh * NC + c) * 4096 + r * 64 + c0;
#pragma unroll
      for (int u = 0; u < 32; u += 4)
        *reinterpret_cast<float4*>(dst + u) = make_float4(dS[u], dS[u + 1], dS[u + 2], dS[u + 3]);
    }
    if (mine) {
#pragma unroll
      for (int u = 0; u < 32; ++u) tcs::st(tB, 64, c0 + u, 64 + r, dS[u]);
    }
    {
      const int bh = my_bh;
      const int64_t bo = ((int64_t)bh * NC + c) * 4096;
      const int bb = valid ? bh / a.H : 0, hh = valid ? bh % a.H : 0;
      const T* dO = dout + (((int64_t)bb * a.Tp + c * 64) * a.H + hh) * 64;
      // the five operand tiles of this sequence: 20 loads in flight per thread, then the stores
      float4 ld[5][4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int idx = tid + n * NTH, rr = idx >> 4, cc = (idx & 15) * 4;
        const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
        ld[0][n] = valid ? *reinterpret_cast<const float4*>(a.buf.P + bo + rr * 64 + cc) : z;
        ld[1][n] = valid ? *reinterpret_cast<const float4*>(a.buf.Kend + bo + rr * 64 + cc) : z;
        if (valid) {
          const T* pd = dO + rr * rs + cc;
          ld[2][n] = make_float4(to_f<T>(pd[0]), to_f<T>(pd[1]), to_f<T>(pd[2]), to_f<T>(pd[3]));
        } else {
          ld[2][n] = z;
        }
        ld[3][n] = valid ? *reinterpret_cast<const float4*>(a.buf.Qg + bo + rr * 64 + cc) : z;
        ld[4][n] = valid ? *reinterpret_cast<const float4*>(a.buf.W + bo + rr * 64 + cc) : z;
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int idx = tid + n * NTH, rr = idx >> 4, cc = (idx & 15) * 4;
        tcs::st4(tA, 64, rr, 64 + cc, ld[1][n]);  // Kend
        const float vP[4] = {ld[0][n].x, ld[0][n].y, ld[0][n].z, ld[0][n].w};
        const float vD[4] = {ld[2][n].x, ld[2][n].y, ld[2][n].z, ld[2][n].w};
        const float vQ[4] = {ld[3][n].x, ld[3][n].y, ld[3][n].z, ld[3][n].w};
        const float vW[4] = {ld[4][n].x, ld[4][n].y, ld[4][n].z, ld[4][n].w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {  // transposed tiles: source column cc + u -> tile row
          tcs::st(tA, 64, cc + u, rr, vP[u]);
          tcs::st(tB, 64, cc + u, rr, vD[u]);
          tcs::st(tC, 64, cc + u, rr, vQ[u]);
          tcs::st(tC, 64, cc + u, 64 + rr, -vW[u]);
        }
      }
    }
    tcs::operands_ready();
    if (tid == 0) {
      tcs::mma_rows128(tm, tA, 64, tB, 64, 0, 64, 0, 128, false);  // dV' -> cols [0, 64)
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 23);
    const int64_t bo = ((int64_t)my_bh * NC + c) * 4096;
    {
      float val[32];
      tcs::tmem_row32(tm, warp, c0, val);
      if (mine) {
        float* dst = a.dVp + bo + r * 64 + c0;
#pragma unroll
        for (int u = 0; u < 32; u += 4)
          *reinterpret_cast<float4*>(dst + u) = make_float4(val[u], val[u + 1], val[u + 2], val[u + 3]);
      }
#pragma unroll
      for (int u = 0; u < 32; ++u)
        if (mine) tcs::st(tB, 64, c0 + u, 64 + r, val[u]);  // dV'^T
    }
    tcs::operands_ready();
    if (tid == 0) {
      tcs::mma_rows128(tm + 64, tC, 64, tB, 64, 0, 64, 0, 128, false);  // Qg^T dO - W^T dV'
      tc::mma_commit(bar);
    }
    tcs::mma_done(bar, phase, a.status, 24);
    {
      float val[32];
      tcs::tmem_row32(tm + 64, warp, c0, val);
      const float e = mine ? a.buf.eGC[((int64_t)my_bh * NC + c) * 64 + r] : 0.f;
#pragma unroll
      for (int u = 0; u < 32; ++u) dS[u] = e * dS[u] + val[u];
    }
  }
  if (mine && a.fin) {
    float* dst = a.fin + (int64_t)my_bh * 4096 + r * 64 + c0;
#pragma unroll
    for (int u = 0; u < 32; ++u) dst[u] = dS[u];
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 0) tc::tmem_dealloc(tm, 128);
}

constexpr size_t kStateSmem = 1024 + 104 * KB + 16;  // backward: three R64 K128 tiles + 8 KB of read-past room

template <typename T>
cudaError_t launch_state(bool fwd, const StateArgs& args, cudaStream_t s) {
  cudaError_t e = ensure_dynamic_smem(kda_state_fwd_tc_kernel<T>, (int)kStateFwdSmem);
  if (e == cudaSuccess) e = ensure_dynamic_smem(kda_state_bwd_tc_kernel<T>, (int)kStateSmem);
  if (e != cudaSuccess) return e;
  if (fwd)
    kda_state_fwd_tc_kernel<T><<<args.B * args.H, NTH, kStateFwdSmem, s>>>(args);
  else
    kda_state_bwd_tc_kernel<T><<<args.B * args.H, NTH, kStateSmem, s>>>(args);
  return cudaGetLastError();
}

int* status_ptr(int* status);

__device__ int g_kda_tc_status = 0;

std::mutex g_status_mutex;
int* g_status_addr[64] = {};  // device address of g_kda_tc_status, per device

int* status_ptr(int* status) {
  if (status) return status;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (!g_status_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_kda_tc_status) != cudaSuccess) return nullptr;
    g_status_addr[dev] = static_cast<int*>(p);
  }
  return g_status_addr[dev];
}

}  // namespace

std::vector<long long> kda_phase_profile(bool enable) {
  std::vector<long long> v(16, 0);
  cudaMemcpyFromSymbol(v.data(), g_kda_phase, sizeof(long long) * 16);
  const int on = enable ? 1 : 0;
  cudaMemcpyToSymbol(g_kda_phase_on, &on, sizeof(int));
  return v;
}

int* kda_tc_default_status() { return status_ptr(nullptr); }

int kda_tc_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_kda_tc_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_kda_tc_status, &zero, sizeof(int));
  }
  return v;
}

cudaError_t kda_intra_bwd_tc(int dtype, const void* q, const void* k, const void* v, const float* g,
                             const float* beta, KdaBuffers buf, const float* araw, const void* dout, const float* dVp,
                             const float* dSn, float* dq, float* dk, float* dv, float* dg, float* dbeta, int B,
                             int Tp, int H, int* status, cudaStream_t s) {
  if (Tp % C || !araw) return cudaErrorInvalidValue;
  status = status_ptr(status);
  if (!status) return cudaErrorInvalidValue;
  BwdArgs args{q, k, v, g, beta, dout, buf.W, buf.U, buf.states, buf.Vp, araw, dVp, dSn,
               dq, dk, dv, dg, dbeta, B, Tp, H, Tp / C, status};
  switch (dtype) {
    case 0: return launch_bwd<float>(args, s);
    case 1: return launch_bwd<__nv_bfloat16>(args, s);
    case 2: return launch_bwd<__half>(args, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace kimi

namespace kimi {

cudaError_t kda_state_fwd_tc(int dtype, KdaBuffers buf, const float* h0, void* o, float* ht, int B, int Tp, int H,
                             int* status, cudaStream_t s) {
  if (Tp % C) return cudaErrorInvalidValue;
  status = status_ptr(status);
  if (!status) return cudaErrorInvalidValue;
  StateArgs args{buf, nullptr, h0, o, ht, nullptr, nullptr, B, Tp, H, Tp / C, status};
  switch (dtype) {
    case 0: return launch_state<float>(true, args, s);
    case 1: return launch_state<__nv_bfloat16>(true, args, s);
    case 2: return launch_state<__half>(true, args, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t kda_state_bwd_tc(int dtype, KdaBuffers buf, const void* dout, const float* dht, float* dVp, float* dSn,
                             float* dh0, int B, int Tp, int H, int* status, cudaStream_t s) {
  if (Tp % C) return cudaErrorInvalidValue;
  status = status_ptr(status);
  if (!status) return cudaErrorInvalidValue;
  StateArgs args{buf, dout, dht, nullptr, dh0, dVp, dSn, B, Tp, H, Tp / C, status};
  switch (dtype) {
    case 0: return launch_state<float>(false, args, s);
    case 1: return launch_state<__nv_bfloat16>(false, args, s);
    case 2: return launch_state<__half>(false, args, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace kimi

namespace kimi {

cudaError_t kda_intra_fwd_tc(int dtype, const void* q, const void* k, const void* v, const float* g,
                             const float* beta, KdaBuffers buf, int B, int Tp, int H, int* status, cudaStream_t s) {
  if (Tp % C || !buf.Araw) return cudaErrorInvalidValue;
  status = status_ptr(status);
  if (!status) return cudaErrorInvalidValue;
  FwdArgs args{q, k, v, g, beta, buf, B, Tp, H, Tp / C, status};
  const int total = B * H * (Tp / C);
  const int sms = device_sms();
  const int grid = total < sms ? total : sms;
  auto go = [&](auto kernel) -> cudaError_t {
    cudaError_t e = ensure_dynamic_smem(kernel, (int)kFwdSmem);
    if (e != cudaSuccess) return e;
    kernel<<<grid, NTH, kFwdSmem, s>>>(args);
    return cudaGetLastError();
  };
  switch (dtype) {
    case 0: return go(kda_intra_fwd_tc_kernel<float>);
    case 1: return go(kda_intra_fwd_tc_kernel<__nv_bfloat16>);
    case 2: return go(kda_intra_fwd_tc_kernel<__half>);
  }
  return cudaErrorInvalidValue;
}

}  // namespace kimi
