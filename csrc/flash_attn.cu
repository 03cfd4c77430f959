// Flash attention forward / backward for head dim 64 (bf16 / fp16 in, fp32 accumulation).
//
// Tiles of 64 queries x 64 keys; 4 warps per block, each warp owning 16 rows of every
// 64x64 product. Operand fragments are loaded with ldmatrix (transposed where the smem
// layout is K-major) and multiplied with mma.sync m16n8k16; the running softmax uses the
// log-sum-exp (natural log) which is saved for the backward pass. Causal masking and
// per-batch key lengths (padding) are applied on the score tile. Q, K, V, O are
// [B, T, H, 64]; LSE is [B, H, T].
#include "common.cuh"
#include "device_info.h"
#include "kernels.h"

namespace kimi {
namespace {

constexpr int HD = 64;     // head dim
constexpr int BM = 64;     // query tile
constexpr int BN = 64;     // key tile
constexpr int LDS = 72;    // padded smem row (elements): 144 B rows keep ldmatrix conflict-free
constexpr int NTH = 128;   // 4 warps

template <typename T> struct MmaType;
template <> struct MmaType<__nv_bfloat16> { static constexpr bool bf16 = true; };
template <> struct MmaType<__half> { static constexpr bool bf16 = false; };

KIMI_D uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

KIMI_D void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
KIMI_D void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

template <bool BF16>
KIMI_D void mma16816(float* c, const uint32_t* a, const uint32_t* b) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
}

// acc[n][4] += A(16 x 64) * B(64 x 64) for one warp.
//   A_T = false: A stored [m][k] (row stride LDS);  true: stored [k][m].
//   B_T = false: B stored [n][k];                    true: stored [k][n].
template <typename T, bool A_T, bool B_T>
KIMI_D void warp_gemm_16x64(float (*acc)[4], const T* A, const T* B) {
  const int lane = threadIdx.x & 31;
  const int j = lane >> 3, r = lane & 7;
#pragma unroll
  for (int k0 = 0; k0 < HD; k0 += 16) {
    uint32_t a[4];
    if (!A_T) {
      const T* p = A + (r + (j & 1) * 8) * LDS + k0 + (j >> 1) * 8;
      ldsm_x4(smem_u32(p), a[0], a[1], a[2], a[3]);
    } else {
      const T* p = A + (k0 + r + (j >> 1) * 8) * LDS + (j & 1) * 8;
      ldsm_x4_t(smem_u32(p), a[0], a[1], a[2], a[3]);
    }
#pragma unroll
    for (int n0 = 0; n0 < 64; n0 += 16) {
      uint32_t b[4];
      if (!B_T) {
        const T* p = B + (n0 + r + (j >> 1) * 8) * LDS + k0 + (j & 1) * 8;
        ldsm_x4(smem_u32(p), b[0], b[1], b[2], b[3]);
      } else {
        const T* p = B + (k0 + r + (j & 1) * 8) * LDS + n0 + (j >> 1) * 8;
        ldsm_x4_t(smem_u32(p), b[0], b[1], b[2], b[3]);
      }
      mma16816<MmaType<T>::bf16>(acc[n0 / 8], a, b);
      mma16816<MmaType<T>::bf16>(acc[n0 / 8 + 1], a, b + 2);
    }
  }
}

// Copy a [rows x 64] tile (row stride `ld` elements in global) into smem, zero-filling rows >= valid.
template <typename T>
KIMI_D void load_tile(T* s, const T* g, int64_t ld, int valid) {
  for (int idx = threadIdx.x; idx < 64 * 8; idx += blockDim.x) {
    const int row = idx >> 3, ch = idx & 7;
    int4 v = make_int4(0, 0, 0, 0);
    if (row < valid) v = *reinterpret_cast<const int4*>(g + row * ld + ch * 8);
    *reinterpret_cast<int4*>(s + row * LDS + ch * 8) = v;
  }
}

// The same copy with cp.async (16-byte units, zero-filled rows >= valid); the caller commits and waits.
template <typename T>
KIMI_D void load_tile_async(T* s, const T* g, int64_t ld, int valid) {
  for (int idx = threadIdx.x; idx < 64 * 8; idx += blockDim.x) {
    const int row = idx >> 3, ch = idx & 7;
    const bool ok = row < valid;
    const uint32_t dst = smem_u32(s + row * LDS + ch * 8);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(ok ? g + row * ld + ch * 8 : g),
                 "r"(ok ? 16 : 0)
                 : "memory");
  }
}
KIMI_D void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
KIMI_D void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Accumulator element (n-tile nt, reg e) -> (row, col) inside the warp's 16 x 64 tile.
KIMI_D int acc_row(int e) { return ((threadIdx.x & 31) >> 2) + (e >= 2 ? 8 : 0); }
KIMI_D int acc_col(int nt, int e) { return nt * 8 + ((threadIdx.x & 3) << 1) + (e & 1); }

template <typename T>
__global__ void __launch_bounds__(NTH) fa_fwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                     const T* __restrict__ v, T* __restrict__ o,
                                                     float* __restrict__ lse, int tq, int tk, int H, bool causal,
                                                     const int* __restrict__ key_lengths, float scale) {
  // K / V tiles are double-buffered: the next tile streams in (cp.async) while this one is used
  extern __shared__ __align__(16) uint8_t fa_smem[];
  T* sQ = reinterpret_cast<T*>(fa_smem);
  T* sP = sQ + BM * LDS;
  T* sKV = sP + BM * LDS;  // [2 buffers][K | V][BN * LDS]
  const int mt = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5;
  const int q0 = mt * BM;
  const int64_t ld = (int64_t)H * HD;
  const T* qb = q + ((int64_t)b * tq * H + h) * HD;
  const T* kb = k + ((int64_t)b * tk * H + h) * HD;
  const T* vb = v + ((int64_t)b * tk * H + h) * HD;
  const int klen = key_lengths ? key_lengths[b] : tk;
  load_tile(sQ, qb + q0 * ld, ld, min(BM, tq - q0));
  float accO[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) accO[n][e] = 0.f;
  float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.f, 0.f};
  const float sl2 = scale * 1.4426950408889634f;  // log2(e) * scale
  int kend = klen;
  if (causal) kend = min(kend, q0 + BM + (tk - tq));
  if (kend > 0) {
    load_tile_async(sKV, kb, ld, min(BN, tk));
    load_tile_async(sKV + BN * LDS, vb, ld, min(BN, tk));
    cp_async_commit();
  }
  int buf = 0;
  for (int k0 = 0; k0 < kend; k0 += BN) {
    __syncthreads();  // every warp is done with the other buffer (the previous tile)
    if (k0 + BN < kend) {
      T* nxt = sKV + (buf ^ 1) * 2 * BN * LDS;
      load_tile_async(nxt, kb + (k0 + BN) * ld, ld, min(BN, tk - k0 - BN));
      load_tile_async(nxt + BN * LDS, vb + (k0 + BN) * ld, ld, min(BN, tk - k0 - BN));
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // this tile landed for every thread
    const T* sK = sKV + buf * 2 * BN * LDS;
    const T* sV = sK + BN * LDS;
    buf ^= 1;
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = 0.f;
    warp_gemm_16x64<T, false, false>(s, sQ + warp * 16 * LDS, sK);
    float rmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = q0 + warp * 16 + acc_row(e), kj = k0 + acc_col(n, e);
        bool ok = kj < klen;
        if (causal) ok = ok && kj <= qi + (tk - tq);
        s[n][e] = ok ? s[n][e] * sl2 : -INFINITY;
        rmax[e >> 1] = fmaxf(rmax[e >> 1], s[n][e]);
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      rmax[hh] = fmaxf(rmax[hh], __shfl_xor_sync(0xffffffffu, rmax[hh], 1));
      rmax[hh] = fmaxf(rmax[hh], __shfl_xor_sync(0xffffffffu, rmax[hh], 2));
    }
    float alpha[2], mnew[2], rsum[2] = {0.f, 0.f};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mnew[hh] = fmaxf(m_i[hh], rmax[hh]);
      alpha[hh] = (mnew[hh] == -INFINITY) ? 1.f : exp2f(m_i[hh] - mnew[hh]);
      m_i[hh] = mnew[hh];
    }
    T* pw = sP + warp * 16 * LDS;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hh = e >> 1;
        const float p = (mnew[hh] == -INFINITY) ? 0.f : exp2f(s[n][e] - mnew[hh]);
        const T pt = from_f<T>(p);
        rsum[hh] += to_f<T>(pt);
        pw[acc_row(e) * LDS + acc_col(n, e)] = pt;
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      rsum[hh] += __shfl_xor_sync(0xffffffffu, rsum[hh], 1);
      rsum[hh] += __shfl_xor_sync(0xffffffffu, rsum[hh], 2);
      l_i[hh] = l_i[hh] * alpha[hh] + rsum[hh];
    }
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) accO[n][e] *= alpha[e >> 1];
    __syncwarp();
    warp_gemm_16x64<T, false, true>(accO, pw, sV);
  }
  // epilogue
  const float ln2 = 0.6931471805599453f;
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int hh = e >> 1;
      const int qi = q0 + warp * 16 + acc_row(e);
      if (qi < tq) {
        const float inv = l_i[hh] > 0.f ? 1.f / l_i[hh] : 0.f;
        o[((int64_t)b * tq + qi) * ld + h * HD + acc_col(n, e)] = from_f<T>(accO[n][e] * inv);
      }
    }
  if ((threadIdx.x & 3) == 0) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int qi = q0 + warp * 16 + ((threadIdx.x & 31) >> 2) + hh * 8;
      if (qi < tq)
        lse[(int64_t)bh * tq + qi] = l_i[hh] > 0.f ? (m_i[hh] + log2f(l_i[hh])) * ln2 : -INFINITY;
    }
  }
}

// delta[b,h,i] = sum_d dO[i,d] * O[i,d]
template <typename T>
__global__ void fa_delta_kernel(const T* __restrict__ o, const T* __restrict__ dout, float* __restrict__ delta,
                                int B, int tq, int H) {
  const int64_t rows = (int64_t)B * tq * H;
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < rows;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const T* orow = o + r * HD;
    const T* drow = dout + r * HD;
    float acc = to_f<T>(orow[lane]) * to_f<T>(drow[lane]) + to_f<T>(orow[lane + 32]) * to_f<T>(drow[lane + 32]);
    acc = warp_sum(acc);
    if (lane == 0) {
      const int h = (int)(r % H);
      const int64_t bt = r / H;
      const int b = (int)(bt / tq), t = (int)(bt % tq);
      delta[((int64_t)b * H + h) * tq + t] = acc;
    }
  }
}

// One block per 64-key tile; loops over the query tiles that can see it.
template <typename T>
__global__ void __launch_bounds__(NTH) fa_bwd_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                     const T* __restrict__ v, const T* __restrict__ dout,
                                                     const float* __restrict__ lse, const float* __restrict__ delta,
                                                     float* __restrict__ dq_acc, T* __restrict__ dk,
                                                     T* __restrict__ dv, int tq, int tk, int H, bool causal,
                                                     const int* __restrict__ key_lengths, float scale) {
  extern __shared__ __align__(16) unsigned char smraw[];
  T* sQ = reinterpret_cast<T*>(smraw);
  T* sdO = sQ + BM * LDS;
  T* sK = sdO + BM * LDS;
  T* sV = sK + BN * LDS;
  T* sP = sV + BN * LDS;
  T* sdS = sP + BM * LDS;
  const int nt = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int warp = threadIdx.x >> 5;
  const int k0 = nt * BN;
  const int64_t ld = (int64_t)H * HD;
  const int klen = key_lengths ? key_lengths[b] : tk;
  const T* qb = q + ((int64_t)b * tq * H + h) * HD;
  const T* kb = k + ((int64_t)b * tk * H + h) * HD;
  const T* vb = v + ((int64_t)b * tk * H + h) * HD;
  const T* dob = dout + ((int64_t)b * tq * H + h) * HD;
  load_tile(sK, kb + k0 * ld, ld, min(BN, tk - k0));
  load_tile(sV, vb + k0 * ld, ld, min(BN, tk - k0));
  float accdK[8][4], accdV[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) accdK[n][e] = accdV[n][e] = 0.f;
  int qstart = 0;
  if (causal) qstart = max(0, (k0 - (tk - tq)) / BM * BM);
  const bool any_keys = k0 < klen;
  for (int q0 = any_keys ? qstart : tq; q0 < tq; q0 += BM) {
    __syncthreads();
    load_tile(sQ, qb + q0 * ld, ld, min(BM, tq - q0));
    load_tile(sdO, dob + q0 * ld, ld, min(BM, tq - q0));
    __syncthreads();
    float s[8][4], dp[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[n][e] = dp[n][e] = 0.f;
    warp_gemm_16x64<T, false, false>(s, sQ + warp * 16 * LDS, sK);
    warp_gemm_16x64<T, false, false>(dp, sdO + warp * 16 * LDS, sV);
    T* pw = sP + warp * 16 * LDS;
    T* dsw = sdS + warp * 16 * LDS;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ri = acc_row(e), cj = acc_col(n, e);
        const int qi = q0 + warp * 16 + ri, kj = k0 + cj;
        bool ok = qi < tq && kj < klen && kj < tk;
        if (causal) ok = ok && kj <= qi + (tk - tq);
        float p = 0.f, ds = 0.f;
        if (ok) {
          const float l = lse[(int64_t)bh * tq + qi];
          p = expf(s[n][e] * scale - l);
          ds = p * (dp[n][e] - delta[(int64_t)bh * tq + qi]);
        }
        pw[ri * LDS + cj] = from_f<T>(p);
        dsw[ri * LDS + cj] = from_f<T>(ds);
      }
    __syncthreads();
    // dV += P^T dO ; dK += dS^T Q  (this warp owns key rows warp*16 .. +15)
    warp_gemm_16x64<T, true, true>(accdV, sP + warp * 16, sdO);
    warp_gemm_16x64<T, true, true>(accdK, sdS + warp * 16, sQ);
    // dQ += dS K  (this warp owns query rows warp*16 .. +15)
    float accdQ[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) accdQ[n][e] = 0.f;
    warp_gemm_16x64<T, false, true>(accdQ, sdS + warp * 16 * LDS, sK);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qi = q0 + warp * 16 + acc_row(e);
        if (qi < tq) atomicAdd(&dq_acc[((int64_t)b * tq + qi) * ld + h * HD + acc_col(n, e)], accdQ[n][e] * scale);
      }
  }
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int kj = k0 + warp * 16 + acc_row(e);
      if (kj < tk) {
        const int64_t off = ((int64_t)b * tk + kj) * ld + h * HD + acc_col(n, e);
        dk[off] = from_f<T>(accdK[n][e] * scale);
        dv[off] = from_f<T>(accdV[n][e]);
      }
    }
}

template <typename T>
cudaError_t fwd_impl(const void* q, const void* k, const void* v, void* o, float* lse, int B, int tq, int tk, int H,
                     bool causal, const int* kl, float scale, cudaStream_t s) {
  dim3 grid((tq + BM - 1) / BM, B * H);
  const size_t smem = (size_t)6 * 64 * LDS * sizeof(T);  // Q, P and two K / V pairs
  KIMI_CUDA_CHECK(ensure_dynamic_smem(fa_fwd_kernel<T>, (int)smem));
  fa_fwd_kernel<T><<<grid, NTH, smem, s>>>((const T*)q, (const T*)k, (const T*)v, (T*)o, lse, tq, tk, H, causal, kl,
                                           scale);
  return cudaGetLastError();
}

template <typename T>
cudaError_t bwd_impl(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
                     float* dq_acc, void* dk, void* dv, float* delta, int B, int tq, int tk, int H, bool causal,
                     const int* kl, float scale, cudaStream_t s) {
  fa_delta_kernel<T><<<device_sms() * 4, 256, 0, s>>>((const T*)o, (const T*)dout, delta, B, tq, H);
  KIMI_CUDA_CHECK(cudaGetLastError());
  const size_t smem = (size_t)6 * 64 * LDS * sizeof(T);
  KIMI_CUDA_CHECK(ensure_dynamic_smem(fa_bwd_kernel<T>, (int)smem));
  dim3 grid((tk + BN - 1) / BN, B * H);
  fa_bwd_kernel<T><<<grid, NTH, smem, s>>>((const T*)q, (const T*)k, (const T*)v, (const T*)dout, lse, delta, dq_acc,
                                           (T*)dk, (T*)dv, tq, tk, H, causal, kl, scale);
  return cudaGetLastError();
}

}  // namespace

cudaError_t flash_attn_fwd(int dtype, const void* q, const void* k, const void* v, void* o, float* lse, int B, int tq,
                           int tk, int H, int dqk, int dvd, bool causal, const int* kl, float scale, cudaStream_t s) {
  if (dqk != HD || dvd != HD) return cudaErrorInvalidValue;
  switch (dtype) {
    case 1: return fwd_impl<__nv_bfloat16>(q, k, v, o, lse, B, tq, tk, H, causal, kl, scale, s);
    case 2: return fwd_impl<__half>(q, k, v, o, lse, B, tq, tk, H, causal, kl, scale, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t flash_attn_bwd(int dtype, const void* q, const void* k, const void* v, const void* o, const void* dout,
                           const float* lse, float* dq_acc, void* dk, void* dv, float* delta, int B, int tq, int tk,
                           int H, int dqk, int dvd, bool causal, const int* kl, float scale, cudaStream_t s) {
  if (dqk != HD || dvd != HD) return cudaErrorInvalidValue;
  switch (dtype) {
    case 1: return bwd_impl<__nv_bfloat16>(q, k, v, o, dout, lse, dq_acc, dk, dv, delta, B, tq, tk, H, causal, kl,
                                           scale, s);
    case 2: return bwd_impl<__half>(q, k, v, o, dout, lse, dq_acc, dk, dv, delta, B, tq, tk, H, causal, kl, scale, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace kimi
