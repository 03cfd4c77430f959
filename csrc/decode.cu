// Decode-step kernels (one new token per sequence) for serving.
//
//   conv_step    causal depthwise short conv over [history, x_t] + SiLU (+ per-head L2 norm) for up
//                to three streams (q, k, v) in one launch; the [B, K-1, C] history is shifted in place.
//                Parity: `src/kda/short_conv.py:85-90` with a cached state (reference).
//   kda_decode   one recurrent KDA token per (batch, head): S <- diag(e^g) S; S += beta k (v - S^T k)^T;
//                o = S^T q, fp32 state [B, H, 64, 64] updated in place or into a second buffer.
//                Parity: `src/kda/recurrent.py:62-74` (reference).
//   mla_decode   weight-absorbed MLA attention of one query per head over the latent cache
//                [B, Tmax, L] with per-row valid lengths: split-T flash decoding (running max and sum
//                per head, partial contexts combined by a second kernel).  The latent rows cross
//                HBM once for all heads.  Parity: the decode path of `src/mla/gated_mla.py:123-124`
//                (reference) without the K/V re-expansion.
//   sample       fused next-token selection per row: repetition penalty (seen-token bitmap),
//                NaN-safe greedy argmax, temperature, top-k (radix select of the k-th largest key),
//                top-p (radix select of the nucleus boundary on probability mass), and a draw from
//                the kept distribution with a counter-based Philox4x32-10 generator (Salmon, Moraes,
//                Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC 2011) keyed by a
//                device seed and step counter, so CUDA-graph replays draw fresh numbers.
//                Parity: `inference/sampling.py:10-91` (reference); ties at the top-k / top-p
//                boundary are all kept (the reference's sort order decides among them).
#include <cstdint>

#include "common.cuh"
#include "device_info.h"
#include "kernels.h"

namespace kimi {
namespace {

// ---------------------------------------------------------------- short conv, one token
template <typename T>
KIMI_D void ld8(const T* p, float* o) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  } else {
    Vec<T> v;
    v.load(p);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = v.f(e);
  }
}
template <typename T>
KIMI_D void st8(T* p, const float* in) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(in[0], in[1], in[2], in[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(in[4], in[5], in[6], in[7]);
  } else {
    Vec<T> v;
#pragma unroll
    for (int e = 0; e < 8; ++e) v.set(e, in[e]);
    v.store(p);
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(256) conv_step_kernel(ConvStepArgs a, float eps) {
  const int s = blockIdx.z, b = blockIdx.y;
  const int channels = a.channels[s];
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const bool active = c0 < channels;
  const int cc = active ? c0 : 0;
  const T* x = static_cast<const T*>(a.x[s]) + (int64_t)b * channels;
  T* hist = static_cast<T*>(a.hist[s]) + (int64_t)b * (K - 1) * channels;
  const float* w = a.w[s];
  float xv[8], h[K > 1 ? K - 1 : 1][8], out[8], ss = 0.f;
  ld8<T>(x + cc, xv);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) ld8<T>(hist + (int64_t)j * channels + cc, h[j]);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float* wc = w + (int64_t)(cc + e) * K;
    float pre = (a.bias[s] != nullptr ? a.bias[s][cc + e] : 0.f) + wc[0] * xv[e];
    // history row j holds x[t - (K - 1 - j)], which weight column K - 1 - j multiplies
#pragma unroll
    for (int j = 0; j < K - 1; ++j) pre += wc[K - 1 - j] * h[j][e];
    out[e] = siluf_(pre);
    ss += out[e] * out[e];
  }
  if (a.head_lanes[s] > 0) {  // whole heads live in aligned lane groups of one warp
    ss = group_sum(active ? ss : 0.f, a.head_lanes[s]);
    const float inv = 1.f / fmaxf(sqrtf(ss), eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] *= inv;
  }
  if (!active) return;
  st8<T>(static_cast<T*>(a.y[s]) + (int64_t)b * channels + cc, out);
#pragma unroll
  for (int j = 0; j + 1 < K - 1; ++j) st8<T>(hist + (int64_t)j * channels + cc, h[j + 1]);
  if constexpr (K > 1) st8<T>(hist + (int64_t)(K - 2) * channels + cc, xv);
}

// ---------------------------------------------------------------- KDA recurrent token
// Thread (group, col): state rows group*16 .. +16 of column col; the two reductions over the key
// axis (S^T k and S^T q) combine the four row groups through shared memory.
template <typename T>
__global__ void __launch_bounds__(256) kda_decode_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                         const T* __restrict__ v, const float* __restrict__ g,
                                                         const float* __restrict__ beta, const float* state_in,
                                                         float* state_out, T* __restrict__ o, int heads) {
  __shared__ float sq[64], sk[64], sv[64], sdec[64], red[4][64];
  const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int64_t bh = (int64_t)b * heads + h;
  if (tid < 64) {
    sq[tid] = to_f<T>(q[bh * 64 + tid]);
    sk[tid] = to_f<T>(k[bh * 64 + tid]);
    sv[tid] = to_f<T>(v[bh * 64 + tid]);
    sdec[tid] = expf(g[bh * 64 + tid]);
  }
  __syncthreads();
  const int col = tid & 63, grp = tid >> 6;
  const float* S = state_in + bh * 4096;
  float s[16], part = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int r = grp * 16 + i;
    s[i] = S[r * 64 + col] * sdec[r];
    part += s[i] * sk[r];
  }
  red[grp][col] = part;
  __syncthreads();
  const float err = sv[col] - (red[0][col] + red[1][col] + red[2][col] + red[3][col]);
  const float bt = beta[bh];
  __syncthreads();
  part = 0.f;
  float* D = state_out + bh * 4096;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int r = grp * 16 + i;
    s[i] += bt * sk[r] * err;
    part += s[i] * sq[r];
    D[r * 64 + col] = s[i];
  }
  red[grp][col] = part;
  __syncthreads();
  if (grp == 0) o[bh * 64 + col] = from_f<T>(red[0][col] + red[1][col] + red[2][col] + red[3][col]);
}

// ---------------------------------------------------------------- MLA latent flash decode
// CTA (split, b): rows [split * rows_per_split, ...) of sequence b, in sub-chunks of ROWS rows kept
// in shared memory in the cache's own dtype (the chunk is read from HBM once, 16-byte vectors).
// Scores: each warp takes ROWS / 8 rows; a lane accumulates the dot products of its latent columns
// for every head and the warp reduces.  Context: thread owns latent columns tid, tid + 256, ... (CPT
// of them) and keeps one running accumulator per (head, column).  Instances: HMAX heads padded to
// 4 / 8 / 16 / 32, CPT = ceil(L / 256) rounded to 2 / 4 / 6 / 8, ROWS 32 (L <= 1024) or 16.
constexpr int kMlaThreads = 256;

// Two adjacent elements as floats (one 4- or 8-byte shared-memory load).
KIMI_D float2 mla_pair(const float* p) { return *reinterpret_cast<const float2*>(p); }
KIMI_D float2 mla_pair(const __nv_bfloat16* p) { return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p)); }
KIMI_D float2 mla_pair(const __half* p) { return __half22float2(*reinterpret_cast<const __half2*>(p)); }

template <typename T, int HMAX, int CPT, int ROWS>
__global__ void __launch_bounds__(kMlaThreads) mla_decode_kernel(const float* __restrict__ qlat,
                                                                 const T* __restrict__ latent,
                                                                 const int32_t* __restrict__ lengths, int heads,
                                                                 int ldim, int64_t tmax, int rows_per_split,
                                                                 float* __restrict__ part_acc,
                                                                 float* __restrict__ part_ml) {
  constexpr int RPW = ROWS / 8;  // rows per warp in the score phase
  static_assert(ROWS <= 32 && ROWS % 8 == 0, "one lane per chunk row in the softmax phase");
  extern __shared__ __align__(16) float smem[];
  float* sq = smem;                                            // [heads][ldim] fp32
  T* sx = reinterpret_cast<T*>(sq + heads * ldim);            // [ROWS][ldim] cache dtype
  float* sp = reinterpret_cast<float*>(sx + ROWS * ldim);     // [ROWS][HMAX] scores, then weights
  float* sstat = sp + ROWS * HMAX;                             // [HMAX] running max, [HMAX] sum, [HMAX] scale
  const int split = blockIdx.x, b = blockIdx.y, nsplit = gridDim.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = (int)min((int64_t)lengths[b], tmax);
  const int r0 = split * rows_per_split, r1 = min(r0 + rows_per_split, len);
  {  // 16-byte loads, several in flight per thread (ldim % 8 == 0)
    const float4* src = reinterpret_cast<const float4*>(qlat + (int64_t)b * heads * ldim);
    float4* dst = reinterpret_cast<float4*>(sq);
    const int n4 = heads * ldim / 4;
#pragma unroll 4
    for (int i = tid; i < n4; i += kMlaThreads) dst[i] = src[i];
  }
  if (tid < HMAX) {
    sstat[tid] = -INFINITY;
    sstat[HMAX + tid] = 0.f;
  }
  float acc[CPT][HMAX];
#pragma unroll
  for (int c = 0; c < CPT; ++c)
#pragma unroll
    for (int h = 0; h < HMAX; ++h) acc[c][h] = 0.f;
  const T* xb = latent + (int64_t)b * tmax * ldim;
  for (int c0 = r0; c0 < r1; c0 += ROWS) {
    const int nr = min(ROWS, r1 - c0);
    __syncthreads();  // previous sub-chunk fully consumed
    {
      const int4* src = reinterpret_cast<const int4*>(xb + (int64_t)c0 * ldim);
      int4* dst = reinterpret_cast<int4*>(sx);
      const int nv = nr * ldim * (int)sizeof(T) / 16;
#pragma unroll 4
      for (int i = tid; i < nv; i += kMlaThreads) dst[i] = src[i];
    }
    __syncthreads();
    {
      float dot[RPW][HMAX];
#pragma unroll
      for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int h = 0; h < HMAX; ++h) dot[r][h] = 0.f;
      const int rb = warp * RPW;
      for (int l = 2 * lane; l < ldim; l += 64) {  // two adjacent columns per lane (ldim is even)
        float2 xv[RPW];
#pragma unroll
        for (int r = 0; r < RPW; ++r) xv[r] = rb + r < nr ? mla_pair(sx + (rb + r) * ldim + l) : make_float2(0.f, 0.f);
#pragma unroll
        for (int h = 0; h < HMAX; ++h) {
          if (h < heads) {
            const float2 qv = *reinterpret_cast<const float2*>(sq + h * ldim + l);
#pragma unroll
            for (int r = 0; r < RPW; ++r) dot[r][h] += qv.x * xv[r].x + qv.y * xv[r].y;
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RPW; ++r)
#pragma unroll
        for (int h = 0; h < HMAX; ++h) {
          const float d = warp_sum(dot[r][h]);
          if (lane == 0 && h < heads) sp[(rb + r) * HMAX + h] = rb + r < nr ? d : -INFINITY;
        }
    }
    __syncthreads();
    // running softmax statistics: one warp per head, one lane per row of the chunk (ROWS <= 32)
    for (int h = warp; h < heads; h += kMlaThreads / 32) {
      const float v = lane < nr ? sp[lane * HMAX + h] : -INFINITY;
      const float m = fmaxf(sstat[h], warp_max(v));
      const float scale = expf(sstat[h] - m);  // exp(-inf) = 0 on the first chunk
      const float p = lane < nr ? expf(v - m) : 0.f;
      if (lane < ROWS) sp[lane * HMAX + h] = p;
      const float sum = warp_sum(p);
      if (lane == 0) {
        sstat[h] = m;
        sstat[HMAX + h] = sstat[HMAX + h] * scale + sum;
        sstat[2 * HMAX + h] = scale;
      }
    }
    __syncthreads();
    {  // rescale, then add this chunk: one row's HMAX weights are read once (float4) for all CPT columns
      float scale[HMAX];
#pragma unroll
      for (int h = 0; h < HMAX; ++h) scale[h] = h < heads ? sstat[2 * HMAX + h] : 0.f;
#pragma unroll
      for (int c = 0; c < CPT; ++c)
#pragma unroll
        for (int h = 0; h < HMAX; ++h) acc[c][h] *= scale[h];
      for (int r = 0; r < nr; ++r) {
        float w[HMAX];
        const float4* wr = reinterpret_cast<const float4*>(sp + r * HMAX);
#pragma unroll
        for (int q = 0; q < HMAX / 4; ++q) {
          const float4 v = wr[q];
          w[4 * q] = v.x;
          w[4 * q + 1] = v.y;
          w[4 * q + 2] = v.z;
          w[4 * q + 3] = v.w;
        }
#pragma unroll
        for (int c = 0; c < CPT; ++c) {
          const int l = tid + c * kMlaThreads;
          if (l < ldim) {
            const float xv = to_f<T>(sx[r * ldim + l]);
#pragma unroll
            for (int h = 0; h < HMAX; ++h) acc[c][h] += w[h] * xv;
          }
        }
      }
    }
  }
  __syncthreads();
  // partials: acc [B, nsplit, heads, ldim]; (max, sum) [B, nsplit, heads, 2]
  const int64_t pb = ((int64_t)b * nsplit + split) * heads;
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    const int l = tid + c * kMlaThreads;
    if (l >= ldim) break;
#pragma unroll
    for (int h = 0; h < HMAX; ++h)
      if (h < heads) part_acc[(pb + h) * ldim + l] = acc[c][h];
  }
  if (tid < heads) {
    part_ml[(pb + tid) * 2] = sstat[tid];
    part_ml[(pb + tid) * 2 + 1] = sstat[HMAX + tid];
  }
}

// ---------------------------------------------------------------- MLA flash decode on tensor cores
// bf16 caches with latent L = 64 * NT (512 / 768 / 1024 / 1536) and at most 16 heads.  Per chunk of 16
// cache rows:  S = Q C^T  (M = 16 heads, N = 16 rows, K = L; warp w takes the K steps w, w + 8, ...)
// and O += P C  (M = 16 heads, N = L, K = 16 rows; warp w owns L / 8 output columns), both with
// mma.sync m16n8k16 (bf16 in, fp32 accumulate).  Q and P enter as bf16 high + low parts (two MMAs
// each), so the products keep about 16 mantissa bits.  Chunks stream through two shared-memory
// buffers with cp.async (the next chunk loads while this one computes); rows past the valid prefix
// are zero-filled.  Shared-memory rows are padded by 8 elements so fragment loads are conflict-free.
KIMI_D void mla_cp_async16(void* smem, const void* gmem, int src_bytes) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(src_bytes) : "memory");
}
KIMI_D void mla_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
KIMI_D void mla_cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
KIMI_D uint32_t mla_ld32(const __nv_bfloat16* p) { return *reinterpret_cast<const uint32_t*>(p); }
KIMI_D void mla_mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
KIMI_D void mla_ldmatrix_x4_trans(uint32_t* r, const __nv_bfloat16* p) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
KIMI_D void mla_split_bf16(float v, __nv_bfloat16* hi, __nv_bfloat16* lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(v);
  *hi = h;
  *lo = __float2bfloat16_rn(v - __bfloat162float(h));
}

constexpr int kMmaRows = 16;

size_t mla_mma_smem(int ldim) {
  const size_t ld = (size_t)ldim + 8;
  return 4 * 16 * ld * 2 + 8 * 16 * kMmaRows * sizeof(float) + 2 * 16 * kMmaRows * 2 + 48 * sizeof(float);
}

template <int NT>
__global__ void __launch_bounds__(256, 1) mla_decode_mma_kernel(const float* __restrict__ qlat,
                                                                const __nv_bfloat16* __restrict__ latent,
                                                                const int32_t* __restrict__ lengths, int heads,
                                                                int64_t tmax, int rows_per_split,
                                                                float* __restrict__ part_acc,
                                                                float* __restrict__ part_ml) {
  constexpr int L = 64 * NT, LD = L + 8, KSTEPS = L / 16, R = kMmaRows, V = L / 8;
  extern __shared__ __align__(16) unsigned char mla_smem_raw[];
  __nv_bfloat16* sqh = reinterpret_cast<__nv_bfloat16*>(mla_smem_raw);  // [16][LD] query, high parts
  __nv_bfloat16* sql = sqh + 16 * LD;                                    // [16][LD] query, low parts
  __nv_bfloat16* sx0 = sql + 16 * LD;                                    // 2 x [R][LD] cache chunks
  float* ss = reinterpret_cast<float*>(sx0 + 2 * R * LD);                // [8 warps][16][R] partial scores
  __nv_bfloat16* sph = reinterpret_cast<__nv_bfloat16*>(ss + 8 * 16 * R);  // [16][R] weights, high
  __nv_bfloat16* spl = sph + 16 * R;                                       // [16][R] weights, low
  float* sstat = reinterpret_cast<float*>(spl + 16 * R);                   // max [16], sum [16], scale [16]
  const int split = blockIdx.x, b = blockIdx.y, nsplit = gridDim.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tg = lane & 3;
  const int len = (int)min((int64_t)lengths[b], tmax);
  const int r0 = split * rows_per_split, r1 = min(r0 + rows_per_split, len);
  const __nv_bfloat16* xb = latent + (int64_t)b * tmax * L;

  auto load_chunk = [&](int c0, __nv_bfloat16* dst) {
    const int nr = min(R, r1 - c0);
    for (int i = tid; i < R * V; i += 256) {
      const int r = i / V, v = i - r * V;
      const bool ok = r < nr;
      mla_cp_async16(dst + r * LD + v * 8, ok ? xb + (int64_t)(c0 + r) * L + v * 8 : xb, ok ? 16 : 0);
    }
    mla_cp_commit();
  };
  if (r0 < r1) load_chunk(r0, sx0);
  {  // query -> bf16 high / low parts, heads padded to 16 with zeros
    const float* qb = qlat + (int64_t)b * heads * L;
    for (int i = tid; i < 16 * L; i += 256) {
      const int h = i / L, l = i - h * L;
      mla_split_bf16(h < heads ? qb[(int64_t)h * L + l] : 0.f, sqh + h * LD + l, sql + h * LD + l);
    }
  }
  if (tid < 16) {
    sstat[tid] = -INFINITY;
    sstat[16 + tid] = 0.f;
    sstat[32 + tid] = 0.f;
  }
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  int buf = 0;
  for (int c0 = r0; c0 < r1; c0 += R) {
    const int nr = min(R, r1 - c0);
    const __nv_bfloat16* sx = sx0 + buf * R * LD;
    if (c0 + R < r1) {
      load_chunk(c0 + R, sx0 + (buf ^ 1) * R * LD);
      mla_cp_wait<1>();
    } else {
      mla_cp_wait<0>();
    }
    __syncthreads();  // this chunk (and, on the first pass, the query and statistics) visible to all
    {  // partial scores of this warp's K steps
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      for (int ks = warp; ks < KSTEPS; ks += 8) {
        const int k0 = ks * 16 + tg * 2;
        uint32_t ah[4], al[4];
        ah[0] = mla_ld32(sqh + g * LD + k0);
        ah[1] = mla_ld32(sqh + (g + 8) * LD + k0);
        ah[2] = mla_ld32(sqh + g * LD + k0 + 8);
        ah[3] = mla_ld32(sqh + (g + 8) * LD + k0 + 8);
        al[0] = mla_ld32(sql + g * LD + k0);
        al[1] = mla_ld32(sql + (g + 8) * LD + k0);
        al[2] = mla_ld32(sql + g * LD + k0 + 8);
        al[3] = mla_ld32(sql + (g + 8) * LD + k0 + 8);
        const __nv_bfloat16* xr0 = sx + g * LD + k0;
        const __nv_bfloat16* xr1 = xr0 + 8 * LD;
        const uint32_t b00 = mla_ld32(xr0), b01 = mla_ld32(xr0 + 8), b10 = mla_ld32(xr1), b11 = mla_ld32(xr1 + 8);
        // the four products interleave two accumulators (no back-to-back dependence)
        mla_mma(sc[0], ah, b00, b01);
        mla_mma(sc[1], ah, b10, b11);
        mla_mma(sc[0], al, b00, b01);
        mla_mma(sc[1], al, b10, b11);
      }
      float* sw = ss + warp * 16 * R;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int c = nt * 8 + tg * 2;
        sw[g * R + c] = sc[nt][0];
        sw[g * R + c + 1] = sc[nt][1];
        sw[(g + 8) * R + c] = sc[nt][2];
        sw[(g + 8) * R + c + 1] = sc[nt][3];
      }
    }
    __syncthreads();
    // online softmax: one warp per head, one lane per chunk row
    for (int h = warp; h < 16; h += 8) {
      float v = -INFINITY;
      if (h < heads && lane < nr) {
        v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += ss[w * 16 * R + h * R + lane];
      }
      float p = 0.f, scale = 0.f, m = -INFINITY;
      if (h < heads) {  // nr >= 1: the maximum is finite
        m = fmaxf(sstat[h], warp_max(v));
        scale = expf(sstat[h] - m);  // exp(-inf) = 0 on the first chunk
        p = lane < nr ? expf(v - m) : 0.f;
      }
      if (lane < R) mla_split_bf16(p, sph + h * R + lane, spl + h * R + lane);
      const float sum = warp_sum(p);
      if (lane == 0) {
        if (h < heads) {
          sstat[h] = m;
          sstat[16 + h] = sstat[16 + h] * scale + sum;
        }
        sstat[32 + h] = scale;
      }
    }
    __syncthreads();
    {  // rescale the running context, then add P C for this warp's columns
      const float s0 = sstat[32 + g], s1 = sstat[32 + g + 8];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        acc[j][0] *= s0;
        acc[j][1] *= s0;
        acc[j][2] *= s1;
        acc[j][3] *= s1;
      }
      uint32_t ph[4], pl[4];
      ph[0] = mla_ld32(sph + g * R + tg * 2);
      ph[1] = mla_ld32(sph + (g + 8) * R + tg * 2);
      ph[2] = mla_ld32(sph + g * R + tg * 2 + 8);
      ph[3] = mla_ld32(sph + (g + 8) * R + tg * 2 + 8);
      pl[0] = mla_ld32(spl + g * R + tg * 2);
      pl[1] = mla_ld32(spl + (g + 8) * R + tg * 2);
      pl[2] = mla_ld32(spl + g * R + tg * 2 + 8);
      pl[3] = mla_ld32(spl + (g + 8) * R + tg * 2 + 8);
      const __nv_bfloat16* xrow = sx + ((lane & 7) + ((lane >> 3) & 1) * 8) * LD + (lane >> 4) * 8;
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        uint32_t bq[4];
        mla_ldmatrix_x4_trans(bq, xrow + warp * NT * 8 + j * 8);
        mla_mma(acc[j], ph, bq[0], bq[1]);
        mla_mma(acc[j + 1], ph, bq[2], bq[3]);
        mla_mma(acc[j], pl, bq[0], bq[1]);
        mla_mma(acc[j + 1], pl, bq[2], bq[3]);
      }
    }
    buf ^= 1;
    __syncthreads();  // the chunk buffer and the weights are rewritten next pass
  }
  __syncthreads();
  const int64_t pb = ((int64_t)b * nsplit + split) * heads;
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int col = warp * NT * 8 + j * 8 + tg * 2;
    if (g < heads)
      *reinterpret_cast<float2*>(part_acc + (pb + g) * L + col) = make_float2(acc[j][0], acc[j][1]);
    if (g + 8 < heads)
      *reinterpret_cast<float2*>(part_acc + (pb + g + 8) * L + col) = make_float2(acc[j][2], acc[j][3]);
  }
  if (tid < heads) {
    part_ml[(pb + tid) * 2] = sstat[tid];
    part_ml[(pb + tid) * 2 + 1] = sstat[16 + tid];
  }
}

__global__ void __launch_bounds__(256) mla_decode_combine_kernel(const float* __restrict__ part_acc,
                                                                 const float* __restrict__ part_ml, int nsplit,
                                                                 int heads, int ldim, float* __restrict__ ctx) {
  const int h = blockIdx.x, b = blockIdx.y;
  float m = -INFINITY;
  for (int s = 0; s < nsplit; ++s) m = fmaxf(m, part_ml[(((int64_t)b * nsplit + s) * heads + h) * 2]);
  float den = 0.f;
#pragma unroll 4
  for (int s = 0; s < nsplit; ++s) {
    const int64_t i = ((int64_t)b * nsplit + s) * heads + h;
    if (part_ml[i * 2] > -INFINITY) den += expf(part_ml[i * 2] - m) * part_ml[i * 2 + 1];
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;  // an empty row attends to nothing
  for (int l = threadIdx.x; l < ldim; l += blockDim.x) {
    float acc = 0.f;
#pragma unroll 4
    for (int s = 0; s < nsplit; ++s) {
      const int64_t i = ((int64_t)b * nsplit + s) * heads + h;
      const float ms = part_ml[i * 2];
      if (ms > -INFINITY) acc += expf(ms - m) * part_acc[i * ldim + l];
    }
    ctx[((int64_t)b * heads + h) * ldim + l] = acc * inv;
  }
}

// ---------------------------------------------------------------- sampling
constexpr int kSampleThreads = 1024;

// Philox4x32-10 (Salmon et al., SC 2011): 10 rounds of the published multipliers and Weyl key
// increments on a 128-bit counter.
KIMI_D uint4 philox4x32_10(uint4 c, uint2 key) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ key.x, lo1, hi0 ^ c.w ^ key.y, lo0);
    key.x += 0x9E3779B9u;
    key.y += 0xBB67AE85u;
  }
  return c;
}

// Order-preserving map of a float to an unsigned key (larger float, larger key).
KIMI_D uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

template <typename T>
struct SampleRow {
  const T* logits;
  const uint32_t* seen;  // nullptr: no penalty
  float penalty, inv_temp;
  KIMI_D float raw(int i) const { return to_f<T>(logits[i]); }
  // penalised logit (the greedy and validity reference)
  KIMI_D float pen(int i) const {
    float x = raw(i);
    if (seen != nullptr && ((seen[i >> 5] >> (i & 31)) & 1u)) x = x < 0.f ? x * penalty : x / penalty;
    return x;
  }
};

// Block-wide (value, index) argmax, first index among equal values.
KIMI_D void block_argmax(float& v, int& idx, float* sv, int* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  __syncthreads();
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  v = sv[lane];
  idx = si[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
}

// Radix descent over 8-bit digits of the keys: returns the key of the k-th largest element
// (count mode, `need` = k) or the nucleus boundary (mass mode, `need` = mass budget).  Elements
// with key < `floor_key` are ignored.  `bins` holds 256 counts and 256 masses.
template <typename T, bool MASS>
KIMI_D uint32_t radix_select(const SampleRow<T>& row, int vocab, float m, uint32_t floor_key, float need,
                             uint32_t* cnt, float* mass, uint32_t* shared_word, float* shared_f) {
  uint32_t prefix = 0, prefix_mask = 0;
  float above = 0.f;      // mass (or count) of elements above the current prefix range
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
      cnt[i] = 0;
      mass[i] = 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float x = row.pen(i) * row.inv_temp;
      const uint32_t key = fkey(x);
      if (key < floor_key || (key & prefix_mask) != prefix) continue;
      const uint32_t d = (key >> shift) & 255u;
      atomicAdd(&cnt[d], 1u);
      if (MASS) atomicAdd(&mass[d], expf(x - m));
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      // lane l covers digits 255 - 8l .. 248 - 8l (descending)
      const int lane = threadIdx.x;
      float w[8], tot = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = 255 - 8 * lane - j;
        w[j] = MASS ? mass[d] : (float)cnt[d];
        tot += w[j];
      }
      float incl = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const float excl = incl - tot;
      // count mode: the digit where the running count first reaches k.
      // mass mode: the lowest non-empty digit whose strictly-greater mass fits the budget.
      int pick = -1;
      float run = above + excl;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = 255 - 8 * lane - j;
        if (MASS) {
          if (cnt[d] > 0 && run <= need) pick = d;  // keeps the lowest qualifying digit of this lane
        } else if (pick < 0 && run + w[j] >= need && cnt[d] > 0) {
          pick = d;
        }
        if (!(MASS) && pick == d) break;
        run += w[j];
      }
      // count mode: the first lane (highest digits) with a pick wins; mass mode: the last one
      const unsigned has = __ballot_sync(0xffffffffu, pick >= 0);
      const int src = MASS ? (31 - __clz(has)) : (__ffs(has) - 1);
      const int d = __shfl_sync(0xffffffffu, pick, src < 0 ? 0 : src);
      // mass/count strictly above the chosen digit within this prefix range
      float run_above = 0.f;
      if (lane == src) {
        run_above = above + excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (255 - 8 * lane - j == d) break;
          run_above += w[j];
        }
      }
      run_above = __shfl_sync(0xffffffffu, run_above, src < 0 ? 0 : src);
      if (lane == 0) {
        shared_word[0] = has ? (uint32_t)d : 0u;
        shared_f[0] = run_above;
      }
    }
    __syncthreads();
    prefix |= shared_word[0] << shift;
    prefix_mask |= 255u << shift;
    above = shared_f[0];
    __syncthreads();
  }
  return prefix;
}

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const T* __restrict__ logits, int vocab,
                                                               const uint32_t* __restrict__ seen, int seen_words,
                                                               float penalty, float temperature, int top_k,
                                                               float top_p, bool do_sample,
                                                               const int64_t* __restrict__ seed_offset,
                                                               int64_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  __shared__ uint32_t cnt[256];
  __shared__ float mass[256];
  __shared__ uint32_t sword[1];
  __shared__ float sf[1];
  __shared__ float scan[kSampleThreads / 32];
  const int b = blockIdx.x;
  SampleRow<T> row{logits + (int64_t)b * vocab, seen != nullptr ? seen + (int64_t)b * seen_words : nullptr, penalty,
                   1.f / temperature};
  // pass 1: NaN-safe argmax of the penalised logits, finiteness, max of the tempered logits
  float best = -INFINITY, mx = -INFINITY;
  int bidx = vocab;
  int finite = 1;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float x = row.pen(i);
    float key = x;
    if (isnan(x)) key = -INFINITY;
    else if (isinf(x)) key = x > 0.f ? 1e30f : -1e30f;
    if (key > best || (key == best && i < bidx)) {
      best = key;
      bidx = i;
    }
    finite &= isfinite(x) ? 1 : 0;
    mx = fmaxf(mx, x * row.inv_temp);
  }
  if (bidx == vocab) bidx = 0;
  block_argmax(best, bidx, sv, si);
  const int all_finite = __syncthreads_and(finite);
  if (!do_sample || !all_finite) {
    if (threadIdx.x == 0) out[b] = bidx;
    return;
  }
  mx = block_max(mx, sv);
  // top-k: key of the k-th largest tempered logit (ties at the boundary are kept)
  uint32_t floor_key = 0;
  if (top_k > 0 && top_k < vocab)
    floor_key = radix_select<T, false>(row, vocab, mx, 0u, (float)top_k, cnt, mass, sword, sf);
  // top-p: the lowest kept value whose strictly-greater mass fits p * Z
  if (top_p < 1.f) {
    float z = 0.f;
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
      const float x = row.pen(i) * row.inv_temp;
      if (fkey(x) >= floor_key) z += expf(x - mx);
    }
    z = block_sum(z, sv);
    const uint32_t pk = radix_select<T, true>(row, vocab, mx, floor_key, top_p * z, cnt, mass, sword, sf);
    floor_key = max(floor_key, pk);
  }
  // draw: contiguous chunks per thread, block exclusive scan of the kept mass
  const int per = (vocab + kSampleThreads - 1) / kSampleThreads;
  const int i0 = min(threadIdx.x * per, vocab), i1 = min(i0 + per, vocab);
  float local = 0.f;
  for (int i = i0; i < i1; ++i) {
    const float x = row.pen(i) * row.inv_temp;
    if (fkey(x) >= floor_key) local += expf(x - mx);
  }
  // inclusive scan over the block
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    float w = scan[lane];
    float wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    scan[lane] = wi - w;  // exclusive warp offsets
  }
  __syncthreads();
  const float excl = scan[warp] + incl - local;
  __shared__ float total;
  if (threadIdx.x == kSampleThreads - 1) total = excl + local;
  __syncthreads();
  const uint4 r = philox4x32_10(make_uint4((uint32_t)b, 0u, (uint32_t)seed_offset[1], (uint32_t)(seed_offset[1] >> 32)),
                                make_uint2((uint32_t)seed_offset[0], (uint32_t)(seed_offset[0] >> 32)));
  const float u = (float)(r.x >> 8) * (1.f / 16777216.f);
  const float target = u * total;
  __shared__ int pick;
  if (threadIdx.x == 0) pick = -1;
  __syncthreads();
  if (local > 0.f && target >= excl && (target < excl + local || threadIdx.x == kSampleThreads - 1 ||
                                        excl + local >= total)) {
    float run = excl;
    int last = -1;
    for (int i = i0; i < i1; ++i) {
      const float x = row.pen(i) * row.inv_temp;
      if (fkey(x) < floor_key) continue;
      last = i;
      run += expf(x - mx);
      if (run > target) break;
    }
    atomicCAS(&pick, -1, last);
  }
  __syncthreads();
  if (threadIdx.x == 0) out[b] = pick >= 0 ? pick : bidx;
}

__global__ void seen_mark_kernel(uint32_t* __restrict__ seen, int seen_words, const int64_t* __restrict__ ids,
                                 int64_t rows, int64_t cols, int64_t ld, int vocab) {
  const int64_t n = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const int64_t t = ids[r * ld + c];
    if (t >= 0 && t < vocab) atomicOr(&seen[r * seen_words + (t >> 5)], 1u << (t & 31));
  }
}

}  // namespace

// ---------------------------------------------------------------- host entry points
cudaError_t conv_step(int dtype, const ConvStepArgs& args, int streams, int batch, int ksize, float eps,
                      cudaStream_t s) {
  int cmax = 0;
  for (int i = 0; i < streams; ++i) {
    const int c = args.channels[i];
    if (c <= 0 || c % 8) return cudaErrorInvalidValue;
    const int hl = args.head_lanes[i];
    if (hl < 0 || hl > 32 || (hl & (hl - 1)) || (hl > 0 && (c / 8) % hl)) return cudaErrorInvalidValue;
    cmax = c > cmax ? c : cmax;
  }
  const dim3 grid((cmax / 8 + 255) / 256, batch, streams);
#define KIMI_CS(TT, KK) conv_step_kernel<TT, KK><<<grid, 256, 0, s>>>(args, eps)
#define KIMI_CS_K(TT)                 \
  switch (ksize) {                    \
    case 1: KIMI_CS(TT, 1); break;    \
    case 2: KIMI_CS(TT, 2); break;    \
    case 3: KIMI_CS(TT, 3); break;    \
    case 4: KIMI_CS(TT, 4); break;    \
    case 5: KIMI_CS(TT, 5); break;    \
    case 6: KIMI_CS(TT, 6); break;    \
    case 7: KIMI_CS(TT, 7); break;    \
    case 8: KIMI_CS(TT, 8); break;    \
    default: return cudaErrorInvalidValue; \
  }
  switch (dtype) {
    case 0: KIMI_CS_K(float); break;
    case 1: KIMI_CS_K(__nv_bfloat16); break;
    case 2: KIMI_CS_K(__half); break;
    default: return cudaErrorInvalidValue;
  }
#undef KIMI_CS_K
#undef KIMI_CS
  return cudaGetLastError();
}

cudaError_t kda_decode(int dtype, const void* q, const void* k, const void* v, const float* g, const float* beta,
                       const float* state_in, float* state_out, void* o, int batch, int heads, cudaStream_t s) {
  const dim3 grid(heads, batch);
  switch (dtype) {
    case 0: kda_decode_kernel<float><<<grid, 256, 0, s>>>((const float*)q, (const float*)k, (const float*)v, g, beta,
                                                          state_in, state_out, (float*)o, heads); break;
    case 1: kda_decode_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
                (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta, state_in,
                state_out, (__nv_bfloat16*)o, heads); break;
    case 2: kda_decode_kernel<__half><<<grid, 256, 0, s>>>((const __half*)q, (const __half*)k, (const __half*)v, g,
                                                           beta, state_in, state_out, (__half*)o, heads); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

namespace {
// Instance choice: heads padded to 4 / 8 / 16 / 32, columns per thread rounded up to 2 / 4 / 6 / 8,
// at most 96 running accumulators per thread (HMAX * CPT), 16 rows per chunk above L = 1024.
struct MlaShape {
  int hmax, cpt, rows;
};
MlaShape mla_shape(int heads, int ldim) {
  MlaShape s{heads <= 4 ? 4 : heads <= 8 ? 8 : heads <= 16 ? 16 : heads <= 32 ? 32 : 0, 0, ldim <= 1024 ? 32 : 16};
  const int need = (ldim + kMlaThreads - 1) / kMlaThreads;
  s.cpt = need <= 2 ? 2 : need <= 4 ? 4 : need <= 6 ? 6 : need <= 8 ? 8 : 0;
  return s;
}
size_t mla_smem(int heads, int ldim, const MlaShape& s, size_t elt) {
  return sizeof(float) * (size_t)heads * ldim + elt * (size_t)s.rows * ldim +
         sizeof(float) * ((size_t)s.rows * s.hmax + 3 * (size_t)s.hmax);
}
}  // namespace

bool mla_decode_supported(int heads, int ldim) {
  if (ldim % 8 || heads <= 0) return false;
  const MlaShape s = mla_shape(heads, ldim);
  if (!s.hmax || !s.cpt || s.hmax * s.cpt > 96) return false;
  return mla_smem(heads, ldim, s, sizeof(float)) <= 200 * 1024;  // fits every cache dtype
}

int mla_decode_splits(int batch, int64_t tmax, int* rows_per_split) {
  // about six CTAs per SM over the grid (several resident per SM keep more cache rows in flight),
  // each with at least one 32-row block
  const int target = device_sms() * 6;
  int splits = (target + batch - 1) / batch;
  constexpr int kMlaSplitRows = 32;  // a multiple of every instance's chunk rows
  const int64_t max_splits = (tmax + kMlaSplitRows - 1) / kMlaSplitRows;
  if (splits > max_splits) splits = (int)max_splits;
  if (splits < 1) splits = 1;
  int64_t rps = (tmax + splits - 1) / splits;
  rps = (rps + kMlaSplitRows - 1) / kMlaSplitRows * kMlaSplitRows;
  *rows_per_split = (int)rps;
  return (int)((tmax + rps - 1) / rps);
}

cudaError_t mla_decode(int dtype, const float* qlat, const void* latent, const int32_t* lengths, int batch,
                       int heads, int ldim, int64_t tmax, float* part_acc, float* part_ml, int splits,
                       int rows_per_split, float* ctx, cudaStream_t s) {
  if (!mla_decode_supported(heads, ldim) || tmax <= 0 || dtype < 0 || dtype > 2) return cudaErrorInvalidValue;
  if (dtype == 1 && heads <= 16 && rows_per_split % kMmaRows == 0 &&
      (ldim == 512 || ldim == 768 || ldim == 1024 || ldim == 1536)) {
    const size_t msm = mla_mma_smem(ldim);
    const dim3 mgrid(splits, batch);
#define KIMI_MLA_MMA(NT)                                                                                     \
  do {                                                                                                       \
    cudaError_t e = ensure_dynamic_smem(mla_decode_mma_kernel<NT>, (int)msm);                                \
    if (e != cudaSuccess) return e;                                                                          \
    mla_decode_mma_kernel<NT><<<mgrid, 256, msm, s>>>(qlat, static_cast<const __nv_bfloat16*>(latent), lengths, \
                                                      heads, tmax, rows_per_split, part_acc, part_ml);        \
  } while (0)
    switch (ldim) {
      case 512: KIMI_MLA_MMA(8); break;
      case 768: KIMI_MLA_MMA(12); break;
      case 1024: KIMI_MLA_MMA(16); break;
      default: KIMI_MLA_MMA(24); break;
    }
#undef KIMI_MLA_MMA
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    mla_decode_combine_kernel<<<dim3(heads, batch), 256, 0, s>>>(part_acc, part_ml, splits, heads, ldim, ctx);
    return cudaGetLastError();
  }
  const MlaShape shp = mla_shape(heads, ldim);
  const size_t sm = mla_smem(heads, ldim, shp, dtype == 0 ? sizeof(float) : 2);
  if (sm > 200 * 1024) return cudaErrorInvalidValue;
  if (rows_per_split % shp.rows) return cudaErrorInvalidValue;
  const dim3 grid(splits, batch);
  cudaError_t err = cudaErrorInvalidValue;
#define KIMI_MLA(TT, HM, CP, RW)                                                                               \
  do {                                                                                                         \
    auto fn = mla_decode_kernel<TT, HM, CP, RW>;                                                               \
    if (sm > 48 * 1024) {                                                                                      \
      cudaError_t e = ensure_dynamic_smem(fn, (int)(200 * 1024));                                             \
      if (e != cudaSuccess) return e;                                                                          \
    }                                                                                                          \
    fn<<<grid, kMlaThreads, sm, s>>>(qlat, (const TT*)latent, lengths, heads, ldim, tmax, rows_per_split,     \
                                     part_acc, part_ml);                                                       \
    err = cudaSuccess;                                                                                         \
  } while (0)
#define KIMI_MLA_R(TT, HM, CP)              \
  if (shp.rows == 32)                       \
    KIMI_MLA(TT, HM, CP, 32);               \
  else                                      \
    KIMI_MLA(TT, HM, CP, 16);
#define KIMI_MLA_T(TT)                                                   \
  switch (shp.hmax * 16 + shp.cpt) {                                     \
    case 4 * 16 + 2: KIMI_MLA_R(TT, 4, 2); break;                        \
    case 4 * 16 + 4: KIMI_MLA_R(TT, 4, 4); break;                        \
    case 4 * 16 + 6: KIMI_MLA_R(TT, 4, 6); break;                        \
    case 4 * 16 + 8: KIMI_MLA_R(TT, 4, 8); break;                        \
    case 8 * 16 + 2: KIMI_MLA_R(TT, 8, 2); break;                        \
    case 8 * 16 + 4: KIMI_MLA_R(TT, 8, 4); break;                        \
    case 8 * 16 + 6: KIMI_MLA_R(TT, 8, 6); break;                        \
    case 8 * 16 + 8: KIMI_MLA_R(TT, 8, 8); break;                        \
    case 16 * 16 + 2: KIMI_MLA_R(TT, 16, 2); break;                      \
    case 16 * 16 + 4: KIMI_MLA_R(TT, 16, 4); break;                      \
    case 16 * 16 + 6: KIMI_MLA_R(TT, 16, 6); break;                      \
    case 32 * 16 + 2: KIMI_MLA_R(TT, 32, 2); break;                      \
    default: return cudaErrorInvalidValue;                               \
  }
  switch (dtype) {
    case 0: KIMI_MLA_T(float); break;
    case 1: KIMI_MLA_T(__nv_bfloat16); break;
    case 2: KIMI_MLA_T(__half); break;
  }
#undef KIMI_MLA_T
#undef KIMI_MLA_R
#undef KIMI_MLA
  if (err != cudaSuccess) return err;
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  mla_decode_combine_kernel<<<dim3(heads, batch), 256, 0, s>>>(part_acc, part_ml, splits, heads, ldim, ctx);
  return cudaGetLastError();
}

cudaError_t sample_tokens(int dtype, const void* logits, int batch, int vocab, const uint32_t* seen, int seen_words,
                          float penalty, float temperature, int top_k, float top_p, bool do_sample,
                          const int64_t* seed_offset, int64_t* out, cudaStream_t s) {
  if (batch <= 0 || vocab <= 0 || !(temperature > 0.f)) return cudaErrorInvalidValue;
  switch (dtype) {
    case 0: sample_kernel<float><<<batch, kSampleThreads, 0, s>>>((const float*)logits, vocab, seen, seen_words,
                                                                  penalty, temperature, top_k, top_p, do_sample,
                                                                  seed_offset, out); break;
    case 1: sample_kernel<__nv_bfloat16><<<batch, kSampleThreads, 0, s>>>(
                (const __nv_bfloat16*)logits, vocab, seen, seen_words, penalty, temperature, top_k, top_p, do_sample,
                seed_offset, out); break;
    case 2: sample_kernel<__half><<<batch, kSampleThreads, 0, s>>>((const __half*)logits, vocab, seen, seen_words,
                                                                   penalty, temperature, top_k, top_p, do_sample,
                                                                   seed_offset, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t seen_mark(uint32_t* seen, int seen_words, const int64_t* ids, int64_t rows, int64_t cols, int64_t ld,
                      int vocab, cudaStream_t s) {
  const int64_t n = rows * cols;
  if (n <= 0) return cudaSuccess;
  int blocks = (int)((n + 255) / 256);
  if (blocks > 1024) blocks = 1024;
  seen_mark_kernel<<<blocks, 256, 0, s>>>(seen, seen_words, ids, rows, cols, ld, vocab);
  return cudaGetLastError();
}

}  // namespace kimi
