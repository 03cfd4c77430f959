// KDA short causal depthwise conv + SiLU (+ L2 normalisation per head), forward and backward.
//
//   pre[t,c] = sum_{j < K, t - j >= 0} w[c,j] x[t-j,c],   s = silu(pre),
//   y = s / max(||s_head||, eps)   (or y = s without the normalisation)
//
// Layout [B, T, C] with C % 64 == 0.  One thread owns 8 consecutive channels (one 16-byte vector
// of bf16 / half, two of fp32) and walks a tile of kTile tokens, so every x / dy element is read
// once and the K-tap history stays in registers; the 64-channel head norm is a shuffle reduction
// over the head_dim / 8 lanes that share the head.  Block = the C / 8 channel chunks (rounded up
// to whole warps), grid = (token tiles, batch).
//
// Backward (one pass): walking the tile's tokens downwards from kTile + K - 2 tokens ahead (the
// first K - 1 of them only recompute the dpre halo from the next tile),
//   dpre = ds * silu'(pre),  ds = dy / n - s (s . dy) / n^3  (n = ||s_head|| > eps; else dy / eps),
//   dx[t,c] = sum_j w[c,j] dpre[t+j,c],   dw[c,j] = sum_t dpre[t,c] x[t-j,c]  (per-thread partials
//   written per block to a scratch row, then one reduction kernel: no contended atomics).
// Parity: `src/kimi_primitives/short_conv.py:84-90` (causal depthwise conv1d, lag-ordered
// weights) followed by SiLU and the per-head L2 normalisation of q and k in
// `src/kda/projections.py:188-200` (reference).
#include "common.cuh"
#include "device_info.h"
#include "kernels.h"
#include "tc_common.cuh"

namespace kimi {
namespace {

constexpr int kTile = 16;

template <typename T>
KIMI_D void load8(const T* p, float* out) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
    Vec<T> v;
    v.load(p);
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = v.f(e);
  }
}
template <typename T>
KIMI_D void store8(T* p, const float* in) {
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
__global__ void __launch_bounds__(256) conv_fwd_v_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                                         T* __restrict__ y, int tokens, int channels, int head_lanes,
                                                         float eps, bool normalize) {
  const int ch = threadIdx.x;
  const bool active = ch * 8 < channels;
  const int c0 = active ? ch * 8 : 0;
  const int b = blockIdx.y, t0 = blockIdx.x * kTile, t1 = min(t0 + kTile, tokens);
  const int64_t rowbase = (int64_t)b * tokens;
  float wr[8][K];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < K; ++j) wr[e][j] = active ? w[(c0 + e) * K + j] : 0.f;
  float hist[K][8];  // hist[j] = x[t - j]; slot 0 is filled each step
#pragma unroll
  for (int j = 1; j < K; ++j) {
    const int t = t0 - j;
    if (active && t >= 0)
      load8<T>(x + (rowbase + t) * channels + c0, hist[j]);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) hist[j][e] = 0.f;
  }
  for (int t = t0; t < t1; ++t) {
    if (active)
      load8<T>(x + (rowbase + t) * channels + c0, hist[0]);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) hist[0][e] = 0.f;
    float s[8], ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float pre = 0.f;
#pragma unroll
      for (int j = 0; j < K; ++j) pre += wr[e][j] * hist[j][e];
      s[e] = siluf_(pre);
      ss += s[e] * s[e];
    }
    if (normalize) {
      ss = group_sum(ss, head_lanes);
      const float inv = 1.f / fmaxf(sqrtf(ss), eps);
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] *= inv;
    }
    if (active) store8<T>(y + (rowbase + t) * channels + c0, s);
#pragma unroll
    for (int j = K - 1; j > 0; --j)
#pragma unroll
      for (int e = 0; e < 8; ++e) hist[j][e] = hist[j - 1][e];
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(256) conv_bwd_v_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                         const float* __restrict__ w, T* __restrict__ dx,
                                                         float* __restrict__ dw, int tokens, int channels,
                                                         int head_lanes, float eps, bool normalize) {
  const int ch = threadIdx.x;
  const bool active = ch * 8 < channels;
  const int c0 = active ? ch * 8 : 0;
  const int b = blockIdx.y, t0 = blockIdx.x * kTile, t1 = min(t0 + kTile, tokens);
  const int64_t rowbase = (int64_t)b * tokens;
  float wr[8][K], dwacc[8][K];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < K; ++j) {
      wr[e][j] = active ? w[(c0 + e) * K + j] : 0.f;
      dwacc[e][j] = 0.f;
    }
  const int tstart = min(t1 + K - 2, tokens - 1);
  float xw[K][8];   // xw[j] = x[t - j]
  float dph[K][8];  // dph[j] = dpre[t + j]; slot 0 is this step's
#pragma unroll
  for (int j = 0; j < K; ++j) {
    const int t = tstart - j;
    if (active && t >= 0)
      load8<T>(x + (rowbase + t) * channels + c0, xw[j]);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) xw[j][e] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) dph[j][e] = 0.f;
  }
  for (int t = tstart; t >= t0; --t) {
    float d[8];
    if (active)
      load8<T>(dy + (rowbase + t) * channels + c0, d);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) d[e] = 0.f;
    float pre[8], s[8], ss = 0.f, dot = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < K; ++j) p += wr[e][j] * xw[j][e];
      pre[e] = p;
      s[e] = siluf_(p);
      ss += s[e] * s[e];
      dot += s[e] * d[e];
    }
    float inv = 1.f, coef = 0.f;
    if (normalize) {
      ss = group_sum(ss, head_lanes);
      dot = group_sum(dot, head_lanes);
      const float n = sqrtf(ss);
      if (n > eps) {
        inv = 1.f / n;
        coef = dot * inv * inv * inv;
      } else {
        inv = 1.f / eps;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float ds = d[e] * inv - s[e] * coef;
      const float sg = sigmoidf_(pre[e]);
      dph[0][e] = ds * sg * (1.f + pre[e] * (1.f - sg));
    }
    if (t < t1) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < K; ++j) acc += wr[e][j] * dph[j][e];
        o[e] = acc;
#pragma unroll
        for (int j = 0; j < K; ++j) dwacc[e][j] += dph[0][e] * xw[j][e];
      }
      if (active) store8<T>(dx + (rowbase + t) * channels + c0, o);
    }
    // slide: dpre history up, x window down (x[t - K] enters)
#pragma unroll
    for (int j = K - 1; j > 0; --j)
#pragma unroll
      for (int e = 0; e < 8; ++e) dph[j][e] = dph[j - 1][e];
#pragma unroll
    for (int j = 0; j < K - 1; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) xw[j][e] = xw[j + 1][e];
    const int tn = t - K;
    if (active && tn >= 0)
      load8<T>(x + (rowbase + tn) * channels + c0, xw[K - 1]);
    else
#pragma unroll
      for (int e = 0; e < 8; ++e) xw[K - 1][e] = 0.f;
  }
  // this block's dw partial: row (blockIdx.y, blockIdx.x) of the [blocks, C * K] scratch
  if (active) {
    float* part = dw + ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * channels * K;
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int j = 0; j < K; ++j) part[(c0 + e) * K + j] = dwacc[e][j];
  }
}

// dw[i] = sum over blocks of part[block][i]: a block owns 32 consecutive columns; its 8 warps read
// interleaved rows (one 128-byte line per warp and row), then combine through shared memory.
__global__ void __launch_bounds__(256) dw_reduce_kernel(const float* __restrict__ part, float* __restrict__ dw,
                                                        int blocks, int n) {
  __shared__ float red[8][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;
  float acc = 0.f;
  if (i < n) {
#pragma unroll 8
    for (int b = blockIdx.y * 8 + warp; b < blocks; b += 8 * gridDim.y) acc += part[(int64_t)b * n + i];
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && i < n) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += red[w][lane];
    atomicAdd(&dw[i], s);  // gridDim.y partial sums per weight; dw starts at zero
  }
}

// ---------------------------------------------------------------- shared-memory staged variants
// The block's token rows (and their K - 1 halo rows) are contiguous in [B, T, C]: one TMA bulk
// copy per tensor brings them into shared memory (mbarrier completion), then each thread walks
// its 8 channels over the tile reading shared memory, so DRAM latency is paid once per block.
// Tokens per block: 32 forward; 16 backward, whose two staged tensors and larger register state would
// otherwise leave two 3-warp blocks per SM (the walk over the tile is a dependent chain, so the
// backward is latency-bound and wants more resident blocks more than it minds the K - 1 halo).
constexpr int kSTileFwd = 32, kSTileBwd = 16;

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   tc::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
               : "memory");
}

// Rows [r0, r1) of one batch: zero the rows outside the sequence (generic stores to addresses the
// bulk copy does not touch) and return the byte count of the rows inside it.
template <typename T>
__device__ uint32_t zero_outside(T* dst, int r0, int r1, int tokens, int channels) {
  for (int r = r0; r < r1; ++r) {
    if (r >= 0 && r < tokens) continue;
    T* row = dst + (int64_t)(r - r0) * channels;
    for (int c = threadIdx.x; c < channels; c += blockDim.x) row[c] = from_f<T>(0.f);
  }
  const int v0 = max(r0, 0), v1 = min(r1, tokens);
  return v1 > v0 ? (uint32_t)((int64_t)(v1 - v0) * channels * sizeof(T)) : 0u;
}
template <typename T>
__device__ void copy_inside(T* dst, const T* src_batch, int r0, int r1, int tokens, int channels, uint64_t* bar) {
  const int v0 = max(r0, 0), v1 = min(r1, tokens);
  if (v1 > v0)
    bulk_g2s(dst + (int64_t)(v0 - r0) * channels, src_batch + (int64_t)v0 * channels,
             (uint32_t)((int64_t)(v1 - v0) * channels * sizeof(T)), bar);
}

// Forward tokens are independent: kFwdGroups groups of whole warps split the block's tile (each
// group walks kSTileFwd / kFwdGroups tokens over the same staged rows).
constexpr int kFwdGroups = 2;

template <typename T, int K>
__global__ void __launch_bounds__(512) conv_fwd_s_kernel(const T* __restrict__ x, const float* __restrict__ w,
                                                         T* __restrict__ y, int tokens, int channels, int head_lanes,
                                                         float eps, bool normalize) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  T* sx = reinterpret_cast<T*>(smem);
  const int per = blockDim.x / kFwdGroups;  // threads of one token group (whole warps)
  const int grp = threadIdx.x / per, ch = threadIdx.x - grp * per;
  const bool active = ch * 8 < channels;
  const int c0 = active ? ch * 8 : 0;
  const int b = blockIdx.y, t0 = blockIdx.x * kSTileFwd, t1 = min(t0 + kSTileFwd, tokens);
  const int tg0 = t0 + grp * (kSTileFwd / kFwdGroups), tg1 = min(tg0 + kSTileFwd / kFwdGroups, t1);
  const int r0 = t0 - (K - 1);
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
  }
  __syncthreads();
  const uint32_t bytes = zero_outside<T>(sx, r0, t1, tokens, channels);
  if (threadIdx.x == 0) {
    tc::mbar_arrive_expect_tx(&bar, bytes);
    copy_inside<T>(sx, x + (int64_t)b * tokens * channels, r0, t1, tokens, channels, &bar);
  }
  float wr[8][K];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < K; ++j) wr[e][j] = active ? w[(c0 + e) * K + j] : 0.f;
  __syncthreads();  // zero rows written
  tc::mbar_wait_local(&bar, 0, nullptr, 0);
  const int64_t rowbase = (int64_t)b * tokens;
  for (int t = tg0; t < tg1; ++t) {
    float s[8], ss = 0.f;
    float xv[K][8];
#pragma unroll
    for (int j = 0; j < K; ++j) load8<T>(sx + (int64_t)(t - j - r0) * channels + c0, xv[j]);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float pre = 0.f;
#pragma unroll
      for (int j = 0; j < K; ++j) pre += wr[e][j] * xv[j][e];
      s[e] = siluf_(pre);
      ss += s[e] * s[e];
    }
    if (normalize) {
      ss = group_sum(ss, head_lanes);
      const float inv = 1.f / fmaxf(sqrtf(ss), eps);
#pragma unroll
      for (int e = 0; e < 8; ++e) s[e] *= inv;
    }
    if (active) store8<T>(y + (rowbase + t) * channels + c0, s);
  }
}

template <typename T, int K>
__global__ void __launch_bounds__(256) conv_bwd_s_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                         const float* __restrict__ w, T* __restrict__ dx,
                                                         float* __restrict__ dw, int tokens, int channels,
                                                         int head_lanes, float eps, bool normalize) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t bar;
  const int ch = threadIdx.x;
  const bool active = ch * 8 < channels;
  const int c0 = active ? ch * 8 : 0;
  const int b = blockIdx.y, t0 = blockIdx.x * kSTileBwd, t1 = min(t0 + kSTileBwd, tokens);
  const int tstart = min(t1 + K - 2, tokens - 1);
  const int xr0 = t0 - (K - 1), xr1 = tstart + 1;  // x rows needed
  const int dr0 = t0, dr1 = tstart + 1;            // dy rows needed
  T* sx = reinterpret_cast<T*>(smem);
  T* sd = sx + (int64_t)(kSTileBwd + 2 * K - 2) * channels;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
  }
  __syncthreads();
  const uint32_t bytes = zero_outside<T>(sx, xr0, xr1, tokens, channels) + zero_outside<T>(sd, dr0, dr1, tokens, channels);
  if (threadIdx.x == 0) {
    tc::mbar_arrive_expect_tx(&bar, bytes);
    copy_inside<T>(sx, x + (int64_t)b * tokens * channels, xr0, xr1, tokens, channels, &bar);
    copy_inside<T>(sd, dy + (int64_t)b * tokens * channels, dr0, dr1, tokens, channels, &bar);
  }
  float wr[8][K], dwacc[8][K];
#pragma unroll
  for (int e = 0; e < 8; ++e)
#pragma unroll
    for (int j = 0; j < K; ++j) {
      wr[e][j] = active ? w[(c0 + e) * K + j] : 0.f;
      dwacc[e][j] = 0.f;
    }
  __syncthreads();
  tc::mbar_wait_local(&bar, 0, nullptr, 0);
  const int64_t rowbase = (int64_t)b * tokens;
  float dph[K][8];  // dph[j] = dpre[t + j]; slot 0 is this step's
#pragma unroll
  for (int j = 0; j < K; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) dph[j][e] = 0.f;
  for (int t = tstart; t >= t0; --t) {
    float d[8], xw[K][8];
    load8<T>(sd + (int64_t)(t - dr0) * channels + c0, d);
#pragma unroll
    for (int j = 0; j < K; ++j) load8<T>(sx + (int64_t)(t - j - xr0) * channels + c0, xw[j]);
    float pre[8], s[8], ss = 0.f, dot = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float p = 0.f;
#pragma unroll
      for (int j = 0; j < K; ++j) p += wr[e][j] * xw[j][e];
      pre[e] = p;
      s[e] = siluf_(p);
      ss += s[e] * s[e];
      dot += s[e] * d[e];
    }
    float inv = 1.f, coef = 0.f;
    if (normalize) {
      ss = group_sum(ss, head_lanes);
      dot = group_sum(dot, head_lanes);
      const float n = sqrtf(ss);
      if (n > eps) {
        inv = 1.f / n;
        coef = dot * inv * inv * inv;
      } else {
        inv = 1.f / eps;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float ds = d[e] * inv - s[e] * coef;
      const float sg = sigmoidf_(pre[e]);
      dph[0][e] = ds * sg * (1.f + pre[e] * (1.f - sg));
    }
    if (t < t1) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < K; ++j) acc += wr[e][j] * dph[j][e];
        o[e] = acc;
#pragma unroll
        for (int j = 0; j < K; ++j) dwacc[e][j] += dph[0][e] * xw[j][e];
      }
      if (active) store8<T>(dx + (rowbase + t) * channels + c0, o);
    }
#pragma unroll
    for (int j = K - 1; j > 0; --j)
#pragma unroll
      for (int e = 0; e < 8; ++e) dph[j][e] = dph[j - 1][e];
  }
  if (active) {
    float* part = dw + ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * channels * K;
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int j = 0; j < K; ++j) part[(c0 + e) * K + j] = dwacc[e][j];
  }
}

size_t conv_fwd_s_smem(int channels, int ksize, size_t es) { return (size_t)(kSTileFwd + ksize - 1) * channels * es; }
size_t conv_bwd_s_smem(int channels, int ksize, size_t es) {
  return (size_t)((kSTileBwd + 2 * ksize - 2) + (kSTileBwd + ksize - 1)) * channels * es;
}
constexpr size_t kConvSmemCap = 200 * 1024;

template <typename T>
cudaError_t launch_conv(bool fwd, const void* dy, const void* x, const float* w, void* out, float* dw_part, int batch,
                        int tokens, int channels, int ksize, int head_dim, float eps, bool normalize,
                        cudaStream_t s) {
  float* dw = dw_part;
  if (channels % 64 || head_dim % 8 || channels % head_dim || head_dim / 8 > 32 || (head_dim / 8 & (head_dim / 8 - 1)))
    return cudaErrorInvalidValue;
  const int threads = ((channels / 8 + 31) / 32) * 32;
  if (threads > 256) return cudaErrorInvalidValue;
  // 16-byte vector accesses and bulk copies of whole rows (channels % 64 == 0 keeps every row
  // offset aligned once the base pointers are)
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) | reinterpret_cast<uintptr_t>(out)) & 15)
    return cudaErrorInvalidValue;
  const bool staged = (fwd ? conv_fwd_s_smem(channels, ksize, sizeof(T))
                           : conv_bwd_s_smem(channels, ksize, sizeof(T))) <= kConvSmemCap;
  const int tile = staged ? (fwd ? kSTileFwd : kSTileBwd) : kTile;
  const dim3 grid((tokens + tile - 1) / tile, batch);
  const int hl = head_dim / 8;
  const size_t ssm = fwd ? conv_fwd_s_smem(channels, ksize, sizeof(T)) : conv_bwd_s_smem(channels, ksize, sizeof(T));
#define KIMI_CONV_CASE(KK)                                                                                          \
  case KK:                                                                                                          \
    if (staged) {                                                                                                   \
      if (ssm > 48 * 1024) {                                                                                        \
        cudaError_t e = fwd ? ensure_dynamic_smem(conv_fwd_s_kernel<T, KK>, (int)kConvSmemCap)                       \
                            : ensure_dynamic_smem(conv_bwd_s_kernel<T, KK>, (int)kConvSmemCap);                      \
        if (e != cudaSuccess) return e;                                                                             \
      }                                                                                                             \
      if (fwd)                                                                                                      \
        conv_fwd_s_kernel<T, KK><<<grid, threads * kFwdGroups, ssm, s>>>((const T*)x, w, (T*)out, tokens, channels, \
                                                                         hl, eps, normalize);                       \
      else                                                                                                          \
        conv_bwd_s_kernel<T, KK><<<grid, threads, ssm, s>>>((const T*)dy, (const T*)x, w, (T*)out, dw, tokens,      \
                                                            channels, hl, eps, normalize);                          \
    } else if (fwd) {                                                                                               \
      conv_fwd_v_kernel<T, KK><<<grid, threads, 0, s>>>((const T*)x, w, (T*)out, tokens, channels, hl, eps,         \
                                                        normalize);                                                 \
    } else {                                                                                                        \
      conv_bwd_v_kernel<T, KK><<<grid, threads, 0, s>>>((const T*)dy, (const T*)x, w, (T*)out, dw, tokens,          \
                                                        channels, hl, eps, normalize);                              \
    }                                                                                                               \
    break;
  switch (ksize) {
    KIMI_CONV_CASE(1)
    KIMI_CONV_CASE(2)
    KIMI_CONV_CASE(3)
    KIMI_CONV_CASE(4)
    KIMI_CONV_CASE(5)
    KIMI_CONV_CASE(6)
    KIMI_CONV_CASE(7)
    KIMI_CONV_CASE(8)
    default:
      return cudaErrorInvalidValue;
  }
#undef KIMI_CONV_CASE
  return cudaGetLastError();
}

}  // namespace

// >= the staged rows (kSTileBwd >= kTile)
int conv_bwd_partial_rows(int batch, int tokens) { return batch * ((tokens + kTile - 1) / kTile); }
static_assert(kSTileBwd >= kTile, "the partial-sum buffer is sized for kTile-token tiles");

cudaError_t conv_silu_norm_fwd(int dtype, const void* x, const float* w, void* y, int batch, int tokens,
                               int channels, int ksize, int head_dim, float eps, bool normalize, cudaStream_t s) {
  switch (dtype) {
    case 0: return launch_conv<float>(true, nullptr, x, w, y, nullptr, batch, tokens, channels, ksize, head_dim, eps,
                                      normalize, s);
    case 1: return launch_conv<__nv_bfloat16>(true, nullptr, x, w, y, nullptr, batch, tokens, channels, ksize,
                                              head_dim, eps, normalize, s);
    case 2: return launch_conv<__half>(true, nullptr, x, w, y, nullptr, batch, tokens, channels, ksize, head_dim, eps,
                                       normalize, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t conv_silu_norm_bwd(int dtype, const void* dy, const void* x, const float* w, void* dx, float* dw,
                               float* dw_part, int batch, int tokens, int channels, int ksize, int head_dim, float eps,
                               bool normalize, cudaStream_t s) {
  cudaError_t e = cudaErrorInvalidValue;
  switch (dtype) {
    case 0: e = launch_conv<float>(false, dy, x, w, dx, dw_part, batch, tokens, channels, ksize, head_dim, eps,
                                   normalize, s); break;
    case 1: e = launch_conv<__nv_bfloat16>(false, dy, x, w, dx, dw_part, batch, tokens, channels, ksize, head_dim,
                                           eps, normalize, s); break;
    case 2: e = launch_conv<__half>(false, dy, x, w, dx, dw_part, batch, tokens, channels, ksize, head_dim, eps,
                                    normalize, s); break;
  }
  if (e != cudaSuccess) return e;
  const int n = channels * ksize;
  const size_t es = dtype == 0 ? 4 : 2;
  const int tile = conv_bwd_s_smem(channels, ksize, es) <= kConvSmemCap ? kSTileBwd : kTile;
  const int rows = batch * ((tokens + tile - 1) / tile);
  const dim3 rgrid((n + 31) / 32, rows >= 64 * 8 ? 8 : 1);
  if (cudaMemsetAsync(dw, 0, sizeof(float) * n, s) != cudaSuccess) return cudaGetLastError();
  dw_reduce_kernel<<<rgrid, 256, 0, s>>>(dw_part, dw, rows, n);
  return cudaGetLastError();
}

}  // namespace kimi
