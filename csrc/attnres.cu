// Attention-residual depth mixing: for each token, softmax over S depth sources of
//   logit_s = q . (RMSNorm(src_s) * w)
// and an fp32 weighted sum of the raw sources. One warp per token; each source tensor is
// read through its own pointer (no stacked copy), once for the logits and once for the sum
// (once in all when there are at most four sources).
#include <algorithm>

#include "common.cuh"
#include "device_info.h"
#include "kernels.h"

namespace kimi {
namespace {

constexpr int kMaxSources = 16;

template <typename T>
struct SrcPtrs {
  const T* p[kMaxSources];
};
template <typename T>
struct DstPtrs {
  T* p[kMaxSources];
};

int grid_tokens(int64_t tokens, int warps_per_block) {
  int64_t g = (tokens + warps_per_block - 1) / warps_per_block;
  const int64_t cap = (int64_t)device_sms() * 8;
  if (g > cap) g = cap;
  return (int)(g < 1 ? 1 : g);
}

// Sources are processed in groups (four rows, two for very wide rows): the rows of a group are
// loaded together (several loads in flight per lane), and the per-source scalars (logit, rstd,
// probability, partial dots) live in lane s of the warp (S <= 16 < 32) and are broadcast with
// shuffles -- no per-thread arrays indexed by a runtime source number.  With at most one group of
// sources, the rows loaded for the logits are reused for the weighted sum.
template <int MAXV>
struct Group {
  static constexpr int n = MAXV >= 8 ? 2 : 4;  // fewer rows in flight for wide rows (register budget)
};

template <typename T, int MAXV, int NG = Group<MAXV>::n>
KIMI_D void load_group(Vec<T> (&xb)[NG][MAXV], const SrcPtrs<T>& src, int s0, int S, int64_t tok,
                       int dim, int lane, int nvec) {
  constexpr int VN = Vec<T>::N;
#pragma unroll
  for (int u = 0; u < NG; ++u) {
    if (s0 + u < S) {
      const T* row = src.p[s0 + u] + tok * dim;
#pragma unroll
      for (int v = 0; v < MAXV; ++v) {
        const int vi = lane + v * 32;
        if (vi < nvec) xb[u][v].load(row + vi * VN);
      }
    }
  }
}

template <typename T, int MAXV>
__global__ void attnres_fwd_kernel(const __grid_constant__ SrcPtrs<T> src, int S, const float* __restrict__ q,
                                   const float* __restrict__ w,
                                   T* __restrict__ out, float* __restrict__ probs, float* __restrict__ rstd,
                                   int64_t tokens, int dim, float eps) {
  constexpr int VN = Vec<T>::N;
  constexpr int kGroup = Group<MAXV>::n;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int nvec = dim / VN;
  float qw[MAXV][VN];
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int vi = lane + v * 32;
#pragma unroll
    for (int j = 0; j < VN; ++j) qw[v][j] = vi < nvec ? q[vi * VN + j] * w[vi * VN + j] : 0.f;
  }
  const float inv_dim = 1.f / dim;
  for (int64_t tok = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); tok < tokens; tok += (int64_t)gridDim.x * wpb) {
    float my_logit = -INFINITY, my_r = 0.f;  // lane s: source s
    Vec<T> xb[kGroup][MAXV];
    for (int s0 = 0; s0 < S; s0 += kGroup) {
      load_group<T, MAXV>(xb, src, s0, S, tok, dim, lane, nvec);
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        float ss = 0.f, a = 0.f;
        if (s0 + u < S) {
#pragma unroll
          for (int v = 0; v < MAXV; ++v) {
            if (lane + v * 32 < nvec) {
#pragma unroll
              for (int j = 0; j < VN; ++j) {
                const float xv = xb[u][v].f(j);
                ss += xv * xv;
                a += qw[v][j] * xv;
              }
            }
          }
        }
        ss = warp_sum(ss);
        a = warp_sum(a);
        if (lane == s0 + u) {
          my_r = rsqrtf(ss * inv_dim + eps);
          my_logit = my_r * a;
        }
      }
    }
    const float mx = warp_max(lane < S ? my_logit : -INFINITY);
    const float e = lane < S ? expf(my_logit - mx) : 0.f;
    const float my_p = e / warp_sum(e);
    if (lane < S) {
      probs[tok * S + lane] = my_p;
      rstd[tok * S + lane] = my_r;
    }
    float acc[MAXV][VN];
#pragma unroll
    for (int v = 0; v < MAXV; ++v)
#pragma unroll
      for (int j = 0; j < VN; ++j) acc[v][j] = 0.f;
    for (int s0 = 0; s0 < S; s0 += kGroup) {
      if (S > kGroup) load_group<T, MAXV>(xb, src, s0, S, tok, dim, lane, nvec);
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        if (s0 + u < S) {
          const float pu = __shfl_sync(0xffffffffu, my_p, s0 + u);
#pragma unroll
          for (int v = 0; v < MAXV; ++v)
#pragma unroll
            for (int j = 0; j < VN; ++j) acc[v][j] += pu * xb[u][v].f(j);
        }
      }
    }
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int vi = lane + v * 32;
      if (vi < nvec) {
        Vec<T> o;
#pragma unroll
        for (int j = 0; j < VN; ++j) o.set(j, acc[v][j]);
        o.store(out + tok * dim + vi * VN);
      }
    }
  }
}

template <typename T, int MAXV>
__global__ void attnres_bwd_kernel(const __grid_constant__ SrcPtrs<T> src, int S, const float* __restrict__ q,
                                   const float* __restrict__ w, const T* __restrict__ dout,
                                   const float* __restrict__ probs, const float* __restrict__ rstd,
                                   const __grid_constant__ DstPtrs<T> dsrc, float* __restrict__ dq,
                                   float* __restrict__ dw, int64_t tokens, int dim) {
  constexpr int VN = Vec<T>::N;
  // two source rows in flight in the backward (it also holds the output-gradient row and the
  // dq / dw accumulators): fewer registers, one more resident block per SM
  constexpr int kGroup = MAXV >= 3 ? 2 : Group<MAXV>::n;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int nvec = dim / VN;
  // dq_d = w_d * C_d and dw_d = q_d * C_d with C_d = sum dlogit * r * x_d: one accumulator.
  float qw[MAXV][VN], acc[MAXV][VN];
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int vi = lane + v * 32;
#pragma unroll
    for (int j = 0; j < VN; ++j) {
      qw[v][j] = vi < nvec ? q[vi * VN + j] * w[vi * VN + j] : 0.f;
      acc[v][j] = 0.f;
    }
  }
  const float inv_dim = 1.f / dim;
  for (int64_t tok = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); tok < tokens; tok += (int64_t)gridDim.x * wpb) {
    // the output gradient row, read once for all sources and both passes
    Vec<T> gv[MAXV];
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int vi = lane + v * 32;
      if (vi < nvec) gv[v].load(dout + tok * dim + vi * VN);
    }
    const float my_p = lane < S ? probs[tok * S + lane] : 0.f;
    const float my_r = lane < S ? rstd[tok * S + lane] : 0.f;
    float my_dp = 0.f, my_a = 0.f;
    Vec<T> xb[kGroup][MAXV];
    for (int s0 = 0; s0 < S; s0 += kGroup) {
      load_group<T, MAXV, kGroup>(xb, src, s0, S, tok, dim, lane, nvec);
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        float d0 = 0.f, a0 = 0.f;
        if (s0 + u < S) {
#pragma unroll
          for (int v = 0; v < MAXV; ++v) {
            if (lane + v * 32 < nvec) {
#pragma unroll
              for (int j = 0; j < VN; ++j) {
                const float xv = xb[u][v].f(j);
                d0 += gv[v].f(j) * xv;
                a0 += qw[v][j] * xv;
              }
            }
          }
        }
        d0 = warp_sum(d0);
        a0 = warp_sum(a0);
        if (lane == s0 + u) {
          my_dp = d0;
          my_a = a0;
        }
      }
    }
    const float pdp = warp_sum(lane < S ? my_p * my_dp : 0.f);
    for (int s0 = 0; s0 < S; s0 += kGroup) {
      if (S > kGroup) load_group<T, MAXV, kGroup>(xb, src, s0, S, tok, dim, lane, nvec);
#pragma unroll
      for (int u = 0; u < kGroup; ++u) {
        if (s0 + u < S) {
          const int sidx = s0 + u;
          const float p = __shfl_sync(0xffffffffu, my_p, sidx), r = __shfl_sync(0xffffffffu, my_r, sidx);
          const float dl = p * (__shfl_sync(0xffffffffu, my_dp, sidx) - pdp);  // d loss / d logit_s
          const float r3 = r * r * r * __shfl_sync(0xffffffffu, my_a, sidx) * inv_dim;
          T* drow = dsrc.p[sidx] + tok * dim;
#pragma unroll
          for (int v = 0; v < MAXV; ++v) {
            const int vi = lane + v * 32;
            if (vi < nvec) {
              Vec<T> o;
#pragma unroll
              for (int j = 0; j < VN; ++j) {
                const float xv = xb[u][v].f(j);
                o.set(j, p * gv[v].f(j) + dl * (r * qw[v][j] - r3 * xv));
                acc[v][j] += dl * r * xv;
              }
              o.store(drow + vi * VN);
            }
          }
        }
      }
    }
  }
  // Reduce the per-warp accumulators in shared memory, then one global atomic per element
  // per block (instead of one per warp: the grid has ~1k blocks of 8 warps).
  extern __shared__ float sacc[];  // dim
  for (int i = threadIdx.x; i < dim; i += blockDim.x) sacc[i] = 0.f;
  __syncthreads();
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int vi = lane + v * 32;
    if (vi < nvec)
#pragma unroll
      for (int j = 0; j < VN; ++j) atomicAdd(&sacc[vi * VN + j], acc[v][j]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) {
    atomicAdd(&dq[i], w[i] * sacc[i]);
    atomicAdd(&dw[i], q[i] * sacc[i]);
  }
}

template <typename T>
int maxv_for(int dim) {
  const int nvec = dim / Vec<T>::N;
  const int per_lane = (nvec + 31) / 32;
  if (per_lane <= 1) return 1;
  if (per_lane <= 2) return 2;
  if (per_lane <= 3) return 3;  // d_model 640 / 768 in bf16: no idle vector slot per lane
  if (per_lane <= 4) return 4;
  if (per_lane <= 6) return 6;
  if (per_lane <= 8) return 8;
  return -1;
}

}  // namespace

#define KIMI_MAXV_SWITCH(mv, MV, ...)            \
  switch (mv) {                                  \
    case 1: { constexpr int MV = 1; __VA_ARGS__; break; } \
    case 2: { constexpr int MV = 2; __VA_ARGS__; break; } \
    case 3: { constexpr int MV = 3; __VA_ARGS__; break; } \
    case 4: { constexpr int MV = 4; __VA_ARGS__; break; } \
    case 6: { constexpr int MV = 6; __VA_ARGS__; break; } \
    case 8: { constexpr int MV = 8; __VA_ARGS__; break; } \
    default: return cudaErrorInvalidValue;       \
  }

template <typename T>
static cudaError_t fwd_impl(const void* const* sources, int S, const float* q, const float* w, void* out, float* probs,
                            float* rstd, int64_t tokens, int dim, float eps, cudaStream_t s) {
  if (S < 1 || S > kMaxSources || dim % Vec<T>::N) return cudaErrorInvalidValue;
  SrcPtrs<T> ptrs{};
  for (int i = 0; i < S; ++i) ptrs.p[i] = (const T*)sources[i];
  // 4-warp blocks: the kernels hold well over 128 registers per thread, so occupancy comes in block
  // steps; smaller blocks let three or four of them share an SM instead of one 8-warp block
  const int threads = 128;
  const int mv = maxv_for<T>(dim);
  KIMI_MAXV_SWITCH(mv, MV, {
    attnres_fwd_kernel<T, MV><<<grid_tokens(tokens, threads / 32), threads, 0, s>>>(ptrs, S, q, w, (T*)out, probs,
                                                                                    rstd, tokens, dim, eps);
  });
  return cudaGetLastError();
}

template <typename T>
static cudaError_t bwd_impl(const void* const* sources, int S, const float* q, const float* w, const void* dout,
                            const float* probs, const float* rstd, void* const* dsources, float* dq, float* dw,
                            int64_t tokens, int dim, cudaStream_t s) {
  if (S < 1 || S > kMaxSources || dim % Vec<T>::N) return cudaErrorInvalidValue;
  SrcPtrs<T> ptrs{};
  DstPtrs<T> dptrs{};
  for (int i = 0; i < S; ++i) {
    ptrs.p[i] = (const T*)sources[i];
    dptrs.p[i] = (T*)dsources[i];
  }
  const int threads = 128;
  const int mv = maxv_for<T>(dim);
  KIMI_MAXV_SWITCH(mv, MV, {
    // every block ends with 2 * dim global atomics into dq / dw: four 4-warp blocks per SM keep the
    // number per element in the hundreds
    attnres_bwd_kernel<T, MV><<<std::min(grid_tokens(tokens, threads / 32), device_sms() * 4), threads, dim * sizeof(float), s>>>(
        ptrs, S, q, w, (const T*)dout, probs, rstd, dptrs, dq, dw, tokens, dim);
  });
  return cudaGetLastError();
}

cudaError_t attnres_mix_fwd(int dtype, const void* const* sources, int S, const float* q, const float* w, void* out,
                            float* probs, float* rstd, int64_t tokens, int dim, float eps, cudaStream_t s) {
  switch (dtype) {
    case 0: return fwd_impl<float>(sources, S, q, w, out, probs, rstd, tokens, dim, eps, s);
    case 1: return fwd_impl<__nv_bfloat16>(sources, S, q, w, out, probs, rstd, tokens, dim, eps, s);
    case 2: return fwd_impl<__half>(sources, S, q, w, out, probs, rstd, tokens, dim, eps, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t attnres_mix_bwd(int dtype, const void* const* sources, int S, const float* q, const float* w,
                            const void* dout, const float* probs, const float* rstd, void* const* dsources, float* dq,
                            float* dw, int64_t tokens, int dim, cudaStream_t s) {
  switch (dtype) {
    case 0: return bwd_impl<float>(sources, S, q, w, dout, probs, rstd, dsources, dq, dw, tokens, dim, s);
    case 1: return bwd_impl<__nv_bfloat16>(sources, S, q, w, dout, probs, rstd, dsources, dq, dw, tokens, dim, s);
    case 2: return bwd_impl<__half>(sources, S, q, w, dout, probs, rstd, dsources, dq, dw, tokens, dim, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace kimi
