// Memory-bound fused kernels: RMSNorm (plain and head-wise), SiTU-GLU, sigmoid gate,
// KDA lower-bounded decay (the short causal conv + SiLU + head norm lives in conv.cu).
//
// Rows are processed by groups of `tpr` threads (a power of two <= 32) so that narrow
// rows (head_dim 64) still keep a warp busy; 16-byte vector loads are used when the row
// width is a multiple of the vector width. All math is fp32; storage rounding follows
// the PyTorch reference (normalised value rounded to the activation dtype before the
// affine multiply).
#include <algorithm>

#include "common.cuh"
#include "device_info.h"
#include "kernels.h"

namespace kimi {
namespace {

int pick_tpr(int nvec) {
  int t = 1;
  while (t < nvec && t < 32) t <<= 1;
  return t;
}

int grid_for(int64_t work_items, int per_block) {
  int64_t g = (work_items + per_block - 1) / per_block;
  const int64_t cap = (int64_t)device_sms() * 16;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return (int)g;
}

// ------------------------------------------------------------------ RMSNorm
template <typename T>
__global__ void rms_fwd_kernel(const T* __restrict__ x, const float* __restrict__ w, T* __restrict__ y,
                               float* __restrict__ rstd, int64_t rows, int dim, int period, float eps, int tpr) {
  constexpr int VN = Vec<T>::N;
  const int nvec = dim / VN;
  const int gid = threadIdx.x / tpr, lane = threadIdx.x % tpr;
  const int rpb = blockDim.x / tpr;
  const int warp_first_gid = (threadIdx.x / 32) * (32 / tpr);
  for (int64_t base = (int64_t)blockIdx.x * rpb; base + warp_first_gid < rows; base += (int64_t)gridDim.x * rpb) {
    const int64_t row = base + gid;
    const bool ok = row < rows;
    const T* xr = x + row * dim;
    float ss = 0.f;
    if (ok)
      for (int i = lane; i < nvec; i += tpr) {
        Vec<T> a;
        a.load(xr + i * VN);
#pragma unroll
        for (int j = 0; j < VN; ++j) ss += a.f(j) * a.f(j);
      }
    ss = group_sum(ss, tpr);
    const float r = rsqrtf(ss / dim + eps);
    if (ok) {
      if (lane == 0 && rstd) rstd[row] = r;
      const float* wr = w ? w + (int64_t)(row % period) * dim : nullptr;
      T* yr = y + row * dim;
      for (int i = lane; i < nvec; i += tpr) {
        Vec<T> a, o;
        a.load(xr + i * VN);
#pragma unroll
        for (int j = 0; j < VN; ++j) {
          float n = round_through<T>(a.f(j) * r);
          if (wr) n = n * round_through<T>(wr[i * VN + j]);
          o.set(j, n);
        }
        o.store(yr + i * VN);
      }
    }
  }
}

// dx = r * (dn - xhat * mean(dn * xhat)),  dn = dy * w ; dw[p, d] += dy * n
template <typename T>
__global__ void rms_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ x, const float* __restrict__ w,
                               const float* __restrict__ rstd, T* __restrict__ dx, float* __restrict__ dw,
                               int64_t rows, int dim, int period, int tpr) {
  constexpr int VN = Vec<T>::N;
  extern __shared__ float sdw[];  // period * dim accumulators
  const int nvec = dim / VN;
  const int gid = threadIdx.x / tpr, lane = threadIdx.x % tpr;
  const int rpb = blockDim.x / tpr;
  const int warp_first_gid = (threadIdx.x / 32) * (32 / tpr);
  if (dw)
    for (int i = threadIdx.x; i < period * dim; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
  for (int64_t base = (int64_t)blockIdx.x * rpb; base + warp_first_gid < rows; base += (int64_t)gridDim.x * rpb) {
    const int64_t row = base + gid;
    const bool ok = row < rows;
    const T* xr = x + row * dim;
    const T* dyr = dy + row * dim;
    const int p = ok ? (int)(row % period) : 0;
    const float* wr = w ? w + (int64_t)p * dim : nullptr;
    const float r = ok ? rstd[row] : 0.f;
    float dot = 0.f;
    if (ok)
      for (int i = lane; i < nvec; i += tpr) {
        Vec<T> a, g;
        a.load(xr + i * VN);
        g.load(dyr + i * VN);
#pragma unroll
        for (int j = 0; j < VN; ++j) {
          const float wv = wr ? round_through<T>(wr[i * VN + j]) : 1.f;
          dot += g.f(j) * wv * a.f(j) * r;
        }
      }
    dot = group_sum(dot, tpr) / dim;
    if (ok) {
      T* dxr = dx + row * dim;
      for (int i = lane; i < nvec; i += tpr) {
        Vec<T> a, g, o;
        a.load(xr + i * VN);
        g.load(dyr + i * VN);
#pragma unroll
        for (int j = 0; j < VN; ++j) {
          const float wv = wr ? round_through<T>(wr[i * VN + j]) : 1.f;
          const float xh = a.f(j) * r;
          o.set(j, r * (g.f(j) * wv - xh * dot));
          if (dw) atomicAdd(&sdw[p * dim + i * VN + j], g.f(j) * round_through<T>(xh));
        }
        o.store(dxr + i * VN);
      }
    }
  }
  __syncthreads();
  if (dw)
    for (int i = threadIdx.x; i < period * dim; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

// Per-channel weight (period 1) and rows of at most 32 * MAXV vectors: one warp per row keeps x and dy
// in registers for both passes, and each lane accumulates its channels' dw partials in registers
// over all the rows it visits (no shared-memory atomics); one block-level reduction at the end.
template <typename T, int MAXV>
__global__ void __launch_bounds__(256) rms_bwd_warp_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                           const float* __restrict__ w,
                                                           const float* __restrict__ rstd, T* __restrict__ dx,
                                                           float* __restrict__ dw, int64_t rows, int dim) {
  constexpr int VN = Vec<T>::N;
  extern __shared__ float sdw[];  // dim
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, wpb = blockDim.x >> 5;
  const int nvec = dim / VN;
  float wv[MAXV][VN], acc[MAXV][VN];
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int vi = lane + 32 * v;
#pragma unroll
    for (int j = 0; j < VN; ++j) {
      wv[v][j] = (w && vi < nvec) ? round_through<T>(w[vi * VN + j]) : 1.f;
      acc[v][j] = 0.f;
    }
  }
  for (int64_t row = (int64_t)blockIdx.x * wpb + warp; row < rows; row += (int64_t)gridDim.x * wpb) {
    const T* xr = x + row * dim;
    const T* dyr = dy + row * dim;
    const float r = rstd[row];
    Vec<T> xa[MAXV], ga[MAXV];
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int vi = lane + 32 * v;
      if (vi < nvec) {
        xa[v].load(xr + vi * VN);
        ga[v].load(dyr + vi * VN);
#pragma unroll
        for (int j = 0; j < VN; ++j) dot += ga[v].f(j) * wv[v][j] * xa[v].f(j) * r;
      }
    }
    dot = warp_sum(dot) / dim;
    T* dxr = dx + row * dim;
#pragma unroll
    for (int v = 0; v < MAXV; ++v) {
      const int vi = lane + 32 * v;
      if (vi < nvec) {
        Vec<T> o;
#pragma unroll
        for (int j = 0; j < VN; ++j) {
          const float xh = xa[v].f(j) * r;
          o.set(j, r * (ga[v].f(j) * wv[v][j] - xh * dot));
          acc[v][j] += ga[v].f(j) * round_through<T>(xh);
        }
        o.store(dxr + vi * VN);
      }
    }
  }
  if (!dw) return;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) sdw[i] = 0.f;
  __syncthreads();
#pragma unroll
  for (int v = 0; v < MAXV; ++v) {
    const int vi = lane + 32 * v;
    if (vi < nvec)
#pragma unroll
      for (int j = 0; j < VN; ++j) atomicAdd(&sdw[vi * VN + j], acc[v][j]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < dim; i += blockDim.x) atomicAdd(&dw[i], sdw[i]);
}

// ------------------------------------------------------------------ SiTU-GLU and sigmoid gate
template <typename T>
__global__ void situ_fwd_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ y, int64_t n,
                                float bg, float bu) {
  constexpr int VN = Vec<T>::N;
  const int64_t nv = n / VN;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    Vec<T> a, b, o;
    a.load(g + i * VN);
    b.load(u + i * VN);
#pragma unroll
    for (int j = 0; j < VN; ++j) {
      const float gv = a.f(j), uv = b.f(j);
      o.set(j, bg * tanhf(gv / bg) * sigmoidf_(gv) * bu * tanhf(uv / bu));
    }
    o.store(y + i * VN);
  }
  for (int64_t i = nv * VN + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gv = to_f<T>(g[i]), uv = to_f<T>(u[i]);
    y[i] = from_f<T>(bg * tanhf(gv / bg) * sigmoidf_(gv) * bu * tanhf(uv / bu));
  }
}

template <typename T>
KIMI_D void situ_grad(float gv, float uv, float d, float bg, float bu, float& dg, float& du) {
  const float tg = tanhf(gv / bg), tu = tanhf(uv / bu), sg = sigmoidf_(gv);
  const float cg = bg * tg, cu = bu * tu;
  dg = d * cu * ((1.f - tg * tg) * sg + cg * sg * (1.f - sg));
  du = d * cg * sg * (1.f - tu * tu);
}

template <typename T>
__global__ void situ_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ g, const T* __restrict__ u,
                                T* __restrict__ dg, T* __restrict__ du, int64_t n, float bg, float bu) {
  constexpr int VN = Vec<T>::N;
  const int64_t nv = n / VN;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    Vec<T> a, b, d, og, ou;
    a.load(g + i * VN);
    b.load(u + i * VN);
    d.load(dy + i * VN);
#pragma unroll
    for (int j = 0; j < VN; ++j) {
      float x0, x1;
      situ_grad<T>(a.f(j), b.f(j), d.f(j), bg, bu, x0, x1);
      og.set(j, x0);
      ou.set(j, x1);
    }
    og.store(dg + i * VN);
    ou.store(du + i * VN);
  }
  for (int64_t i = nv * VN + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float x0, x1;
    situ_grad<T>(to_f<T>(g[i]), to_f<T>(u[i]), to_f<T>(dy[i]), bg, bu, x0, x1);
    dg[i] = from_f<T>(x0);
    du[i] = from_f<T>(x1);
  }
}

template <typename T>
__global__ void sigmul_fwd_kernel(const T* __restrict__ z, const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    y[i] = from_f<T>(round_through<T>(sigmoidf_(to_f<T>(z[i]))) * to_f<T>(x[i]));
}

template <typename T>
__global__ void sigmul_bwd_kernel(const T* __restrict__ dy, const T* __restrict__ z, const T* __restrict__ x,
                                  T* __restrict__ dz, T* __restrict__ dx, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float s = sigmoidf_(to_f<T>(z[i])), d = to_f<T>(dy[i]);
    dz[i] = from_f<T>(d * to_f<T>(x[i]) * s * (1.f - s));
    dx[i] = from_f<T>(d * s);
  }
}

// ------------------------------------------------------------------ KDA decay gate
// g = g_min * clamp(sigmoid(exp(A_log[h]) * z), eps, 1-eps)  (fp32 output)
template <typename T>
__global__ void decay_fwd_kernel(const T* __restrict__ z, const float* __restrict__ a_log, float* __restrict__ g,
                                 int64_t n, int heads, int kdim, float g_min, float ceps) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int h = (int)((i / kdim) % heads);
    const float p = sigmoidf_(expf(a_log[h]) * to_f<T>(z[i]));
    g[i] = g_min * fminf(fmaxf(p, ceps), 1.f - ceps);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) decay_bwd_kernel(const float* __restrict__ dg, const T* __restrict__ z,
                                                        const float* __restrict__ a_log, T* __restrict__ dz,
                                                        float* __restrict__ da_log, int64_t n, int heads, int kdim,
                                                        float g_min, float ceps) {
  // 8 consecutive elements per thread (kdim % 64 == 0: they share one head); the lanes of a head
  // (kdim / 8 of them, contiguous) reduce with shuffles, one shared atomic per head segment, and
  // the grid is capped so each block flushes its per-head partials once.
  extern __shared__ float sda[];
  for (int i = threadIdx.x; i < heads; i += blockDim.x) sda[i] = 0.f;
  __syncthreads();
  const int seg = kdim / 8 < 32 ? kdim / 8 : 32;  // lanes per head segment inside a warp
  const int64_t nv = n / 8;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < nv; base += (int64_t)gridDim.x * blockDim.x) {
    const int64_t v = base + threadIdx.x;
    float part = 0.f;
    int h = 0;
    if (v < nv) {
      const int64_t i0 = v * 8;
      h = (int)((i0 / kdim) % heads);
      const float sc = expf(a_log[h]);
      float zv[8], gv[8];
      if constexpr (sizeof(T) == 4) {
        const float4 z0 = reinterpret_cast<const float4*>(z)[2 * v], z1 = reinterpret_cast<const float4*>(z)[2 * v + 1];
        zv[0] = z0.x; zv[1] = z0.y; zv[2] = z0.z; zv[3] = z0.w; zv[4] = z1.x; zv[5] = z1.y; zv[6] = z1.z; zv[7] = z1.w;
      } else {
        Vec<T> zz;
        zz.load(z + i0);
#pragma unroll
        for (int j = 0; j < 8; ++j) zv[j] = zz.f(j);
      }
      const float4 g0 = reinterpret_cast<const float4*>(dg)[2 * v], g1 = reinterpret_cast<const float4*>(dg)[2 * v + 1];
      gv[0] = g0.x; gv[1] = g0.y; gv[2] = g0.z; gv[3] = g0.w; gv[4] = g1.x; gv[5] = g1.y; gv[6] = g1.z; gv[7] = g1.w;
      float out[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float p = sigmoidf_(sc * zv[j]);
        const bool inside = p > ceps && p < 1.f - ceps;
        const float dpre = inside ? gv[j] * g_min * p * (1.f - p) : 0.f;  // d/d(sc*z)
        out[j] = dpre * sc;
        part += dpre * zv[j] * sc;
      }
      if constexpr (sizeof(T) == 4) {
        reinterpret_cast<float4*>(dz)[2 * v] = make_float4(out[0], out[1], out[2], out[3]);
        reinterpret_cast<float4*>(dz)[2 * v + 1] = make_float4(out[4], out[5], out[6], out[7]);
      } else {
        Vec<T> o;
#pragma unroll
        for (int j = 0; j < 8; ++j) o.set(j, out[j]);
        o.store(dz + i0);
      }
    }
    part = group_sum(part, seg);
    if (v < nv && (threadIdx.x % seg) == 0) atomicAdd(&sda[h], part);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < heads; i += blockDim.x) atomicAdd(&da_log[i], sda[i]);
}

}  // namespace

#define KIMI_DISPATCH(dtype, T, ...)                       \
  switch (dtype) {                                         \
    case 0: { using T = float; __VA_ARGS__; break; }       \
    case 1: { using T = __nv_bfloat16; __VA_ARGS__; break; } \
    case 2: { using T = __half; __VA_ARGS__; break; }      \
    default: return cudaErrorInvalidValue;                 \
  }

cudaError_t rms_norm_fwd(int dtype, const void* x, const float* w, void* y, float* rstd, int64_t rows, int dim,
                         int period, float eps, cudaStream_t s) {
  KIMI_DISPATCH(dtype, T, {
    if (dim % Vec<T>::N) return cudaErrorInvalidValue;
    const int tpr = pick_tpr(dim / Vec<T>::N);
    const int threads = 256;
    rms_fwd_kernel<T><<<grid_for(rows, threads / tpr), threads, 0, s>>>(
        (const T*)x, w, (T*)y, rstd, rows, dim, period < 1 ? 1 : period, eps, tpr);
  });
  return cudaGetLastError();
}

cudaError_t rms_norm_bwd(int dtype, const void* dy, const void* x, const float* w, const float* rstd, void* dx,
                         float* dw, int64_t rows, int dim, int period, cudaStream_t s) {
  KIMI_DISPATCH(dtype, T, {
    if (dim % Vec<T>::N) return cudaErrorInvalidValue;
    const int tpr = pick_tpr(dim / Vec<T>::N);
    const int threads = 256;
    const int p = period < 1 ? 1 : period;
    const size_t smem = dw ? (size_t)p * dim * sizeof(float) : 0;
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    // The dw partials are flushed once per block: keep the grid near 4 blocks per SM so the
    // global atomics per weight element stay in the hundreds.
    int grid = grid_for(rows, threads / tpr);
    if (dw && grid > device_sms() * 4) grid = device_sms() * 4;
    const int nvec = dim / Vec<T>::N;
    if (p == 1 && nvec <= 32 * 4) {
      // 4-warp blocks (the wide instances hold well over 128 registers per thread, so occupancy comes
      // in block steps).  With dw, every block ends with one global atomic per weight element: four
      // such blocks per SM keep those few hundred per element (32 warps per SM made the flush, not
      // the rows, the cost)
      const int wgrid = (int)std::min<int64_t>((rows + 3) / 4, dw ? device_sms() * 4 : device_sms() * 16);
      const size_t wsmem = dw ? (size_t)dim * sizeof(float) : 0;
      if (nvec <= 32)
        rms_bwd_warp_kernel<T, 1><<<wgrid, 128, wsmem, s>>>((const T*)dy, (const T*)x, w, rstd, (T*)dx, dw, rows, dim);
      else if (nvec <= 64)
        rms_bwd_warp_kernel<T, 2><<<wgrid, 128, wsmem, s>>>((const T*)dy, (const T*)x, w, rstd, (T*)dx, dw, rows, dim);
      else if (nvec <= 96)  // d_model 640 / 768 in bf16: no idle vector slot per lane
        rms_bwd_warp_kernel<T, 3><<<wgrid, 128, wsmem, s>>>((const T*)dy, (const T*)x, w, rstd, (T*)dx, dw, rows, dim);
      else
        rms_bwd_warp_kernel<T, 4><<<wgrid, 128, wsmem, s>>>((const T*)dy, (const T*)x, w, rstd, (T*)dx, dw, rows, dim);
      break;
    }
    rms_bwd_kernel<T><<<grid, threads, smem, s>>>(
        (const T*)dy, (const T*)x, w, rstd, (T*)dx, dw, rows, dim, p, tpr);
  });
  return cudaGetLastError();
}

cudaError_t situ_glu_fwd(int dtype, const void* g, const void* u, void* y, int64_t n, float bg, float bu,
                         cudaStream_t s) {
  KIMI_DISPATCH(dtype, T, {
    situ_fwd_kernel<T><<<grid_for(n / Vec<T>::N + 1, 256), 256, 0, s>>>((const T*)g, (const T*)u, (T*)y, n, bg, bu);
  });
  return cudaGetLastError();
}

cudaError_t situ_glu_bwd(int dtype, const void* dy, const void* g, const void* u, void* dg, void* du, int64_t n,
                         float bg, float bu, cudaStream_t s) {
  KIMI_DISPATCH(dtype, T, {
    situ_bwd_kernel<T><<<grid_for(n / Vec<T>::N + 1, 256), 256, 0, s>>>((const T*)dy, (const T*)g, (const T*)u,
                                                                       (T*)dg, (T*)du, n, bg, bu);
  });
  return cudaGetLastError();
}

cudaError_t sigmoid_mul_fwd(int dtype, const void* z, const void* x, void* y, int64_t n, cudaStream_t s) {
  KIMI_DISPATCH(dtype, T, { sigmul_fwd_kernel<T><<<grid_for(n, 256), 256, 0, s>>>((const T*)z, (const T*)x, (T*)y, n); });
  return cudaGetLastError();
}

cudaError_t sigmoid_mul_bwd(int dtype, const void* dy, const void* z, const void* x, void* dz, void* dx, int64_t n,
                            cudaStream_t s) {
  KIMI_DISPATCH(dtype, T, {
    sigmul_bwd_kernel<T><<<grid_for(n, 256), 256, 0, s>>>((const T*)dy, (const T*)z, (const T*)x, (T*)dz, (T*)dx, n);
  });
  return cudaGetLastError();
}

cudaError_t kda_decay_fwd(int dtype, const void* z, const float* a_log, float* g, int64_t rows, int heads, int kdim,
                          float g_min, float ceps, cudaStream_t s) {
  const int64_t n = rows * heads * kdim;
  KIMI_DISPATCH(dtype, T, {
    decay_fwd_kernel<T><<<grid_for(n, 256), 256, 0, s>>>((const T*)z, a_log, g, n, heads, kdim, g_min, ceps);
  });
  return cudaGetLastError();
}

cudaError_t kda_decay_bwd(int dtype, const float* dg, const void* z, const float* a_log, void* dz, float* da_log,
                          int64_t rows, int heads, int kdim, float g_min, float ceps, cudaStream_t s) {
  const int64_t n = rows * heads * kdim;
  if (kdim % 64) return cudaErrorInvalidValue;
  KIMI_DISPATCH(dtype, T, {
    const int grid = (int)std::min<int64_t>(grid_for(n / 8, 256), device_sms() * 4);
    decay_bwd_kernel<T><<<grid, 256, heads * sizeof(float), s>>>(dg, (const T*)z, a_log, (T*)dz, da_log, n, heads,
                                                                 kdim, g_min, ceps);
  });
  return cudaGetLastError();
}

}  // namespace kimi
