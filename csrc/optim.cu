// Fused Muon passes around the batched Newton-Schulz GEMMs (one bucket of equal-shape matrices).
//
//   muon_momentum:  mom = momentum * mom + g;  raw = g + momentum * mom (Nesterov) or mom;
//                   x = bf16(raw);  sumsq[m] += ||raw_m||^2           (one pass over g and mom)
//   muon_normalize: x_m *= 1 / max(||raw_m||, eps)                    (bf16 in place)
//   muon_apply:     p_m = p_m * (1 - lr wd) - lr * scale * [||raw_m|| > eps] * o_m, with the
//                   per-matrix sums of squares of o_m, of the update and of p_m (before the
//                   update) for the optimizer statistics                (one pass over o and p)
//
// A matrix m is `mn` consecutive elements of the bucket; grid = (blocks per matrix, matrices).
// A device `skip` flag (non-finite gradients) leaves the momentum untouched and zeroes the update
// without a host branch; `lr` is a device scalar so CUDA-graph replays see the scheduler's value.
// Parity: the Muon update of `training/optimizer/muon.py` (reference) with the bucketed batching
// of this framework's optimizer.
#include "common.cuh"
#include "device_info.h"
#include "kernels.h"

namespace kimi {
namespace {

constexpr int kThreads = 256;

KIMI_D float block_reduce_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = 0.f;
  if (warp == 0) {
    r = lane < (int)(blockDim.x >> 5) ? scratch[lane] : 0.f;
    r = warp_sum(r);
  }
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kThreads) muon_momentum_kernel(const float* __restrict__ g, float* __restrict__ mom,
                                                                 __nv_bfloat16* __restrict__ x,
                                                                 float* __restrict__ sumsq, int64_t mn,
                                                                 float momentum, bool nesterov,
                                                                 const bool* __restrict__ skip) {
  __shared__ float scratch[kThreads / 32];
  const int m = blockIdx.y;
  const bool sk = skip != nullptr && *skip;
  const float mu = sk ? 1.f : momentum, gs = sk ? 0.f : 1.f;
  const float* gm = g + (int64_t)m * mn;
  float* mm = mom + (int64_t)m * mn;
  __nv_bfloat16* xm = x + (int64_t)m * mn;
  float acc = 0.f;
  const int64_t n4 = mn / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 gv = reinterpret_cast<const float4*>(gm)[i];
    float4 mv = reinterpret_cast<float4*>(mm)[i];
    const float ga[4] = {gv.x * gs, gv.y * gs, gv.z * gs, gv.w * gs};
    float ma[4] = {mv.x, mv.y, mv.z, mv.w}, ra[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      ma[u] = mu * ma[u] + ga[u];
      ra[u] = nesterov ? ga[u] + momentum * ma[u] : ma[u];
      acc += ra[u] * ra[u];
    }
    reinterpret_cast<float4*>(mm)[i] = make_float4(ma[0], ma[1], ma[2], ma[3]);
    __nv_bfloat162* xp = reinterpret_cast<__nv_bfloat162*>(xm + 4 * i);
    xp[0] = __floats2bfloat162_rn(ra[0], ra[1]);
    xp[1] = __floats2bfloat162_rn(ra[2], ra[3]);
  }
  for (int64_t i = n4 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < mn;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gv = gm[i] * gs;
    const float mv = mu * mm[i] + gv;
    const float r = nesterov ? gv + momentum * mv : mv;
    mm[i] = mv;
    xm[i] = __float2bfloat16_rn(r);
    acc += r * r;
  }
  acc = block_reduce_sum(acc, scratch);
  if (threadIdx.x == 0) atomicAdd(&sumsq[m], acc);
}

__global__ void __launch_bounds__(kThreads) muon_normalize_kernel(__nv_bfloat16* __restrict__ x,
                                                                  const float* __restrict__ sumsq, int64_t mn,
                                                                  float eps) {
  const int m = blockIdx.y;
  const float inv = 1.f / fmaxf(sqrtf(sumsq[m]), eps);
  __nv_bfloat162* xm = reinterpret_cast<__nv_bfloat162*>(x + (int64_t)m * mn);
  const int64_t n2 = mn / 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  // eight values (16 bytes) per step when the matrix starts on a 16-byte boundary
  const bool vec = (mn & 7) == 0 && (reinterpret_cast<uintptr_t>(xm) & 15) == 0;
  const int64_t n8 = vec ? mn / 8 : 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += stride) {
    uint4 raw = reinterpret_cast<uint4*>(xm)[i];
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 f = __bfloat1622float2(h[u]);
      h[u] = __floats2bfloat162_rn(f.x * inv, f.y * inv);
    }
    reinterpret_cast<uint4*>(xm)[i] = raw;
  }
  for (int64_t i = n8 * 4 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n2; i += stride) {
    float2 f = __bfloat1622float2(xm[i]);
    xm[i] = __floats2bfloat162_rn(f.x * inv, f.y * inv);
  }
  if ((mn & 1) && blockIdx.x == 0 && threadIdx.x == 0) {
    __nv_bfloat16* last = x + (int64_t)m * mn + mn - 1;
    *last = __float2bfloat16_rn(__bfloat162float(*last) * inv);
  }
}

// stats[m] = {||o_m||^2, ||update_m||^2, ||p_m||^2 before the update}
__global__ void __launch_bounds__(kThreads) muon_apply_kernel(const __nv_bfloat16* __restrict__ o,
                                                              float* const* __restrict__ params,
                                                              const float* __restrict__ sumsq, int64_t mn,
                                                              const float* __restrict__ lr, float wd, float scale,
                                                              float eps, const bool* __restrict__ skip,
                                                              float* __restrict__ stats) {
  __shared__ float scratch[kThreads / 32];
  const int m = blockIdx.y;
  const bool sk = skip != nullptr && *skip;
  const float lr_eff = sk ? 0.f : *lr;
  const float keep = sqrtf(sumsq[m]) > eps ? 1.f : 0.f;
  const float decay = 1.f - lr_eff * wd;
  const float coef = -lr_eff * scale * keep;
  const __nv_bfloat16* om = o + (int64_t)m * mn;
  float* pm = params[m];
  float so = 0.f, su = 0.f, sp = 0.f;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t t0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  // four elements per step (16-byte parameter and 8-byte update accesses) when aligned
  const bool vec = (mn & 3) == 0 && (reinterpret_cast<uintptr_t>(pm) & 15) == 0;
  const int64_t nv = vec ? mn / 4 : 0;
  for (int64_t i = t0; i < nv; i += stride) {
    const uint2 raw = reinterpret_cast<const uint2*>(om)[i];
    const float2 o01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
    const float2 o23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
    const float ov[4] = {o01.x, o01.y, o23.x, o23.y};
    float4 pv = reinterpret_cast<float4*>(pm)[i];
    float pa[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float o = ov[u] * keep;
      so += o * o;
      sp += pa[u] * pa[u];
      const float up = o * scale;
      su += up * up;
      pa[u] = pa[u] * decay + coef * ov[u];
    }
    reinterpret_cast<float4*>(pm)[i] = make_float4(pa[0], pa[1], pa[2], pa[3]);
  }
  for (int64_t i = nv * 4 + t0; i < mn; i += stride) {
    const float ov = __bfloat162float(om[i]) * keep;
    const float pv = pm[i];
    so += ov * ov;
    sp += pv * pv;
    const float up = ov * scale;
    su += up * up;
    pm[i] = pv * decay + coef * __bfloat162float(om[i]);
  }
  so = block_reduce_sum(so, scratch);
  su = block_reduce_sum(su, scratch);
  sp = block_reduce_sum(sp, scratch);
  if (threadIdx.x == 0) {
    atomicAdd(&stats[3 * m], so);
    atomicAdd(&stats[3 * m + 1], su);
    atomicAdd(&stats[3 * m + 2], sp);
  }
}

int blocks_per_matrix(int64_t mn) {
  const int64_t per = (int64_t)kThreads * 8;
  int64_t b = (mn + per - 1) / per;
  return (int)(b < 1 ? 1 : (b > 64 ? 64 : b));
}

// bf16 mirrors of fp32 tensors (one launch for a whole table).  `vec_off[t]` is the first 8-element
// vector of tensor t in a virtual concatenation (prefix sums of ceil(numel / 8)); a thread converts
// one vector: 32 bytes read, 16 bytes written.
__global__ void __launch_bounds__(kThreads) cast_bf16_multi_kernel(const float* const* __restrict__ src,
                                                                   __nv_bfloat16* const* __restrict__ dst,
                                                                   const int64_t* __restrict__ numel,
                                                                   const int64_t* __restrict__ vec_off, int tensors) {
  const int64_t total = vec_off[tensors];
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    int lo = 0, hi = tensors - 1;  // last t with vec_off[t] <= v
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (vec_off[mid] <= v) lo = mid;
      else hi = mid - 1;
    }
    const int64_t e = (v - vec_off[lo]) * 8, n = numel[lo];
    const float* sp = src[lo] + e;
    __nv_bfloat16* dp = dst[lo] + e;
    if (e + 8 <= n) {
      const float4 a = reinterpret_cast<const float4*>(sp)[0], b = reinterpret_cast<const float4*>(sp)[1];
      Vec<__nv_bfloat16> o;
      o.v[0] = __float2bfloat16_rn(a.x); o.v[1] = __float2bfloat16_rn(a.y);
      o.v[2] = __float2bfloat16_rn(a.z); o.v[3] = __float2bfloat16_rn(a.w);
      o.v[4] = __float2bfloat16_rn(b.x); o.v[5] = __float2bfloat16_rn(b.y);
      o.v[6] = __float2bfloat16_rn(b.z); o.v[7] = __float2bfloat16_rn(b.w);
      o.store(dp);
    } else {
      for (int64_t i = 0; e + i < n; ++i) dp[i] = __float2bfloat16_rn(sp[i]);
    }
  }
}

// Newton-Schulz polynomial of a batch of Gram matrices: P = c * G2 + b * G + a * I (bf16 in and out,
// fp32 arithmetic, one rounding).  G and G2 are [batch * m, m] row-major; one thread per 8 columns.
__global__ void __launch_bounds__(kThreads) ns_poly_kernel(const __nv_bfloat16* __restrict__ g,
                                                           const __nv_bfloat16* __restrict__ g2,
                                                           __nv_bfloat16* __restrict__ out, int64_t rows, int m,
                                                           float a, float b, float c) {
  const int per_row = m >> 3;
  const int64_t total = rows * per_row;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = v / per_row;
    const int c0 = (int)(v - r * per_row) * 8;
    const int diag = (int)(r % m);
    Vec<__nv_bfloat16> x, y, o;
    x.load(g + r * m + c0);
    y.load(g2 + r * m + c0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float val = c * __bfloat162float(y.v[i]) + b * __bfloat162float(x.v[i]);
      if (c0 + i == diag) val += a;
      o.v[i] = __float2bfloat16_rn(val);
    }
    o.store(out + r * m + c0);
  }
}

}  // namespace

cudaError_t ns_poly(const void* g, const void* g2, void* out, int64_t rows, int m, float a, float b, float c,
                    cudaStream_t s) {
  if (rows <= 0 || m <= 0) return cudaSuccess;
  if ((m & 7) || (reinterpret_cast<uintptr_t>(g) & 15) || (reinterpret_cast<uintptr_t>(g2) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    return cudaErrorInvalidValue;
  int64_t blocks = (rows * (m >> 3) + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)device_sms() * 16;
  if (blocks > cap) blocks = cap;
  ns_poly_kernel<<<(int)blocks, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(g),
                                                  static_cast<const __nv_bfloat16*>(g2),
                                                  static_cast<__nv_bfloat16*>(out), rows, m, a, b, c);
  return cudaGetLastError();
}

cudaError_t cast_bf16_multi(const float* const* src, void* const* dst, const int64_t* numel, const int64_t* vec_off,
                            int tensors, int64_t total_vec, cudaStream_t s) {
  if (tensors <= 0 || total_vec <= 0) return cudaSuccess;
  int64_t blocks = (total_vec + kThreads - 1) / kThreads;
  const int64_t cap = (int64_t)device_sms() * 16;
  if (blocks > cap) blocks = cap;
  cast_bf16_multi_kernel<<<(int)blocks, kThreads, 0, s>>>(src, reinterpret_cast<__nv_bfloat16* const*>(dst), numel,
                                                          vec_off, tensors);
  return cudaGetLastError();
}

cudaError_t muon_momentum(const float* g, float* mom, void* x_bf16, float* sumsq, int count, int64_t mn,
                          float momentum, bool nesterov, const bool* skip, cudaStream_t s) {
  if (count <= 0 || mn <= 0 || (reinterpret_cast<uintptr_t>(g) & 15) || (reinterpret_cast<uintptr_t>(mom) & 15) ||
      (reinterpret_cast<uintptr_t>(x_bf16) & 7) || ((mn & 3) && count > 1))
    return cudaErrorInvalidValue;
  const dim3 grid(blocks_per_matrix(mn), count);
  muon_momentum_kernel<<<grid, kThreads, 0, s>>>(g, mom, reinterpret_cast<__nv_bfloat16*>(x_bf16), sumsq, mn,
                                                  momentum, nesterov, skip);
  return cudaGetLastError();
}

cudaError_t muon_normalize(void* x_bf16, const float* sumsq, int count, int64_t mn, float eps, cudaStream_t s) {
  if (count <= 0 || mn <= 0 || ((mn & 1) && count > 1)) return cudaErrorInvalidValue;
  const dim3 grid(blocks_per_matrix(mn), count);
  muon_normalize_kernel<<<grid, kThreads, 0, s>>>(reinterpret_cast<__nv_bfloat16*>(x_bf16), sumsq, mn, eps);
  return cudaGetLastError();
}

cudaError_t muon_apply(const void* o_bf16, float* const* params, const float* sumsq, int count, int64_t mn,
                       const float* lr, float wd, float scale, float eps, const bool* skip, float* stats,
                       cudaStream_t s) {
  if (count <= 0 || mn <= 0) return cudaErrorInvalidValue;
  const dim3 grid(blocks_per_matrix(mn), count);
  muon_apply_kernel<<<grid, kThreads, 0, s>>>(reinterpret_cast<const __nv_bfloat16*>(o_bf16), params, sumsq, mn, lr,
                                               wd, scale, eps, skip, stats);
  return cudaGetLastError();
}

}  // namespace kimi
