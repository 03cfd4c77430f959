// Device-side routing for the grouped expert GEMMs (no host synchronisation, static shapes).
//
//   moe_route_prep:  per-expert counts -> 128-row aligned segment offsets -> for every (token, slot)
//                    a row in its expert's segment (row_token / row_weight per row, row_of per slot).
//                    Rows that carry no assignment keep row_token = -1.
//   moe_gather:      xs[row] = latent[row_token[row]] (zeros for padding rows)
//   moe_dy:          dY[row] = w[row] * dagg[tok]; dw_row[row] = <dagg[tok], Y[row]>
//   moe_slot_sum:    dlatent[t] = sum_j dxs[row_of[t, j]]
//   situ_bwd_cat:    [dGate | dUp] of the SiTU-GLU into one [R, 2H] buffer
// Buffers have R_max = M*k + E*128 rows so the launch shape never depends on the routing.
#include "common.cuh"
#include "device_info.h"
#include "moe_route.h"

namespace kimi {
namespace {

constexpr int kAlign = 128;

__global__ void init_kernel(int* counts, int E, int* row_token, int64_t r_max) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < r_max; i += (int64_t)gridDim.x * blockDim.x)
    row_token[i] = -1;
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[e] = 0;
}

__global__ void count_kernel(const int64_t* __restrict__ sel, int64_t n, int E, int* counts) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = sel[i];
    if (e >= 0 && e < E) atomicAdd(&counts[e], 1);
  }
}

// Single block: exclusive scan of aligned counts; cursors start at the segment bases.
__global__ void scan_kernel(const int* __restrict__ counts, int E, int* offsets, int* cursor) {
  __shared__ int s[1024];
  int running = 0;
  for (int base = 0; base < E; base += blockDim.x) {
    const int e = base + threadIdx.x;
    const int v = e < E ? (counts[e] + kAlign - 1) / kAlign * kAlign : 0;
    s[threadIdx.x] = v;
    __syncthreads();
    for (int o = 1; o < blockDim.x; o <<= 1) {
      const int add = threadIdx.x >= o ? s[threadIdx.x - o] : 0;
      __syncthreads();
      s[threadIdx.x] += add;
      __syncthreads();
    }
    if (e < E) {
      offsets[e] = running + s[threadIdx.x] - v;
      cursor[e] = offsets[e];
    }
    running += s[blockDim.x - 1];
    __syncthreads();
  }
  if (threadIdx.x == 0) offsets[E] = running;
}

__global__ void assign_kernel(const int64_t* __restrict__ sel, const float* __restrict__ w, int64_t n, int E,
                              int k, int* cursor, int* row_token, float* row_weight, int* row_of) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = sel[i];
    if (e < 0 || e >= E) {
      row_of[i] = -1;
      continue;
    }
    const int pos = atomicAdd(&cursor[e], 1);
    row_token[pos] = (int)(i / k);
    row_weight[pos] = w[i];
    row_of[i] = pos;
  }
}

template <typename T>
__global__ void gather_kernel(const T* __restrict__ latent, const int* __restrict__ row_token, T* __restrict__ xs,
                              int64_t r_max, int L) {
  constexpr int VN = Vec<T>::N;
  const int nv = L / VN;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < r_max * nv;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nv;
    const int c = (int)(i % nv);
    const int t = row_token[r];
    Vec<T> v;
    if (t >= 0) {
      v.load(latent + (int64_t)t * L + c * VN);
    } else {
#pragma unroll
      for (int j = 0; j < VN; ++j) v.v[j] = from_f<T>(0.f);
    }
    v.store(xs + r * L + c * VN);
  }
}

// One warp per row; each lane handles 8 consecutive columns per step (two float4 of dagg, one
// 16-byte vector of y and of dy).
template <typename T>
__global__ void dy_kernel(const float* __restrict__ dagg, const int* __restrict__ row_token,
                          const float* __restrict__ row_weight, const T* __restrict__ y, T* __restrict__ dy,
                          float* __restrict__ dw_row, int64_t r_max, int L) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < r_max;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int t = row_token[r];
    float acc = 0.f;
    const float w = t >= 0 ? row_weight[r] : 0.f;
    for (int c = lane * 8; c < L; c += 256) {
      Vec<T> out;
      if (t >= 0) {
        const float4 g0 = *reinterpret_cast<const float4*>(dagg + (int64_t)t * L + c);
        const float4 g1 = *reinterpret_cast<const float4*>(dagg + (int64_t)t * L + c + 4);
        Vec<T> yv;
        yv.load(y + r * L + c);
        const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          acc += gv[e] * yv.f(e);
          out.set(e, w * gv[e]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) out.set(e, 0.f);
      }
      out.store(dy + r * L + c);
    }
    acc = warp_sum(acc);
    if (lane == 0) dw_row[r] = t >= 0 ? acc : 0.f;
  }
}

// 8 columns of one token per thread: sum of its k slot rows.
template <typename T, typename TO>
__global__ void slot_sum_kernel(const T* __restrict__ dxs, const int* __restrict__ row_of, TO* __restrict__ out,
                                int64_t M, int k, int L) {
  const int nv = L / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < M * nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / nv;
    const int c = (int)(i % nv) * 8;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int r = row_of[t * k + j];
      if (r < 0) continue;
      Vec<T> v;
      v.load(dxs + (int64_t)r * L + c);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v.f(e);
    }
    TO* o = out + t * L + c;
    if constexpr (sizeof(TO) == 4) {
      reinterpret_cast<float4*>(o)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      reinterpret_cast<float4*>(o)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      Vec<TO> v;
#pragma unroll
      for (int e = 0; e < 8; ++e) v.set(e, acc[e]);
      v.store(o);
    }
  }
}

// 8 consecutive hidden units per thread (H % 8 == 0): one 16-byte load of each input and one
// 16-byte store into each half of the [dGate | dUp] row.
template <typename T>
__global__ void situ_bwd_cat_kernel(const T* __restrict__ dh, const T* __restrict__ g, const T* __restrict__ u,
                                    T* __restrict__ dgu, int64_t rows, int H, float bg, float bu) {
  const int nv = H / 8;
  const float ibg = 1.f / bg, ibu = 1.f / bu;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / nv;
    const int c = (int)(i % nv) * 8;
    const int64_t src = r * H + c;
    Vec<T> gv, uv, dv, og, ou;
    gv.load(g + src);
    uv.load(u + src);
    dv.load(dh + src);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float gg = gv.f(e), uu = uv.f(e), d = dv.f(e);
      const float tg = tanhf(gg * ibg), tu = tanhf(uu * ibu), sg = sigmoidf_(gg);
      const float cg = bg * tg, cu = bu * tu;
      og.set(e, d * cu * ((1.f - tg * tg) * sg + cg * sg * (1.f - sg)));
      ou.set(e, d * cg * sg * (1.f - tu * tu));
    }
    og.store(dgu + r * 2 * H + c);
    ou.store(dgu + r * 2 * H + H + c);
  }
}

int grid_of(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  if (g > (int64_t)device_sms() * 16) g = (int64_t)device_sms() * 16;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace

cudaError_t moe_route_prep(const int64_t* sel, const float* w, int64_t M, int k, int E, int64_t r_max, int* counts,
                           int* offsets, int* cursor, int* row_token, float* row_weight, int* row_of,
                           cudaStream_t s) {
  if (E > 1024 * 64) return cudaErrorInvalidValue;
  init_kernel<<<grid_of(r_max, 256), 256, 0, s>>>(counts, E, row_token, r_max);
  count_kernel<<<grid_of(M * k, 256), 256, 0, s>>>(sel, M * k, E, counts);
  scan_kernel<<<1, 1024, 0, s>>>(counts, E, offsets, cursor);
  assign_kernel<<<grid_of(M * k, 256), 256, 0, s>>>(sel, w, M * k, E, k, cursor, row_token, row_weight, row_of);
  return cudaGetLastError();
}

cudaError_t moe_gather(const void* latent, const int* row_token, void* xs, int64_t r_max, int L, cudaStream_t s) {
  if (L % 8) return cudaErrorInvalidValue;
  gather_kernel<__nv_bfloat16><<<grid_of(r_max * L / 8, 256), 256, 0, s>>>(
      (const __nv_bfloat16*)latent, row_token, (__nv_bfloat16*)xs, r_max, L);
  return cudaGetLastError();
}

cudaError_t moe_dy(const float* dagg, const int* row_token, const float* row_weight, const void* y, void* dy,
                   float* dw_row, int64_t r_max, int L, cudaStream_t s) {
  if (L % 8) return cudaErrorInvalidValue;
  dy_kernel<__nv_bfloat16><<<grid_of(r_max * 32, 256), 256, 0, s>>>(dagg, row_token, row_weight,
                                                                    (const __nv_bfloat16*)y, (__nv_bfloat16*)dy,
                                                                    dw_row, r_max, L);
  return cudaGetLastError();
}

cudaError_t moe_slot_sum(const void* dxs, const int* row_of, void* out, bool out_fp32, int64_t M, int k, int L,
                         cudaStream_t s) {
  if (L % 8) return cudaErrorInvalidValue;
  if (out_fp32)
    slot_sum_kernel<__nv_bfloat16, float><<<grid_of(M * L / 8, 256), 256, 0, s>>>((const __nv_bfloat16*)dxs, row_of,
                                                                             (float*)out, M, k, L);
  else
    slot_sum_kernel<__nv_bfloat16, __nv_bfloat16><<<grid_of(M * L / 8, 256), 256, 0, s>>>(
        (const __nv_bfloat16*)dxs, row_of, (__nv_bfloat16*)out, M, k, L);
  return cudaGetLastError();
}

cudaError_t situ_bwd_cat(const void* dh, const void* g, const void* u, void* dgu, int64_t rows, int H, float bg,
                         float bu, cudaStream_t s) {
  if (H % 8) return cudaErrorInvalidValue;
  situ_bwd_cat_kernel<__nv_bfloat16><<<grid_of(rows * H / 8, 256), 256, 0, s>>>(
      (const __nv_bfloat16*)dh, (const __nv_bfloat16*)g, (const __nv_bfloat16*)u, (__nv_bfloat16*)dgu, rows, H, bg,
      bu);
  return cudaGetLastError();
}

}  // namespace kimi
