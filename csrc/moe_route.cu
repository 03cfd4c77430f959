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

// One warp per row.
template <typename T>
__global__ void dy_kernel(const float* __restrict__ dagg, const int* __restrict__ row_token,
                          const float* __restrict__ row_weight, const T* __restrict__ y, T* __restrict__ dy,
                          float* __restrict__ dw_row, int64_t r_max, int L) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < r_max;
       r += (int64_t)gridDim.x * (blockDim.x >> 5)) {
    const int t = row_token[r];
    float acc = 0.f;
    if (t >= 0) {
      const float w = row_weight[r];
      for (int c = lane; c < L; c += 32) {
        const float g = dagg[(int64_t)t * L + c];
        acc += g * to_f<T>(y[r * L + c]);
        dy[r * L + c] = from_f<T>(w * g);
      }
    } else {
      for (int c = lane; c < L; c += 32) dy[r * L + c] = from_f<T>(0.f);
    }
    acc = warp_sum(acc);
    if (lane == 0) dw_row[r] = t >= 0 ? acc : 0.f;
  }
}

template <typename T, typename TO>
__global__ void slot_sum_kernel(const T* __restrict__ dxs, const int* __restrict__ row_of, TO* __restrict__ out,
                                int64_t M, int k, int L) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < M * L; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i / L;
    const int c = (int)(i % L);
    float acc = 0.f;
    for (int j = 0; j < k; ++j) {
      const int r = row_of[t * k + j];
      if (r >= 0) acc += to_f<T>(dxs[(int64_t)r * L + c]);
    }
    out[i] = from_f<TO>(acc);
  }
}

template <typename T>
__global__ void situ_bwd_cat_kernel(const T* __restrict__ dh, const T* __restrict__ g, const T* __restrict__ u,
                                    T* __restrict__ dgu, int64_t rows, int H, float bg, float bu) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * H; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / H;
    const int c = (int)(i % H);
    const float gv = to_f<T>(g[i]), uv = to_f<T>(u[i]), d = to_f<T>(dh[i]);
    const float tg = tanhf(gv / bg), tu = tanhf(uv / bu), sg = sigmoidf_(gv);
    const float cg = bg * tg, cu = bu * tu;
    dgu[r * 2 * H + c] = from_f<T>(d * cu * ((1.f - tg * tg) * sg + cg * sg * (1.f - sg)));
    dgu[r * 2 * H + H + c] = from_f<T>(d * cg * sg * (1.f - tu * tu));
  }
}

int grid_of(int64_t n, int threads) {
  int64_t g = (n + threads - 1) / threads;
  if (g > 148 * 16) g = 148 * 16;
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
  dy_kernel<__nv_bfloat16><<<grid_of(r_max * 32, 256), 256, 0, s>>>(dagg, row_token, row_weight,
                                                                    (const __nv_bfloat16*)y, (__nv_bfloat16*)dy,
                                                                    dw_row, r_max, L);
  return cudaGetLastError();
}

cudaError_t moe_slot_sum(const void* dxs, const int* row_of, void* out, bool out_fp32, int64_t M, int k, int L,
                         cudaStream_t s) {
  if (out_fp32)
    slot_sum_kernel<__nv_bfloat16, float><<<grid_of(M * L, 256), 256, 0, s>>>((const __nv_bfloat16*)dxs, row_of,
                                                                             (float*)out, M, k, L);
  else
    slot_sum_kernel<__nv_bfloat16, __nv_bfloat16><<<grid_of(M * L, 256), 256, 0, s>>>(
        (const __nv_bfloat16*)dxs, row_of, (__nv_bfloat16*)out, M, k, L);
  return cudaGetLastError();
}

cudaError_t situ_bwd_cat(const void* dh, const void* g, const void* u, void* dgu, int64_t rows, int H, float bg,
                         float bu, cudaStream_t s) {
  situ_bwd_cat_kernel<__nv_bfloat16><<<grid_of(rows * H, 256), 256, 0, s>>>(
      (const __nv_bfloat16*)dh, (const __nv_bfloat16*)g, (const __nv_bfloat16*)u, (__nv_bfloat16*)dgu, rows, H, bg,
      bu);
  return cudaGetLastError();
}

}  // namespace kimi
