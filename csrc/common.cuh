// Shared device helpers for the kimi_k3_b200 sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define KIMI_HD __host__ __device__ __forceinline__
#define KIMI_D __device__ __forceinline__

namespace kimi {

// ---------------------------------------------------------------- scalar conversion
template <typename T> KIMI_D float to_f(T v);
template <> KIMI_D float to_f<float>(float v) { return v; }
template <> KIMI_D float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> KIMI_D float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> KIMI_D T from_f(float v);
template <> KIMI_D float from_f<float>(float v) { return v; }
template <> KIMI_D __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> KIMI_D __half from_f<__half>(float v) { return __float2half_rn(v); }

// Round a float through T and back (models the storage rounding of the reference).
template <typename T> KIMI_D float round_through(float v) { return to_f<T>(from_f<T>(v)); }

// ---------------------------------------------------------------- 16-byte vectors
// A Vec<T> holds 16 bytes: 8 bf16/half or 4 float.
template <typename T> struct VecTraits { static constexpr int N = 16 / sizeof(T); };

template <typename T>
struct alignas(16) Vec {
  static constexpr int N = VecTraits<T>::N;
  T v[N];
  KIMI_D void load(const T* p) { *reinterpret_cast<int4*>(v) = *reinterpret_cast<const int4*>(p); }
  KIMI_D void store(T* p) const { *reinterpret_cast<int4*>(p) = *reinterpret_cast<const int4*>(v); }
  KIMI_D float f(int i) const { return to_f<T>(v[i]); }
  KIMI_D void set(int i, float x) { v[i] = from_f<T>(x); }
};

// ---------------------------------------------------------------- reductions
KIMI_D float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
KIMI_D float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Sum over aligned groups of `width` lanes (width a power of two <= 32).
KIMI_D float group_sum(float v, int width) {
  for (int o = width >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide sum; `scratch` needs blockDim.x/32 floats. Result broadcast to all threads.
KIMI_D float block_sum(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = lane < nw ? scratch[lane] : 0.f;
  r = warp_sum(r);
  return r;
}
KIMI_D float block_max(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = lane < nw ? scratch[lane] : -INFINITY;
  r = warp_max(r);
  return r;
}

// ---------------------------------------------------------------- activations
KIMI_D float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }
KIMI_D float siluf_(float x) { return x * sigmoidf_(x); }

}  // namespace kimi

#define KIMI_CUDA_CHECK(expr)                                                      \
  do {                                                                             \
    cudaError_t _e = (expr);                                                       \
    if (_e != cudaSuccess) return _e;                                              \
  } while (0)
