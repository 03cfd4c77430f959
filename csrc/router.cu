// Stable LatentMoE router: sigmoid scores, biased top-(k[+1]) selection, unbiased
// renormalised weights and the per-expert load histogram, one warp per token.
// Selection is k rounds of a warp arg-max over the lanes' candidates; among equal biased
// scores the lowest expert index wins.
#include "common.cuh"
#include "device_info.h"
#include "kernels.h"

namespace kimi {
namespace {

constexpr int kMaxPerLane = 32;  // experts <= 1024
constexpr int kMaxTopK = 32;

template <typename T>
__global__ void router_kernel(const T* __restrict__ logits, const float* __restrict__ bias, int64_t rows,
                              int experts, int k, bool need_cutoff, float eps, int64_t* __restrict__ sel,
                              float* __restrict__ raw_sel, float* __restrict__ weights, float* __restrict__ cutoff,
                              unsigned long long* __restrict__ load, float* __restrict__ raw_out) {
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int per_lane = (experts + 31) / 32;
  for (int64_t row = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); row < rows; row += (int64_t)gridDim.x * wpb) {
    float raw[kMaxPerLane], biased[kMaxPerLane];
    unsigned taken = 0u;
    for (int i = 0; i < per_lane; ++i) {
      const int e = lane + i * 32;
      if (e < experts) {
        raw[i] = sigmoidf_(to_f<T>(logits[row * experts + e]));
        biased[i] = raw[i] + bias[e];
        if (raw_out) raw_out[row * experts + e] = raw[i];
      } else {
        raw[i] = 0.f;
        biased[i] = -INFINITY;
        taken |= 1u << i;
      }
    }
    const int rounds = k + (need_cutoff ? 1 : 0);
    float my_raw[kMaxTopK];
    int my_idx[kMaxTopK];
    float total = 0.f;
    for (int r = 0; r < rounds; ++r) {
      // local best among this lane's untaken candidates
      float bv = -INFINITY;
      int bi = 0x7fffffff, bslot = -1;
      for (int i = 0; i < per_lane; ++i) {
        if (taken & (1u << i)) continue;
        const int e = lane + i * 32;
        if (biased[i] > bv || (biased[i] == bv && e < bi)) {
          bv = biased[i];
          bi = e;
          bslot = i;
        }
      }
      // warp arg-max (value desc, index asc)
      float wv = bv;
      int wi = bi;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, wv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, wi, o);
        if (ov > wv || (ov == wv && oi < wi)) {
          wv = ov;
          wi = oi;
        }
      }
      const int owner = wi & 31;
      float rv = 0.f;
      if (lane == owner && bslot >= 0 && bi == wi) {
        taken |= 1u << bslot;
        rv = raw[bslot];
      }
      rv = __shfl_sync(0xffffffffu, rv, owner);
      if (r < k) {
        my_raw[r] = rv;
        my_idx[r] = wi;
        total += rv;
      } else if (lane == 0) {
        cutoff[row] = wv;
      }
    }
    const float denom = fmaxf(total, eps);
    if (lane < k) {
      float rv = 0.f;
      int iv = 0;
      for (int r = 0; r < k; ++r)
        if (r == lane) { rv = my_raw[r]; iv = my_idx[r]; }
      sel[row * k + lane] = iv;
      raw_sel[row * k + lane] = rv;
      weights[row * k + lane] = rv / denom;
      atomicAdd(&load[iv], 1ull);
    }
  }
}

}  // namespace

cudaError_t router_topk(int dtype, const void* logits, const float* bias, int64_t rows, int experts, int k,
                        bool need_cutoff, float eps, int64_t* sel, float* raw_sel, float* weights, float* cutoff,
                        int64_t* load, float* raw_out, cudaStream_t s) {
  if (experts > 32 * kMaxPerLane || k < 1 || k + 1 > kMaxTopK || k > experts) return cudaErrorInvalidValue;
  const int threads = 256;
  int64_t grid = (rows + 7) / 8;
  if (grid > device_sms() * 16) grid = device_sms() * 16;
  if (grid < 1) grid = 1;
  switch (dtype) {
    case 0: router_kernel<float><<<grid, threads, 0, s>>>((const float*)logits, bias, rows, experts, k, need_cutoff,
                                                         eps, sel, raw_sel, weights, cutoff,
                                                         (unsigned long long*)load, raw_out); break;
    case 1: router_kernel<__nv_bfloat16><<<grid, threads, 0, s>>>((const __nv_bfloat16*)logits, bias, rows, experts,
                                                                 k, need_cutoff, eps, sel, raw_sel, weights, cutoff,
                                                                 (unsigned long long*)load, raw_out); break;
    case 2: router_kernel<__half><<<grid, threads, 0, s>>>((const __half*)logits, bias, rows, experts, k,
                                                          need_cutoff, eps, sel, raw_sel, weights, cutoff,
                                                          (unsigned long long*)load, raw_out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace kimi
