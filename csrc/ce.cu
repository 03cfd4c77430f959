// Cross-entropy over vocabulary rows, fused with its own gradient.
// For each row: lse = logsumexp(logits), loss = lse - logits[target] (valid rows only), and
// the logits buffer is overwritten in place with d(loss)/d(logits) * grad_scale
// = (softmax - onehot) * grad_scale (zero for invalid rows). The caller then runs the two
// backward GEMMs on that buffer, so the fp32 [N,V] probability tensor never exists.
#include "common.cuh"
#include "kernels.h"

namespace kimi {
namespace {

template <typename T>
__global__ void ce_rows_kernel(T* __restrict__ logits, int64_t ld, int64_t rows, int vocab,
                               const int64_t* __restrict__ targets, const bool* __restrict__ valid,
                               float* __restrict__ loss_rows, float grad_scale) {
  __shared__ float scratch[32];
  constexpr int VN = Vec<T>::N;
  const bool vec_ok = ((ld * sizeof(T)) % 16 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    T* lr = logits + row * ld;
    const bool ok = valid == nullptr || valid[row];
    // pass 1: online max / sum of exponentials
    float m = -INFINITY, s = 0.f;
    const int nv = vec_ok ? vocab / VN : 0;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      Vec<T> a;
      a.load(lr + i * VN);
#pragma unroll
      for (int j = 0; j < VN; ++j) {
        const float x = a.f(j);
        if (x > m) {
          s = s * expf(m - x) + 1.f;
          m = x;
        } else {
          s += expf(x - m);
        }
      }
    }
    for (int i = nv * VN + threadIdx.x; i < vocab; i += blockDim.x) {
      const float x = to_f<T>(lr[i]);
      if (x > m) {
        s = s * expf(m - x) + 1.f;
        m = x;
      } else {
        s += expf(x - m);
      }
    }
    const float gm = block_max(m, scratch);
    const float part = (m == -INFINITY) ? 0.f : s * expf(m - gm);
    const float gs = block_sum(part, scratch);
    const float lse = gm + logf(gs);
    const int64_t tgt = ok ? targets[row] : -1;
    if (threadIdx.x == 0) {
      float lv = 0.f;
      if (ok && tgt >= 0 && tgt < vocab) lv = lse - to_f<T>(lr[tgt]);
      loss_rows[row] = lv;
    }
    __syncthreads();  // every thread has read lr[tgt] through pass 1 before it is overwritten
    // pass 2: gradient in place
    const float sc = ok ? grad_scale : 0.f;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      Vec<T> a;
      a.load(lr + i * VN);
#pragma unroll
      for (int j = 0; j < VN; ++j) {
        const int64_t col = (int64_t)i * VN + j;
        const float p = expf(a.f(j) - lse);
        a.set(j, sc * (p - (col == tgt ? 1.f : 0.f)));
      }
      a.store(lr + i * VN);
    }
    for (int i = nv * VN + threadIdx.x; i < vocab; i += blockDim.x) {
      const float p = expf(to_f<T>(lr[i]) - lse);
      lr[i] = from_f<T>(sc * (p - (i == tgt ? 1.f : 0.f)));
    }
    __syncthreads();
  }
}

}  // namespace

cudaError_t ce_rows_fwd_bwd(int dtype, void* logits, int64_t ld, int64_t rows, int vocab, const int64_t* targets,
                            const bool* valid, float* loss_rows, float grad_scale, cudaStream_t s) {
  int64_t grid = rows < 148 * 8 ? rows : 148 * 8;
  if (grid < 1) grid = 1;
  switch (dtype) {
    case 0: ce_rows_kernel<float><<<grid, 512, 0, s>>>((float*)logits, ld, rows, vocab, targets, valid, loss_rows,
                                                      grad_scale); break;
    case 1: ce_rows_kernel<__nv_bfloat16><<<grid, 512, 0, s>>>((__nv_bfloat16*)logits, ld, rows, vocab, targets,
                                                              valid, loss_rows, grad_scale); break;
    case 2: ce_rows_kernel<__half><<<grid, 512, 0, s>>>((__half*)logits, ld, rows, vocab, targets, valid, loss_rows,
                                                       grad_scale); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace kimi
