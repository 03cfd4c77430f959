// Cross-entropy over vocabulary rows, fused with its own gradient.
// For each row: lse = logsumexp(logits), loss = lse - logits[target] (valid rows only), and
// the logits buffer is overwritten in place with d(loss)/d(logits) * grad_scale
// = (softmax - onehot) * grad_scale (zero for invalid rows). The caller then runs the two
// backward GEMMs on that buffer, so the fp32 [N,V] probability tensor never exists.
//
// 16-bit rows up to 96K entries take the staged path: one persistent CTA per SM double-buffers
// whole rows in shared memory with a TMA bulk copy (cp.async.bulk global -> shared, completion on
// an mbarrier; no multicast), so the max / sum / gradient passes read shared memory and HBM sees
// each logit read once and written once.  Other rows use the two-pass kernel below.
#include "common.cuh"
#include "device_info.h"
#include "kernels.h"
#include "tc_common.cuh"

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

constexpr int kStagedThreads = 512;
constexpr int kMaxStagedBytes = 100 * 1024;  // per buffer; two buffers per CTA

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   tc::smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
               : "memory");
}

constexpr float kLog2e = 1.4426950408889634f;  // log2(e)
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__global__ void __launch_bounds__(kStagedThreads, 1) ce_rows_staged_kernel(T* __restrict__ logits, int64_t ld,
                                                                           int64_t rows, int vocab,
                                                                           const int64_t* __restrict__ targets,
                                                                           const bool* __restrict__ valid,
                                                                           float* __restrict__ loss_rows,
                                                                           float grad_scale, uint32_t row_bytes) {
  extern __shared__ __align__(128) uint8_t sbuf[];
  __shared__ uint64_t bars[2];
  __shared__ float scratch[32];
  constexpr int VN = Vec<T>::N;
  T* buf[2] = {reinterpret_cast<T*>(sbuf), reinterpret_cast<T*>(sbuf + row_bytes)};
  const int tid = threadIdx.x;
  if (tid == 0) {
    tc::mbar_init(&bars[0], 1);
    tc::mbar_init(&bars[1], 1);
    tc::fence_barrier_init();
  }
  __syncthreads();
  int64_t row = blockIdx.x;
  if (tid == 0 && row < rows) {
    tc::mbar_arrive_expect_tx(&bars[0], row_bytes);
    bulk_g2s(buf[0], logits + row * ld, row_bytes, &bars[0]);
  }
  const int nv = vocab / VN;
  for (int it = 0; row < rows; row += gridDim.x, ++it) {
    const int b = it & 1;
    const int64_t next = row + gridDim.x;
    if (tid == 0 && next < rows) {  // the other buffer was released by the barrier ending the last row
      tc::fence_proxy_async();
      tc::mbar_arrive_expect_tx(&bars[b ^ 1], row_bytes);
      bulk_g2s(buf[b ^ 1], logits + next * ld, row_bytes, &bars[b ^ 1]);
    }
    tc::mbar_wait_local(&bars[b], (uint32_t)((it >> 1) & 1), nullptr, 0);
    const T* sr = buf[b];
    float m = -INFINITY;
    for (int i = tid; i < nv; i += kStagedThreads) {
      Vec<T> a;
      a.load(sr + i * VN);
#pragma unroll
      for (int j = 0; j < VN; ++j) m = fmaxf(m, a.f(j));
    }
    for (int i = nv * VN + tid; i < vocab; i += kStagedThreads) m = fmaxf(m, to_f<T>(sr[i]));
    const float gm = block_max(m, scratch);
    // e^{x - m} as 2^{(x - m) log2 e} on the hardware exp2 (relative error near 2^-22): the row's
    // two exponential passes are what bounds this kernel
    const float gml = gm * kLog2e;
    float se = 0.f;
    for (int i = tid; i < nv; i += kStagedThreads) {
      Vec<T> a;
      a.load(sr + i * VN);
#pragma unroll
      for (int j = 0; j < VN; ++j) se += exp2_approx(fmaf(a.f(j), kLog2e, -gml));
    }
    for (int i = nv * VN + tid; i < vocab; i += kStagedThreads) se += expf(to_f<T>(sr[i]) - gm);
    const float lse = gm + logf(block_sum(se, scratch));
    const bool ok = valid == nullptr || valid[row];
    const int64_t tgt = ok ? targets[row] : -1;
    if (tid == 0) loss_rows[row] = (ok && tgt >= 0 && tgt < vocab) ? lse - to_f<T>(sr[tgt]) : 0.f;
    const float sc = ok ? grad_scale : 0.f;
    const float lsel = lse * kLog2e;
    T* gr = logits + row * ld;
    for (int i = tid; i < nv; i += kStagedThreads) {
      Vec<T> a;
      a.load(sr + i * VN);
#pragma unroll
      for (int j = 0; j < VN; ++j) {
        const int64_t col = (int64_t)i * VN + j;
        a.set(j, sc * (exp2_approx(fmaf(a.f(j), kLog2e, -lsel)) - (col == tgt ? 1.f : 0.f)));
      }
      a.store(gr + i * VN);
    }
    for (int i = nv * VN + tid; i < vocab; i += kStagedThreads)
      gr[i] = from_f<T>(sc * (expf(to_f<T>(sr[i]) - lse) - (i == tgt ? 1.f : 0.f)));
    __syncthreads();  // every thread is done with buf[b] before it is refilled two rows later
  }
}

}  // namespace

cudaError_t ce_rows_fwd_bwd(int dtype, void* logits, int64_t ld, int64_t rows, int vocab, const int64_t* targets,
                            const bool* valid, float* loss_rows, float grad_scale, cudaStream_t s) {
  if (dtype == 1 || dtype == 2) {
    const uint32_t row_bytes = (uint32_t)(((int64_t)vocab * 2 + 15) / 16 * 16);
    const bool aligned = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (ld * 2) % 16 == 0 &&
                         (int64_t)row_bytes <= ld * 2;
    if (aligned && row_bytes <= (uint32_t)kMaxStagedBytes && rows > 0) {
      const size_t smem = 2 * (size_t)row_bytes;
      const int sms = device_sms();
      const int grid = (int)(rows < sms ? rows : sms);
      {  // the attribute covers the largest staged row
        const cudaError_t e = dtype == 1 ? ensure_dynamic_smem(ce_rows_staged_kernel<__nv_bfloat16>,
                                                               2 * kMaxStagedBytes)
                                         : ensure_dynamic_smem(ce_rows_staged_kernel<__half>, 2 * kMaxStagedBytes);
        if (e != cudaSuccess) return e;
      }
      if (dtype == 1) {
        ce_rows_staged_kernel<__nv_bfloat16><<<grid, kStagedThreads, smem, s>>>(
            (__nv_bfloat16*)logits, ld, rows, vocab, targets, valid, loss_rows, grad_scale, row_bytes);
      } else {
        ce_rows_staged_kernel<__half><<<grid, kStagedThreads, smem, s>>>((__half*)logits, ld, rows, vocab, targets,
                                                                        valid, loss_rows, grad_scale, row_bytes);
      }
      return cudaGetLastError();
    }
  }
  const int64_t cap = (int64_t)device_sms() * 8;
  int64_t grid = rows < cap ? rows : cap;
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
