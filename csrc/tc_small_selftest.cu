// Self-test of the small-matrix tcgen05 path (tc_small.cuh): the operand writer, the tf32
// MMA at several N, K slices and B row offsets, and the TMEM read-back.
//   mode 0: out[128 x n] = A[128 x K] B[n x K]^T                   (n <= 256, K in {32,64,128})
//   mode 1: out[:, 64 I + c] = A[:, 16I:16I+16] B[c, 16I:16I+16]^T  (four K slices, n = 64, K = 64)
//   mode 2: out[:, 16 J + c] = A B[16J + c, :]^T                     (four row offsets, N = 16 each)
#include "kernels.h"
#include "tc_small.cuh"
#include "device_info.h"

namespace kimi {
namespace {

__global__ void __launch_bounds__(128) tcs_selftest_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                           float* __restrict__ out, int K, int n, int mode,
                                                           int* status) {
  extern __shared__ uint8_t raw[];
  float* sA = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  float* sB = sA + 128 * K;
  __shared__ uint64_t bar;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5;
  const int nb = mode == 0 ? n : 64;
  for (int idx = threadIdx.x; idx < 128 * K; idx += blockDim.x) tcs::st(sA, 128, idx / K, idx % K, A[idx]);
  for (int idx = threadIdx.x; idx < nb * K; idx += blockDim.x) tcs::st(sB, nb, idx / K, idx % K, B[idx]);
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_barrier_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(&slot, 256);
    tc::tmem_relinquish();
  }
  tcs::operands_ready();
  const uint32_t tm = slot;
  if (threadIdx.x == 0) {
    if (mode == 0) {
      tcs::mma_rows128(tm, sA, 128, sB, nb, 0, n, 0, K, false);
    } else if (mode == 1) {
      for (int I = 0; I < 4; ++I) tcs::mma_rows128(tm + 64 * I, sA, 128, sB, nb, 0, 64, 16 * I, 16, false);
    } else {
      for (int J = 0; J < 4; ++J) tcs::mma_rows128(tm + 16 * J, sA, 128, sB, nb, 16 * J, 16, 0, K, false);
    }
    tc::mma_commit(&bar);
  }
  uint32_t phase = 0;
  tcs::mma_done(&bar, phase, status, 1);
  const int ncols = mode == 0 ? n : (mode == 1 ? 256 : 64);
  for (int c0 = 0; c0 < ncols; c0 += 32) {
    float v[32];
    tcs::tmem_row32(tm, warp, c0, v);
    for (int i = 0; i < 32; ++i)
      if (c0 + i < ncols) out[(int64_t)threadIdx.x * ncols + c0 + i] = v[i];
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (warp == 0) tc::tmem_dealloc(tm, 256);
}

}  // namespace

cudaError_t tcs_selftest(const float* A, const float* B, float* out, int K, int n, int mode, int* status,
                         cudaStream_t s) {
  if (K % 32 || K > 128 || n % 16 || n > 256 || mode < 0 || mode > 2) return cudaErrorInvalidValue;
  if (mode != 0 && K != 64) return cudaErrorInvalidValue;
  const int nb = mode == 0 ? n : 64;
  const size_t smem = 1024 + (size_t)(128 + nb) * K * 4;
  cudaError_t e = ensure_dynamic_smem(tcs_selftest_kernel, (int)smem);
  if (e != cudaSuccess) return e;
  tcs_selftest_kernel<<<1, 128, smem, s>>>(A, B, out, K, n, mode, status);
  return cudaGetLastError();
}

}  // namespace kimi
