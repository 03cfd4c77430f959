// Small-matrix tcgen05 building blocks (sm_100a) for chunked kernels whose operands are
// produced by the threads themselves (scaled, masked or transposed on the way into shared
// memory) rather than copied by TMA.
//
// Operand tiles are fp32 in shared memory, K-major with the 128-byte swizzle: a tile of R rows
// (R % 8 == 0) and K columns (K % 32 == 0) is K/32 "atoms" of R x 32 floats; atom a starts at
// byte a * R * 128, row r of an atom at (r / 8) * 1024 + (r % 8) * 128, and its eight 16-byte
// chunks are permuted by chunk ^ (r % 8).  This is the layout TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B, so the shared-memory descriptor is the one the bf16 GEMM uses
// (leading byte offset 16, stride byte offset 1024); a K step of 8 tf32 values is 32 bytes.
// Tile bases must be 1024-byte aligned.
//
// Products run as kind::tf32 MMAs with M = 128 (accumulator row i in TMEM lane i), fp32
// accumulation in TMEM, issued by one thread and completed through an mbarrier.  Smaller
// problems are stacked along M or N and the unused blocks of the result are ignored.
#pragma once
#include "common.cuh"
#include "tc_common.cuh"

namespace kimi {
namespace tcs {

KIMI_D uint32_t kmaj_off(int row, int k, int R) {
  const int a = k >> 5, kk = k & 31;
  return (uint32_t)(a * R * 128 + (row >> 3) * 1024 + (row & 7) * 128 + ((((kk >> 2) ^ (row & 7))) << 4) +
                    ((kk & 3) << 2));
}
KIMI_D void st(float* tile, int R, int row, int k, float v) {
  *reinterpret_cast<float*>(reinterpret_cast<char*>(tile) + kmaj_off(row, k, R)) = v;
}
// Four consecutive K values (k % 4 == 0) of one row: one 16-byte store.
KIMI_D void st4(float* tile, int R, int row, int k, float4 v) {
  *reinterpret_cast<float4*>(reinterpret_cast<char*>(tile) + kmaj_off(row, k, R)) = v;
}
KIMI_D float ld(const float* tile, int R, int row, int k) {
  return *reinterpret_cast<const float*>(reinterpret_cast<const char*>(tile) + kmaj_off(row, k, R));
}

// kind::tf32 instruction descriptor: fp32 accumulator, tf32 A and B (format 2), both K-major.
KIMI_HD uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

KIMI_D void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[128 x n] (+)= A[rows 0..127, k in [a_k0, a_k0 + kn)] * B[rows b_row0 .. b_row0 + n, k in [b_k0, b_k0 + kn)]^T.
// a_R / b_R are the row counts the tiles were written with; k offsets and kn are multiples of 8,
// b_row0 a multiple of 8.  Called by one thread.
KIMI_D void mma_rows128_ab(uint32_t tmem_d, const float* a, int a_R, int a_k0, const float* b, int b_R, int b_row0,
                           int b_k0, int n, int kn, bool accumulate) {
  const uint32_t id = idesc_tf32(128, n);
  const uint32_t a0 = tc::smem_u32(a), b0 = tc::smem_u32(b) + (uint32_t)(b_row0 >> 3) * 1024u;
  for (int k = 0; k < kn; k += 8) {
    const int ka = a_k0 + k, kb = b_k0 + k;
    const uint64_t ad = tc::smem_desc_sw128(a0 + (uint32_t)(ka >> 5) * (uint32_t)a_R * 128u + (uint32_t)(ka & 31) * 4u,
                                            16, 1024);
    const uint64_t bd = tc::smem_desc_sw128(b0 + (uint32_t)(kb >> 5) * (uint32_t)b_R * 128u + (uint32_t)(kb & 31) * 4u,
                                            16, 1024);
    mma_tf32(tmem_d, ad, bd, id, (accumulate || k > 0) ? 1u : 0u);
  }
}
// Same K range for both operands.
KIMI_D void mma_rows128(uint32_t tmem_d, const float* a, int a_R, const float* b, int b_R, int b_row0, int n, int k0,
                        int kn, bool accumulate) {
  mma_rows128_ab(tmem_d, a, a_R, k0, b, b_R, b_row0, k0, n, kn, accumulate);
}

// Row `lane` of the accumulator (this warp's TMEM sub-partition) at columns [col, col + 32).
KIMI_D void tmem_row32(uint32_t tmem_base, int warp, int col, float* v) {
  tc::tmem_ld_32x32b_x32(tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)col, v);
}

// Row `lane` of the accumulator at columns [col, col + 16).
KIMI_D void tmem_row16(uint32_t tmem_base, int warp, int col, float* v) {
  tc::tmem_ld_32x32b_x16(tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)col, v);
}

KIMI_D void bar_sync(int id, int threads) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory"); }

// Publish thread-written operand tiles to the tensor core and order earlier TMEM reads
// before the MMA that will overwrite them; all threads of the block call it.
KIMI_D void operands_ready() {
  tc::fence_proxy_async();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
}

// Wait for the MMAs committed to `bar` (phase bit flips per use); bounded.
KIMI_D bool mma_done(uint64_t* bar, uint32_t& phase, int* status, int code) {
  const bool ok = tc::mbar_wait_local(bar, phase, status, code);
  phase ^= 1u;
  tc::tc_fence_after();
  return ok;
}

}  // namespace tcs
}  // namespace kimi
