// Host interface of the tcgen05 GEMM (gemm_tc.cu).
//   C = A * B^T with bf16 operands and fp32 accumulation.
//   A storage: K-major [a_rows = M_total, a_cols = K] or MN-major [a_rows = K_total, a_cols = M] (a_ld elems).
//   B storage: K-major [b_groups, b_rows = N, b_cols = K] or MN-major [b_groups, b_rows = K, b_cols = N]
//              (row stride b_ld elems, group stride b_gstride elems).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace kimi {

struct TcGemmArgs {
  int mode = 0;  // 0 dense, 1 grouped over M rows, 2 grouped over K rows
  int bn = 128;  // 128 or 256 output columns per tile (SiTU always uses 256 = 128 gate + 128 up)
  bool a_mn = false, b_mn = false;
  const void* a = nullptr;
  int64_t a_rows = 0, a_cols = 0, a_ld = 0;
  const void* b = nullptr;
  const void* b2 = nullptr;  // SiTU "up" weights, or the second half of a concatenated K
  int64_t b_groups = 1, b_rows = 0, b_cols = 0, b_ld = 0, b_gstride = 0;
  int b2_k_split = 0;
  int M = 0, N = 0, K = 0, G = 1;
  const int* offsets = nullptr;  // device [G+1]
  int uniform_rows = 0;          // mode 1: every segment has this many rows (offsets[g] = g * rows)
  int epi = 0;                   // 0 store, 1 SiTU, 2 weighted scatter-add (fp32), 3 fp32 add into out
  void* out = nullptr;
  bool out_fp32 = false;
  int64_t ldc = 0;
  void* out_g = nullptr;
  void* out_u = nullptr;
  float bg = 4.f, bu = 25.f;
  const int* row_token = nullptr;
  const float* row_weight = nullptr;
  // epi 2 only: row_token = rank * agg_tokens + token adds into agg_peer[rank] (row stride ldc)
  uint64_t agg_peer[8] = {};
  int agg_tokens = 0;
  // all-gather fused into A (dense, K-major A): `a` is this rank's [M, K] gather buffer (rows
  // [ag_rank * ag_rows, ...) hold its own shard), ag_peer[r] rank r's buffer; M = ag_world * ag_rows;
  // ag_flags: local [M / 128] block flags; ag_epoch: device call counter
  uint64_t ag_peer[8] = {};
  int ag_world = 0, ag_rows = 0, ag_rank = 0;
  uint32_t* ag_flags = nullptr;
  const uint32_t* ag_epoch = nullptr;
  // Dense mode only: split the K range into `ksplit` slices (epi 3 adds them into `out`); an fp32
  // bias [N] or a bf16 residual [M, ldr] added in the store epilogue; CTA pairs (cta_group::2,
  // 256-row tiles): 1 on, 0 off, -1 whenever M > 128.
  int ksplit = 1;
  const float* bias = nullptr;
  const void* resid = nullptr;
  int64_t ldr = 0;
  int pair = -1;
  int debug = 0;  // bit 0: skip the store epilogue's global writes; bit 1: role wait counters into dbg
  // Fused projection groups (dense mode): kind 1 splits the output's columns over seg_ptr (bf16
  // [M, width] row-major outputs), kind 2 takes A's K range from K-major segments [M, width], kind 3
  // takes A's rows from MN-major segments [K, width].  seg_width[s] > 0, seg_ld[s] in elements.
  int seg_kind = 0, nseg = 0;
  void* seg_ptr[8] = {};
  int64_t seg_width[8] = {}, seg_ld[8] = {};
  unsigned long long* dbg = nullptr;
  int* status = nullptr;     // null: the device's default status word (tc_gemm_status)
  uint32_t spin_limit = 0;   // polls per pipeline wait before giving up; 0 = the built-in limit
  int num_sms = 0;
  // Comm modes (dense, bf16 output, A K-major, N % 8 == 0): `out` / `ldc` must be this rank's
  // symmetric partial buffer [M, N] (ldc == N); the summed result goes to comm_out.
  int comm_mode = 0;  // 0 off, 1 all-reduce, 2 reduce-scatter
  int comm_rank = 0, comm_world = 1, comm_rows_per_rank = 0;
  uint64_t part_peer[8] = {};
  uint64_t part_mc = 0;
  uint64_t flags_peer[8] = {};
  int tiles_cap = 0;
  void* comm_out = nullptr;
  int64_t comm_ldo = 0;
  int64_t timeout_ns = 10000000000LL;
};

// Output tiles of a dense launch (for sizing the comm flag region).
inline int tc_gemm_tiles(int M, int N, int bn) { return ((M + 127) / 128) * ((N + bn - 1) / bn); }

cudaError_t tc_gemm(const TcGemmArgs& args, cudaStream_t stream);

// Read (and with clear, reset) the current device's default GEMM status word: 0 = every wait of
// every launch that used it completed; otherwise the code of the first wait that gave up.
// Synchronous (a device-to-host copy); -1 if the copy failed.
int tc_gemm_status(bool clear);
// Device address of the current device's default status word (for stream-ordered reads).
int* tc_gemm_default_status();

}  // namespace kimi
