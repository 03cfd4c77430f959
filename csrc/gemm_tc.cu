// Persistent warp-specialised tcgen05 GEMM for sm_100a:  C = A * B^T  (bf16 in, fp32 accumulate).
//
//   warp 0      TMA producer: A and B tiles (128B-swizzled) into a STAGES-deep smem ring
//   warp 1      MMA issuer: tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM accumulators;
//               allocates / frees TMEM
//   warps 2..9  epilogue: tcgen05.ld of the finished accumulator (one row per thread; warps 2..5 and
//               6..9 take the two column halves of the tile) and a fused store, overlapping the
//               MMAs of the next tile (double-buffered TMEM)
//
// Modes:  0 dense;  1 grouped over M (row segments of A, one B matrix per segment: MoE experts);
//         2 grouped over K (reduction over row segments, one C matrix per segment: expert weight
//           gradients).  Segment offsets are device arrays (multiples of 128 rows in mode 1 and of
//           64 rows in mode 2), so the launch shape never depends on the routing.
// Operands may be K-major or MN-major (``a_mn`` / ``b_mn``), which covers the forward and both
// backward products without transposed copies.
// Epilogues:  0 store (bf16 or fp32), 1 SiTU-GLU of a (gate | up) tile pair (stores h, gate, up),
//             2 weighted scatter-add into fp32 rows (row_token[r] < 0 skips the row).
// Comm modes (dense mode, bf16 output): the epilogue stores each tile's partial product into a
// symmetric buffer shared with the other ranks of a tensor-parallel group and signals the tile's
// owner; four extra "comm" warps reduce the tiles this rank owns across all ranks while the
// MMAs of later tiles proceed:  all-reduce (every rank ends with the sum, copied out of the
// buffer tile by tile) or reduce-scatter (the owner of a row block writes the sum into its own
// output).  The reduction reads the ranks' partials with one NVLink-multicast multimem.ld_reduce
// per 16 bytes and writes the sum back with multimem.st (NVLS), or with peer loads and stores
// when the group has no multicast object.  Flags are counting semaphores in the same buffer, so
// consecutive calls (and CUDA-graph replays) need no host-side epoch.  Every wait on a peer is
// bounded by a time limit and reports through the status word.
// TMA loads never use cluster multicast; every mbarrier wait is bounded (status word).
#include <cuda.h>
#include <cstdio>
#include <cstdlib>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "device_info.h"
#include "tc_common.cuh"
#include "tc_gemm.h"

namespace kimi {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;

constexpr int kMaxRanks = 8;
constexpr int kMaxSegs = 8;

struct CommParams {
  int mode;                     // 0 off, 1 all-reduce, 2 reduce-scatter
  int rank, world;
  int rows_per_rank;            // reduce-scatter: output rows owned by each rank
  uint64_t part_peer[kMaxRanks];   // partial buffer [M, N] bf16 on every rank (this rank's included)
  uint64_t part_mc;             // multicast address of the partial buffer (0: peer loads / stores)
  uint64_t flags_peer[kMaxRanks];  // flag words on every rank: ready[tiles] then done[tiles]
  int tiles_cap;                // flag capacity (tiles)
  void* out;                    // all-reduce: [M, N] result; reduce-scatter: [rows_per_rank, N]
  int64_t ldo;
  int64_t timeout_ns;
};

struct DevParams {
  CUtensorMap map_a;
  CUtensorMap map_b;
  CUtensorMap map_b2;
  CUtensorMap map_c;  // the output [M, N] (bf16: 32 x 32 boxes; fp32: 16 x 32), 64-byte swizzle
  // Segmented operands of fused projection groups (several weights sharing one input):
  //   kind 1: the output's columns [start[s], start[s+1]) go to seg_map[s] (forward, N = sum of widths)
  //   kind 2: A's K range [start[s], start[s+1]) comes from seg_map[s] (input gradient dX = sum_s dY_s W_s)
  //   kind 3: A's rows [start[s], start[s+1]) come from seg_map[s], A MN-major (weight gradients dY_s^T X)
  // Boundaries are multiples of 32 (kind 1) or 64 (kinds 2, 3) except the last.
  CUtensorMap seg_map[kMaxSegs];
  int nseg, seg_kind;
  int seg_start[kMaxSegs + 1];
  int tma_store;      // epi 0 stores through shared memory + TMA (see the epilogue)
  // All-gather fused into the A operand (dense mode, A K-major, comm warps): every rank holds an
  // [M, K] gather buffer (symmetric) whose rows [r * ag_rows, (r + 1) * ag_rows) rank r fills with its
  // shard.  The comm warps copy each remote 128-row block from its owner's buffer into this rank's
  // buffer (each byte crosses NVLink once) and release a per-block flag; tiles of local rows run
  // first, and the producer waits for a remote block's flag before its first TMA load of it.
  int ag_world, ag_rows, ag_rank;
  const uint8_t* ag_peer[8];
  uint8_t* ag_local;
  uint32_t* ag_flags;        // local, one per 128-row block, monotonic (value = call number + 1)
  const uint32_t* ag_epoch;  // call number, advanced by the host wrapper after each call
  int64_t ag_ld;             // row stride of the gather buffers in bytes
  int mode, M, N, K, G;
  const int* offsets;
  int uniform_rows;  // mode 1 with equal segments: tile -> segment by division, no offset scan
  int b2_k_split;  // k-blocks at k >= split read map_b2 at (k - split); 0 = off
  int situ;        // B tile = [gate 128 rows | up 128 rows] from map_b / map_b2
  int epi;
  void* out;
  int out_fp32;
  int64_t ldc;
  void* out_g;
  void* out_u;
  float bg, bu;
  const int* row_token;
  const float* row_weight;
  // Remote combine (epi 2): row_token = rank * agg_tokens + token selects rank's aggregate
  // agg_peer[rank] (a peer's memory over NVLink); agg_tokens == 0 keeps the local `out`.
  float* agg_peer[8];
  int agg_tokens;
  int* status;
  uint32_t spin_limit;  // polls per pipeline wait before it gives up (tests shorten it)
  int ksplit;           // dense mode: the K range is split into this many slices (epi 3 adds them up)
  int debug;            // bit 0: skip the epilogue's global stores; bit 1: role wait counters (experiments)
  unsigned long long* dbg;  // bit 1: [0] MMA waits on full, [1] MMA waits on tempty, [2] producer waits on
                            // empty, [3] epilogue waits on tfull, [4] MMA loop, [5] epilogue loop (cycles)
  const float* bias;    // epi 0: fp32 [N] added to every row (or null)
  const __nv_bfloat16* resid;  // epi 0, bf16 output: [M, ldr] added to the result (or null)
  int64_t ldr;
  CommParams cm;
};

struct TileInfo {
  int g;        // group
  int m0;       // A row coordinate (mode 0/1) or C row (mode 2)
  int n0;       // C column
  int k0;       // first reduction coordinate
  int num_kb;   // k blocks
  int c_row0;   // output row base (modes 0/1: m0; mode 2: m within group)
};

template <int BNT>
__device__ __forceinline__ int tiles_n_of(const DevParams& p) {
  return (p.N + BNT - 1) / BNT;
}

// Work units of a launch.  BMT is the output rows of a tile: 128 for one CTA, 256 for a CTA pair.
template <int BNT, int BMT = BM>
__device__ int total_tiles(const DevParams& p) {
  const int tn = tiles_n_of<BNT>(p);
  if (p.mode == 0) return ((p.M + BMT - 1) / BMT) * tn * p.ksplit;
  if (p.mode == 1) {
    if (p.uniform_rows > 0) return p.G * (p.uniform_rows / BM) * tn;
    int t = 0;
    for (int g = 0; g < p.G; ++g) t += ((p.offsets[g + 1] - p.offsets[g]) / BM) * tn;
    return t;
  }
  return p.G * ((p.M + BM - 1) / BM) * tn;
}

template <int BNT, int BMT = BM>
__device__ TileInfo tile_info(const DevParams& p, int tile) {
  const int tn = tiles_n_of<BNT>(p);
  TileInfo ti;
  if (p.mode == 0) {
    const int tm = (p.M + BMT - 1) / BMT;
    ti.g = 0;
    const int total_kb = (p.K + BK - 1) / BK;
    int split = 0, kb_per = total_kb;
    if (p.ksplit > 1) {  // slices of the K range: every output tile of slice 0, then slice 1, ...
      split = tile / (tm * tn);
      tile -= split * tm * tn;
      kb_per = (total_kb + p.ksplit - 1) / p.ksplit;
    }
    if (p.ag_world > 0) {  // this rank's row blocks first (every column tile), then the remote ones
      const int bpr = p.ag_rows / BM, first = p.ag_rank * bpr, local = bpr * tn;
      if (tile < local) {
        ti.m0 = (first + tile % bpr) * BM;
        ti.n0 = (tile / bpr) * BNT;
      } else {
        const int t2 = tile - local, rem = tm - bpr;
        ti.m0 = ((first + bpr + t2 % rem) % tm) * BM;
        ti.n0 = (t2 / rem) * BNT;
      }
    } else {
      ti.m0 = (tile % tm) * BMT;
      ti.n0 = (tile / tm) * BNT;
    }
    ti.k0 = split * kb_per * BK;
    const int left = total_kb - split * kb_per;
    ti.num_kb = left < kb_per ? (left > 0 ? left : 0) : kb_per;
    ti.c_row0 = ti.m0;
    return ti;
  }
  if (p.mode == 1 && p.uniform_rows > 0) {
    const int tm = p.uniform_rows / BM, per = tm * tn;
    const int g = tile / per, local = tile - g * per;
    ti.g = g;
    ti.m0 = g * p.uniform_rows + (local % tm) * BM;
    ti.n0 = (local / tm) * BNT;
    ti.k0 = 0;
    ti.num_kb = (p.K + BK - 1) / BK;
    ti.c_row0 = ti.m0;
    return ti;
  }
  if (p.mode == 1) {
    int g = 0, base = 0;
    for (; g < p.G; ++g) {
      const int tg = ((p.offsets[g + 1] - p.offsets[g]) / BM) * tn;
      if (tile < base + tg) break;
      base += tg;
    }
    const int local = tile - base;
    const int tm = (p.offsets[g + 1] - p.offsets[g]) / BM;
    ti.g = g;
    ti.m0 = p.offsets[g] + (local % tm) * BM;
    ti.n0 = (local / tm) * BNT;
    ti.k0 = 0;
    ti.num_kb = (p.K + BK - 1) / BK;
    ti.c_row0 = ti.m0;
    return ti;
  }
  const int tm = (p.M + BM - 1) / BM;
  const int per = tm * tn;
  ti.g = tile / per;
  const int local = tile % per;
  ti.m0 = (local % tm) * BM;
  ti.n0 = (local / tm) * BNT;
  ti.k0 = p.offsets[ti.g];
  ti.num_kb = (p.offsets[ti.g + 1] - p.offsets[ti.g]) / BK;
  ti.c_row0 = ti.m0;
  return ti;
}

// ---------------------------------------------------------------- cross-rank helpers (comm modes)
constexpr int kCommTimeout = 5;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ uint4 ld_sys16(const void* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_sys16(void* p, uint4 v) {
  asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
// Sum of the eight bf16 values at `addr` over every rank of the multicast group (fp32 accumulation).
__device__ __forceinline__ uint4 mc_ld_reduce_bf16x8(uint64_t addr) {
  uint4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void mc_st16(uint64_t addr, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
// Bounded wait for *flag >= target; on timeout (or an error already raised) returns false.
__device__ bool wait_geq(const uint32_t* flag, uint32_t target, int64_t timeout_ns, int* status) {
  const uint64_t t0 = global_ns();
  while (ld_acquire_sys(flag) < target) {
    if (*reinterpret_cast<volatile int*>(status) != 0) return false;
    if ((int64_t)(global_ns() - t0) > timeout_ns) {
      atomicCAS(status, 0, kCommTimeout);
      return false;
    }
    __nanosleep(100);
  }
  return true;
}
__device__ __forceinline__ void comm_bar() { asm volatile("bar.sync 2, 128;" ::: "memory"); }
// Named-barrier OR vote over `threads` threads: true when any of them passes pred = true.
__device__ __forceinline__ bool bar_red_or(int id, int threads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(threads)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ void add_bf16x8(float* acc, uint4 v) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = __bfloat1622float2(h[j]);
    acc[2 * j] += f.x;
    acc[2 * j + 1] += f.y;
  }
}
__device__ __forceinline__ uint4 pack_bf16x8(const float* acc) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
  return v;
}

// Rank that reduces a tile: spread over CTAs and over a CTA's successive tiles (all-reduce), or
// the rank owning the tile's rows (reduce-scatter).
__device__ __forceinline__ int tile_owner(const CommParams& c, int tile, int m0) {
  if (c.mode == 2) return m0 / c.rows_per_rank;
  return (int)((tile % gridDim.x + tile / gridDim.x) % c.world);
}

// SiTU-GLU in the GEMM epilogue, with the hardware approximations of tanh and 2^x (MUFU; relative
// error near 2^-11, below the bf16 rounding of the stored result).  The epilogue evaluates this
// once per output element and is otherwise the bottleneck of the short-K expert GEMM; the
// backward recomputes the derivative from the stored bf16 gate / up values.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float sigmoid_approx(float x) {
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-1.4426950408889634f * x));  // e^{-x} = 2^{-x log2 e}
  return __frcp_rn(1.f + e);
}
__device__ __forceinline__ float situ_fwd(float g, float u, float bg, float bu, float ibg, float ibu) {
  return bg * tanh_approx(g * ibg) * sigmoid_approx(g) * bu * tanh_approx(u * ibu);
}

template <int BN>
__device__ void comm_loop(const DevParams& p, int total);
__device__ void ag_copy_loop(const DevParams& p);

// Output staging of the TMA-store epilogue: 8 warps x 2 buffers x (32 rows x 64 bytes).
constexpr int kStagingBytes = 8 * 2 * 2048;

// Shared-memory ring depth: about 192 KB of stages whatever the tile shape.
template <int BN, bool PAIR>
constexpr int ring_stages() {
  return (192 * 1024) / (BM * BK * 2 + (PAIR ? BN / 2 : BN) * BK * 2);
}

// Segment holding coordinate `c` (the last one for coordinates past the end: its map reads zeros there).
__device__ __forceinline__ int seg_of(const DevParams& p, int c) {
  int s = 0;
  while (s + 1 < p.nseg && c >= p.seg_start[s + 1]) ++s;
  return s;
}

// debug bit 2: launch timeline (globaltimer ns) into dbg[8..15]: [8] earliest CTA start (min),
// [9] latest CTA start, [10] latest end of set-up, [11] latest first stage seen by an MMA issuer,
// [12] latest MMA loop end, [13] latest epilogue end, [14] latest CTA exit
__device__ __forceinline__ void dbg_stamp(const DevParams& p, int slot, bool as_min) {
  if (!(p.debug & 4)) return;
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  if (as_min)
    atomicMin(p.dbg + slot, (unsigned long long)t);
  else
    atomicMax(p.dbg + slot, (unsigned long long)t);
}

template <int BN, bool A_MN, bool B_MN, int CM, bool PAIR>
__global__ void __launch_bounds__(CM ? 448 : 320, 1) gemm_tc_kernel(const __grid_constant__ DevParams p) {
  // PAIR: two CTAs of a cluster compute one 256 x BN tile with tcgen05.mma.cta_group::2, issued by
  // the even CTA.  Each CTA's shared memory holds its 128 rows of A and its BN / 2 rows of B; the even
  // CTA's producer issues all four copies of a stage (the odd CTA's through shared::cluster
  // addresses) against its own `full` barrier, so one commit per K block frees the stage.  Each CTA
  // owns 128 rows of the accumulator in its own TMEM and stores them.  Halving each SM's share of B halves the B traffic per MMA, which keeps
  // the tensor pipe fed at N = 128 and takes a quarter off the L2 -> SMEM bytes at N = 256.
  constexpr int CTAS = PAIR ? 2 : 1;
  constexpr int BMT = BM * CTAS;           // output rows of a tile
  constexpr int BNL = BN / CTAS;           // rows of the B tile held by this CTA
  constexpr int A_BYTES = BM * BK * 2;
  constexpr int B_BYTES = BNL * BK * 2;
  constexpr int STAGE = A_BYTES + B_BYTES;
  constexpr int STAGES = ring_stages<BN, PAIR>();
  constexpr int TMEM_COLS = 2 * BN;
  static_assert(!PAIR || CM == 0, "CTA pairs run the plain (non-comm) kernel");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // TMA-store staging: two 2 KB buffers per epilogue warp after the ring
  uint8_t* staging = smem + STAGES * STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + kStagingBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;  // MMA warp's exit barrier: every issued MMA has completed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(drain + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bnt = p.situ ? BN / 2 : BN;  // output columns per tile
  const uint32_t rank = PAIR ? tc::cluster_ctarank() : 0u;
  if (threadIdx.x == 0) {
    dbg_stamp(p, 8, true);
    dbg_stamp(p, 9, false);
  }
  const int first_unit = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int unit_stride = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 8 * CTAS);  // one arrival per epilogue warp of every CTA
    }
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
    tc::fence_proxy_async();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tc::tmem_alloc_pair(tslot, TMEM_COLS);
      tc::tmem_relinquish_pair();
    } else {
      tc::tmem_alloc(tslot, TMEM_COLS);
      tc::tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    tc::tma_prefetch(&p.map_a);
    tc::tma_prefetch(&p.map_b);
    if (p.situ || p.b2_k_split) tc::tma_prefetch(&p.map_b2);
    if (p.tma_store) tc::tma_prefetch(&p.map_c);
  }
  tc::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) tc::cluster_sync();  // both CTAs' barriers are initialised before any remote use
  tc::tc_fence_after();
  const uint32_t tmem_base = *tslot;
  if (threadIdx.x == 0) dbg_stamp(p, 10, false);
  const int total = p.situ ? total_tiles<BN / 2, BMT>(p) : total_tiles<BN, BMT>(p);

  if (warp == 0) {
    if (lane == 0 && (!PAIR || rank == 0)) {
      // Roles leave their loops at the first failed wait (their own timeout, or another role's
      // or CTA's recorded in the status word).  On the way out the producer waits for the TMA
      // copies it has in flight, so no copy lands in shared memory after the CTA has exited.
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      uint32_t inflight = 0, inflight_ph = 0;  // stages filled since their last consumption, and their phase
      uint32_t ag_target = 0u;
      if constexpr (CM == 3) ag_target = *p.ag_epoch + 1u;
      for (int tile = first_unit; ok && tile < total; tile += unit_stride) {
        const TileInfo ti = p.situ ? tile_info<BN / 2, BMT>(p, tile) : tile_info<BN, BMT>(p, tile);
        for (int kb = 0; kb < ti.num_kb; ++kb) {
          const long long w0 = (p.debug & 2) ? clock64() : 0;
          if (!tc::mbar_wait(&empty[s], ph ^ 1, p.status, tc::kTimeoutEmpty, p.spin_limit)) {
            ok = false;
            break;
          }
          if (p.debug & 2) atomicAdd(p.dbg + 2, (unsigned long long)(clock64() - w0));
          inflight &= ~(1u << s);
          uint8_t* sa = smem + s * STAGE;
          uint8_t* sb = sa + A_BYTES;
          const int k = ti.k0 + kb * BK;
          if constexpr (CM == 3 && !A_MN) {
            if (kb == 0 && ti.m0 / p.ag_rows != p.ag_rank) {
              // remote rows: wait until a comm warp has copied this block into the local buffer
              const uint32_t* f = p.ag_flags + ti.m0 / BM;
              const uint64_t t0 = global_ns();
              uint32_t v;
              while (true) {
                asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
                if (v >= ag_target) break;
                if (tc::status_peek(p.status) != 0) {
                  ok = false;
                  break;
                }
                if ((int64_t)(global_ns() - t0) > (int64_t)10000000000LL) {
                  atomicCAS(p.status, 0, kCommTimeout);
                  ok = false;
                  break;
                }
                __nanosleep(64);
              }
              if (!ok) break;
              asm volatile("fence.proxy.async.global;" ::: "memory");
            }
          }
          const CUtensorMap* mb = &p.map_b;
          int kb_coord = k;
          if (p.b2_k_split && k >= p.b2_k_split) {
            mb = &p.map_b2;
            kb_coord = k - p.b2_k_split;
          }
          if constexpr (PAIR) {
            // the leader fills the stage in both CTAs (its own rows, then the peer's through its
            // shared::cluster address); every copy is counted on the leader's barrier
            const uint32_t fb = tc::smem_u32(&full[s]);
            tc::mbar_arrive_expect_tx(&full[s], 2 * STAGE);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              const uint32_t da = r == 0 ? tc::smem_u32(sa) : tc::mapa_shared(sa, 1);
              const uint32_t db = da + A_BYTES;
              const int arow = ti.m0 + r * BM;
              if (!A_MN) {
                if (p.seg_kind == 2) {
                  const int sg = seg_of(p, k);
                  tc::tma_load_2d_pair_to(da, &p.seg_map[sg], fb, k - p.seg_start[sg], arow);
                } else {
                  tc::tma_load_2d_pair_to(da, &p.map_a, fb, k, arow);
                }
              } else if (p.seg_kind == 3) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int mm = arow + 64 * h, sg = seg_of(p, mm);
                  tc::tma_load_2d_pair_to(da + h * (A_BYTES / 2), &p.seg_map[sg], fb, mm - p.seg_start[sg], k);
                }
              } else {
                tc::tma_load_2d_pair_to(da, &p.map_a, fb, arow, k);
                tc::tma_load_2d_pair_to(da + A_BYTES / 2, &p.map_a, fb, arow + 64, k);
              }
              if (p.situ) {  // the even CTA holds the gate rows of the tile, the odd one the up rows
                tc::tma_load_3d_pair_to(db, r == 0 ? &p.map_b : &p.map_b2, fb, kb_coord, ti.n0, ti.g);
              } else if (!B_MN) {
                tc::tma_load_3d_pair_to(db, mb, fb, kb_coord, ti.n0 + r * BNL, 0);
              } else {
#pragma unroll
                for (int q = 0; q < BNL / 64; ++q)
                  tc::tma_load_3d_pair_to(db + q * (BK * 64 * 2), mb, fb, ti.n0 + r * BNL + q * 64, kb_coord, 0);
              }
            }
          } else {
            tc::mbar_arrive_expect_tx(&full[s], STAGE);
            if (!A_MN) {
              if (p.seg_kind == 2) {
                const int sg = seg_of(p, k);
                tc::tma_load_2d(sa, &p.seg_map[sg], &full[s], k - p.seg_start[sg], ti.m0);
              } else {
                tc::tma_load_2d(sa, &p.map_a, &full[s], k, ti.m0);
              }
            } else if (p.seg_kind == 3) {
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const int mm = ti.m0 + 64 * h, sg = seg_of(p, mm);
                tc::tma_load_2d(sa + h * (A_BYTES / 2), &p.seg_map[sg], &full[s], mm - p.seg_start[sg], k);
              }
            } else {
              tc::tma_load_2d(sa, &p.map_a, &full[s], ti.m0, k);
              tc::tma_load_2d(sa + A_BYTES / 2, &p.map_a, &full[s], ti.m0 + 64, k);
            }
            if (p.situ) {
              tc::tma_load_3d(sb, &p.map_b, &full[s], kb_coord, ti.n0, ti.g);
              tc::tma_load_3d(sb + B_BYTES / 2, &p.map_b2, &full[s], kb_coord, ti.n0, ti.g);
            } else if (!B_MN) {
              tc::tma_load_3d(sb, mb, &full[s], kb_coord, ti.n0, p.mode == 2 ? 0 : ti.g);
            } else {
#pragma unroll
              for (int q = 0; q < BN / 64; ++q)
                tc::tma_load_3d(sb + q * (BK * 64 * 2), mb, &full[s], ti.n0 + q * 64, kb_coord,
                                p.mode == 2 ? 0 : ti.g);
            }
          }
          inflight |= 1u << s;
          inflight_ph = (inflight_ph & ~(1u << s)) | (ph << s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok)
        for (int q = 0; q < STAGES; ++q)
          if (inflight & (1u << q))
            tc::mbar_wait_local(&full[q], (inflight_ph >> q) & 1u, p.status, tc::kTimeoutDrain, tc::kDrainNs);
    }
  } else if (warp == 1) {
    if (lane == 0 && (!PAIR || rank == 0)) {
      const uint32_t idesc = tc::instr_desc_f16(BMT, BN, true, A_MN, B_MN);
      // Descriptors of stage 0 at K offset 0; a stage / K step only moves the 14-bit start-address
      // field (16-byte units), so the loop adds small constants to precomputed 64-bit values.
      const uint32_t ring0 = tc::smem_u32(smem);
      const uint64_t adesc0 = A_MN ? tc::smem_desc_sw128(ring0, 8192, 1024) : tc::smem_desc_sw128(ring0, 16, 1024);
      const uint64_t bdesc0 = B_MN ? tc::smem_desc_sw128(ring0 + A_BYTES, 8192, 1024)
                                   : tc::smem_desc_sw128(ring0 + A_BYTES, 16, 1024);
      constexpr uint64_t A_KSTEP = (A_MN ? 2048 : 32) >> 4, B_KSTEP = (B_MN ? 2048 : 32) >> 4;
      constexpr uint64_t STAGE16 = STAGE >> 4;
      // commit target: the stage's `empty` barrier of the producer that refills it
      const uint32_t empty_c0 = PAIR ? tc::mapa_shared(&empty[0], 0) : tc::smem_u32(&empty[0]);
      int s = 0, it = 0;
      uint32_t ph = 0;
      bool ok = true, issued = false;
      const long long t_mma = (p.debug & 2) ? clock64() : 0;
      for (int tile = first_unit; ok && tile < total; tile += unit_stride, ++it) {
        const int num_kb = p.situ ? tile_info<BN / 2, BMT>(p, tile).num_kb : tile_info<BN, BMT>(p, tile).num_kb;
        const int buf = it & 1;
        const uint32_t tph = (it >> 1) & 1;
        const long long w1 = (p.debug & 2) ? clock64() : 0;
        if (!tc::mbar_wait(&tempty[buf], tph ^ 1, p.status, tc::kTimeoutTmemEmpty, p.spin_limit)) {
          ok = false;
          break;
        }
        if (p.debug & 2) atomicAdd(p.dbg + 1, (unsigned long long)(clock64() - w1));
        tc::tc_fence_after();
        const uint32_t d = tmem_base + buf * BN;
        uint32_t acc = 0;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (p.debug & 2) {
            const long long w2 = clock64();
            while (!tc::mbar_try_wait(&full[s], ph)) {}
            atomicAdd(p.dbg + 0, (unsigned long long)(clock64() - w2));
          }
          if (!tc::mbar_wait(&full[s], ph, p.status, tc::kTimeoutFull, p.spin_limit)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          if (!issued) dbg_stamp(p, 11, false);
          const uint64_t soff = (uint64_t)s * STAGE16;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = adesc0 + soff + kk * A_KSTEP, bd = bdesc0 + soff + kk * B_KSTEP;
            if constexpr (PAIR)
              tc::mma_f16_pair(d, ad, bd, idesc, acc);
            else
              tc::mma_f16(d, ad, bd, idesc, acc);
            acc = 1u;
          }
          issued = true;
          if constexpr (PAIR) {  // the leader's producer refills both CTAs' halves of the stage
            tc::mma_commit_pair(empty_c0 + 8u * s);
          } else {
            tc::mma_commit_addr(empty_c0 + 8u * s);
          }
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          tc::mma_commit_pair(tc::mapa_shared(&tfull[buf], 0));
          tc::mma_commit_pair(tc::mapa_shared(&tfull[buf], 1));
        } else {
          tc::mma_commit(&tfull[buf]);
        }
      }
      if (p.debug & 2) atomicAdd(p.dbg + 4, (unsigned long long)(clock64() - t_mma));
      dbg_stamp(p, 12, false);
      if (!ok && issued) {
        // let every issued MMA finish before the CTA frees its TMEM and shared memory
        if constexpr (PAIR)
          tc::mma_commit_pair(tc::mapa_shared(drain, 0));
        else
          tc::mma_commit(drain);
        tc::mbar_wait_local(drain, 0, p.status, tc::kTimeoutDrain, tc::kDrainNs);
      }
    }
  } else if (warp < 10) {
    const int sub = warp & 3;
    const int r_local = sub * 32 + lane;
    const int chalf = (warp - 2) >> 2;  // column half of the tile handled by this warpgroup
    const float ibg = 1.f / p.bg, ibu = 1.f / p.bu;
    const uint32_t tempty_c0_0 = PAIR ? tc::mapa_shared(&tempty[0], 0) : 0u;
    const uint32_t tempty_c0_1 = PAIR ? tc::mapa_shared(&tempty[1], 0) : 0u;
    // TMA-store epilogue: this warp's two staging buffers (32 rows x 64 bytes each, 64-byte swizzle)
    // alternate between chunks; a buffer is rewritten only after the store issued from it two
    // chunks earlier has finished reading it.
    uint8_t* my_stage = staging + (warp - 2) * 2 * 2048;
    uint32_t stores = 0;
    // one 32-row x 64-byte chunk: row `lane` writes its 16-byte pieces at their swizzled slots
    auto stage_and_store = [&](const uint4* pieces, int x, int y, bool reduce_add) {
      uint8_t* b = my_stage + (stores & 1) * 2048;
      if (lane == 0) tc::bulk_wait_read<1>();
      __syncwarp();
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(b + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) = pieces[c];
      tc::fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        const CUtensorMap* map = &p.map_c;
        if (p.seg_kind == 1) {  // a fused projection group: this chunk's columns belong to one output
          const int sg = seg_of(p, x);
          map = &p.seg_map[sg];
          x -= p.seg_start[sg];
        }
        if (reduce_add)
          tc::tma_reduce_add_2d(map, b, x, y);
        else
          tc::tma_store_2d(map, b, x, y);
        tc::bulk_commit();
      }
      ++stores;
    };
    int it = 0;
    const long long t_epi = (p.debug & 2) ? clock64() : 0;
    for (int tile = first_unit; tile < total; tile += unit_stride, ++it) {
      const TileInfo ti = p.situ ? tile_info<BN / 2, BMT>(p, tile) : tile_info<BN, BMT>(p, tile);
      const int buf = it & 1;
      const uint32_t tph = (it >> 1) & 1;
      const long long w3 = (p.debug & 2) ? clock64() : 0;
      bool ok = tc::mbar_wait(&tfull[buf], tph, p.status, tc::kTimeoutTmemFull, p.spin_limit, 128);
      if ((p.debug & 2) && lane == 0 && warp == 2) atomicAdd(p.dbg + 3, (unsigned long long)(clock64() - w3));
      if constexpr (CM == 1 || CM == 2) {
        // the comm epilogue meets at a named barrier per tile: leave together or not at all
        ok = !bar_red_or(1, 256, !ok);
      }
      if (!ok) break;
      tc::tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + buf * BN;
      const int row = ti.c_row0 + (int)rank * BM + r_local;
      const bool row_ok = (p.mode == 1) ? true : row < p.M;
      for (int c0 = chalf * (bnt / 2); c0 < (chalf + 1) * (bnt / 2); c0 += 32) {
        float v[32];
        if (ti.num_kb > 0) {
          tc::tmem_ld_32x32b_x32(taddr + c0, v);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = 0.f;
        }
        const int col0 = ti.n0 + c0;
        if (p.situ) {
          float u[32];
          if (ti.num_kb > 0) {
            tc::tmem_ld_32x32b_x32(taddr + bnt + c0, u);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = 0.f;
          }
          if (row_ok) {
            __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)row * p.ldc;
            __nv_bfloat16* og = reinterpret_cast<__nv_bfloat16*>(p.out_g) + (int64_t)row * p.ldc;
            __nv_bfloat16* ou = reinterpret_cast<__nv_bfloat16*>(p.out_u) + (int64_t)row * p.ldc;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              if (col0 + i + 8 <= p.N) {
                Vec<__nv_bfloat16> vh, vg, vu;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const float gq = to_f<__nv_bfloat16>(from_f<__nv_bfloat16>(v[i + j]));
                  const float uq = to_f<__nv_bfloat16>(from_f<__nv_bfloat16>(u[i + j]));
                  vg.v[j] = from_f<__nv_bfloat16>(gq);
                  vu.v[j] = from_f<__nv_bfloat16>(uq);
                  vh.v[j] = from_f<__nv_bfloat16>(situ_fwd(gq, uq, p.bg, p.bu, ibg, ibu));
                }
                vh.store(h + col0 + i);
                vg.store(og + col0 + i);
                vu.store(ou + col0 + i);
              }
            }
          }
        } else if (p.epi == 2) {
          if (row_ok) {
            const int tok = p.row_token[row];
            if (tok >= 0) {
              const float w = p.row_weight[row];
              // four columns per vector reduction (ldc and N are multiples of 4)
              if (p.agg_tokens > 0) {
                // expert-parallel combine: add into the source rank's aggregate over NVLink;
                // system scope, since experts on several ranks add into one row
                float* o = p.agg_peer[tok / p.agg_tokens] + (int64_t)(tok % p.agg_tokens) * p.ldc;
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                  if (col0 + i < p.N)
                    asm volatile("red.relaxed.sys.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(o + col0 + i),
                                 "f"(w * v[i]), "f"(w * v[i + 1]), "f"(w * v[i + 2]), "f"(w * v[i + 3])
                                 : "memory");
              } else {
                float* o = reinterpret_cast<float*>(p.out) + (int64_t)tok * p.ldc;
#pragma unroll
                for (int i = 0; i < 32; i += 4)
                  if (col0 + i < p.N)
                    asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(o + col0 + i),
                                 "f"(w * v[i]), "f"(w * v[i + 1]), "f"(w * v[i + 2]), "f"(w * v[i + 3])
                                 : "memory");
              }
            }
          }
        } else if (p.epi == 3 && p.tma_store) {
          // fp32 accumulation through shared memory and TMA reduce-add (whole warp; an empty K slice adds nothing)
          if (ti.num_kb > 0) {
            const int y = ti.c_row0 + (int)rank * BM + sub * 32;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint4 pieces[4];
#pragma unroll
              for (int c = 0; c < 4; ++c)
                pieces[c] = make_uint4(__float_as_uint(v[h * 16 + 4 * c]), __float_as_uint(v[h * 16 + 4 * c + 1]),
                                       __float_as_uint(v[h * 16 + 4 * c + 2]), __float_as_uint(v[h * 16 + 4 * c + 3]));
              stage_and_store(pieces, col0 + h * 16, y, true);
            }
          }
        } else if (p.epi == 3) {
          // fp32 accumulation into `out` (split-K slices, or a gradient that already holds a value)
          if (row_ok && ti.num_kb > 0) {
            float* o = reinterpret_cast<float*>(p.out) + (int64_t)row * p.ldc;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              if (col0 + i + 4 <= p.N) {
                asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(o + col0 + i),
                             "f"(v[i]), "f"(v[i + 1]), "f"(v[i + 2]), "f"(v[i + 3])
                             : "memory");
              } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  if (col0 + i + j < p.N) atomicAdd(o + col0 + i + j, v[i + j]);
              }
            }
          }
        } else if (p.tma_store) {
          // the whole warp takes part (rows past the end are clipped by the TMA store)
          if (p.bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < p.N) v[i] += __ldg(p.bias + col0 + i);
          }
          const int y = ti.c_row0 + (int)rank * BM + sub * 32;
          if (p.out_fp32) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              uint4 pieces[4];
#pragma unroll
              for (int c = 0; c < 4; ++c)
                pieces[c] = make_uint4(__float_as_uint(v[h * 16 + 4 * c]), __float_as_uint(v[h * 16 + 4 * c + 1]),
                                       __float_as_uint(v[h * 16 + 4 * c + 2]), __float_as_uint(v[h * 16 + 4 * c + 3]));
              stage_and_store(pieces, col0 + h * 16, y, false);
            }
          } else {
            if (p.resid && row_ok) {
              const __nv_bfloat16* rr = p.resid + (int64_t)row * p.ldr;
#pragma unroll
              for (int i = 0; i < 32; i += 8) {
                if (col0 + i + 8 <= p.N) {
                  Vec<__nv_bfloat16> vr;
                  vr.load(rr + col0 + i);
#pragma unroll
                  for (int j = 0; j < 8; ++j) v[i + j] += vr.f(j);
                } else {
                  for (int j = 0; j < 8; ++j)
                    if (col0 + i + j < p.N) v[i + j] += to_f<__nv_bfloat16>(rr[col0 + i + j]);
                }
              }
            }
            uint4 pieces[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              Vec<__nv_bfloat16> o;
#pragma unroll
              for (int j = 0; j < 8; ++j) o.v[j] = from_f<__nv_bfloat16>(v[8 * c + j]);
              pieces[c] = *reinterpret_cast<const uint4*>(o.v);
            }
            stage_and_store(pieces, col0, y, false);
          }
        } else if (row_ok && !(p.debug & 1)) {
          const int64_t goff = p.mode == 2 ? (int64_t)ti.g * p.M * p.ldc : 0;
          if (p.bias) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (col0 + i < p.N) v[i] += __ldg(p.bias + col0 + i);
          }
          if (p.out_fp32) {
            float* o = reinterpret_cast<float*>(p.out) + goff + (int64_t)row * p.ldc;
#pragma unroll
            for (int i = 0; i < 32; i += 4) {
              if (col0 + i + 4 <= p.N) {
                *reinterpret_cast<float4*>(o + col0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
              } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  if (col0 + i + j < p.N) o[col0 + i + j] = v[i + j];
              }
            }
          } else {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + goff + (int64_t)row * p.ldc;
            const __nv_bfloat16* rr = p.resid ? p.resid + (int64_t)row * p.ldr : nullptr;
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              if (col0 + i + 8 <= p.N) {
                Vec<__nv_bfloat16> vo;
                if (rr) {
                  Vec<__nv_bfloat16> vr;
                  vr.load(rr + col0 + i);
#pragma unroll
                  for (int j = 0; j < 8; ++j) vo.v[j] = from_f<__nv_bfloat16>(v[i + j] + vr.f(j));
                } else {
#pragma unroll
                  for (int j = 0; j < 8; ++j) vo.v[j] = from_f<__nv_bfloat16>(v[i + j]);
                }
                vo.store(o + col0 + i);
              } else {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  if (col0 + i + j < p.N)
                    o[col0 + i + j] =
                        from_f<__nv_bfloat16>(v[i + j] + (rr ? to_f<__nv_bfloat16>(rr[col0 + i + j]) : 0.f));
              }
            }
          }
        }
      }
      // this warp is done with the accumulator: one arrival per warp on the MMA issuer's barrier
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR)
          tc::mbar_arrive_cluster(buf ? tempty_c0_1 : tempty_c0_0);
        else
          tc::mbar_arrive(&tempty[buf]);
      }
      if constexpr (CM == 1 || CM == 2) {
        // this rank's partial tile is in the symmetric buffer: tell the tile's owner
        fence_sys();
        epi_bar();
        if (threadIdx.x == 64) {
          const int owner = tile_owner(p.cm, tile, ti.m0);
          red_release_sys(reinterpret_cast<uint32_t*>(p.cm.flags_peer[owner]) + tile, 1u);
        }
      }
    }
    // the staging buffers are shared memory of this CTA: its stores must have read them before it exits
    if (lane == 0 && stores) tc::bulk_wait_read<0>();
    if ((p.debug & 2) && lane == 0 && warp == 2) atomicAdd(p.dbg + 5, (unsigned long long)(clock64() - t_epi));
    if (lane == 0) dbg_stamp(p, 13, false);
    __syncwarp();
  } else {
    if constexpr (CM == 3)
      ag_copy_loop(p);
    else if constexpr (CM != 0)
      comm_loop<BN>(p, total);
  }
  tc::tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) tc::cluster_sync();  // neither CTA leaves while the other may still touch its memory
  tc::tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      tc::tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tc::tmem_dealloc(tmem_base, TMEM_COLS);
    if (lane == 0) dbg_stamp(p, 14, false);
  }
}


// All-gather comm warps (threads 320..447): copy remote 128-row blocks of A into the local gather
// buffer in the order the tiles consume them, eight 16-byte loads in flight per thread, then
// release the block's flag.
__device__ void ag_copy_loop(const DevParams& p) {
  const int ct = threadIdx.x - 320;
  const int tm = p.M / BM, bpr = p.ag_rows / BM, rem = tm - bpr;
  const uint32_t target = *p.ag_epoch + 1u;
  const int chunks = (int)(p.ag_ld / 16);  // 16-byte chunks per row (K * 2 / 16)
  const int per_block = BM * chunks;
  for (int j = blockIdx.x; j < rem; j += gridDim.x) {
    const int mb = (p.ag_rank * bpr + bpr + j) % tm;
    const int owner = mb / bpr;
    const int64_t base = (int64_t)mb * BM * p.ag_ld;
    const uint4* src = reinterpret_cast<const uint4*>(p.ag_peer[owner] + base);
    uint4* dst = reinterpret_cast<uint4*>(p.ag_local + base);
    for (int i0 = ct; i0 < per_block; i0 += 128 * 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * 128;
        if (i < per_block) v[u] = src[i];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * 128;
        if (i < per_block) dst[i] = v[u];
      }
    }
    __threadfence();
    comm_bar();
    if (ct == 0) asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p.ag_flags + mb), "r"(target) : "memory");
  }
}

// Comm warps (threads 320..447): reduce the tiles this rank owns, then hand every tile's sum out.
template <int BN>
__device__ void comm_loop(const DevParams& p, int total) {
  __shared__ int s_ok;
  const CommParams& c = p.cm;
  const int ct = threadIdx.x - 320;
  uint32_t* my_flags = reinterpret_cast<uint32_t*>(c.flags_peer[c.rank]);
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
    const TileInfo ti = tile_info<BN>(p, tile);
    const int rows = min(BM, p.M - ti.m0), cols = min(BN, p.N - ti.n0);
    const int cpr = cols / 8;  // 16-byte chunks per row
    const int n = rows * cpr;
    if (tile_owner(c, tile, ti.m0) == c.rank) {
      if (ct == 0) {
        const bool ok = wait_geq(my_flags + tile, (uint32_t)c.world, c.timeout_ns, p.status);
        if (ok) atomicSub(my_flags + tile, (uint32_t)c.world);
        s_ok = ok;
      }
      comm_bar();
      if (s_ok) {
        for (int idx = ct; idx < n; idx += 128) {
          const int r = idx / cpr, c8 = idx - r * cpr;
          const int64_t off = ((int64_t)(ti.m0 + r) * p.N + ti.n0 + c8 * 8) * 2;  // bytes
          uint4 v;
          if (c.part_mc) {
            v = mc_ld_reduce_bf16x8(c.part_mc + off);
          } else {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int q = 0; q < c.world; ++q)
              add_bf16x8(acc, ld_sys16(reinterpret_cast<const void*>(c.part_peer[q] + off)));
            v = pack_bf16x8(acc);
          }
          if (c.mode == 2) {
            __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(c.out) +
                               (int64_t)(ti.m0 + r - c.rank * c.rows_per_rank) * c.ldo + ti.n0 + c8 * 8;
            *reinterpret_cast<uint4*>(o) = v;
          } else if (c.part_mc) {
            mc_st16(c.part_mc + off, v);
          } else {
            for (int q = 0; q < c.world; ++q) st_sys16(reinterpret_cast<void*>(c.part_peer[q] + off), v);
          }
        }
        fence_sys();
      }
      comm_bar();
      if (ct == 0 && s_ok)
        for (int q = 0; q < c.world; ++q)
          red_release_sys(reinterpret_cast<uint32_t*>(c.flags_peer[q]) + c.tiles_cap + tile, 1u);
    }
    // every rank: wait for the owner's sum, then (all-reduce) copy it out of the buffer
    if (ct == 0) {
      const bool ok = wait_geq(my_flags + c.tiles_cap + tile, 1u, c.timeout_ns, p.status);
      if (ok) atomicSub(my_flags + c.tiles_cap + tile, 1u);
      s_ok = ok;
    }
    comm_bar();
    if (s_ok && c.mode == 1) {
      const char* part = reinterpret_cast<const char*>(c.part_peer[c.rank]);
      for (int idx = ct; idx < n; idx += 128) {
        const int r = idx / cpr, c8 = idx - r * cpr;
        const int64_t e = (int64_t)(ti.m0 + r) * p.N + ti.n0 + c8 * 8;
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(c.out) + (int64_t)(ti.m0 + r) * c.ldo + ti.n0 +
                                  c8 * 8) = ld_sys16(part + e * 2);
      }
    }
    comm_bar();
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 3-D bf16 map: dims (d0 innermost, d1, d2), strides in bytes for d1 and d2, box (b0, b1, 1), 128B swizzle.
bool make_map(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
              uint32_t b0, uint32_t b1) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_map_2d(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t s1, uint32_t b0, uint32_t b1) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {d0, d1};
  cuuint64_t strides[1] = {s1};
  cuuint32_t box[2] = {b0, b1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Output map of the TMA-store epilogue: [rows, cols] with a row pitch of ld_bytes, boxes of 32 rows x 64
// bytes (32 bf16 or 16 fp32 columns), 64-byte swizzle (the layout the epilogue writes into shared memory).
bool make_store_map(CUtensorMap* m, void* ptr, uint64_t cols, uint64_t rows, uint64_t ld_bytes, bool fp32) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_bytes};
  cuuint32_t box[2] = {fp32 ? 16u : 32u, 32u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool debug_on() {
  static const bool on = getenv("KIMI_K3_DEBUG") != nullptr;
  return on;
}

template <int BN, bool AMN, bool BMN, int CM = 0, bool PAIR = false>
cudaError_t launch(const DevParams& dp, int num_sms, cudaStream_t s) {
  // an error left by an unrelated earlier call on this host thread is not this launch's
  const cudaError_t stale = cudaGetLastError();
  if (debug_on() && stale != cudaSuccess) fprintf(stderr, "tc_gemm: stale error before launch: %s\n", cudaGetErrorString(stale));
  constexpr int STAGES = ring_stages<BN, PAIR>();
  constexpr int STAGE = BM * BK * 2 + (PAIR ? BN / 2 : BN) * BK * 2;
  const size_t smem = 1024 + (size_t)STAGES * STAGE + kStagingBytes + (2 * STAGES + 5) * 8 + 16;
  auto kern = gemm_tc_kernel<BN, AMN, BMN, CM, PAIR>;
  constexpr int threads = CM ? 448 : 320;
  {
    cudaError_t e = ensure_dynamic_smem(kern, (int)smem);
    if (debug_on() && e != cudaSuccess) fprintf(stderr, "tc_gemm: smem attribute failed: %s\n", cudaGetErrorString(e));
    if (e != cudaSuccess) return e;
  }
  int grid = num_sms;
  if constexpr (PAIR) {
    // one CTA pair (a cluster of two) per pair of SMs, as many as can be resident at once
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int clusters[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && clusters[dev] == 0) {
      int n = 0;
      cfg.gridDim = dim3(num_sms & ~1);
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = num_sms / 2;
      }
      clusters[dev] = n < num_sms / 2 ? n : num_sms / 2;
    }
    grid = 2 * ((dev >= 0 && dev < 64) ? clusters[dev] : num_sms / 2);
    cfg.gridDim = dim3(grid);
    cudaLaunchKernelEx(&cfg, kern, dp);
  } else {
    kern<<<grid, threads, smem, s>>>(dp);
  }
  const cudaError_t e = cudaGetLastError();
  if (debug_on() && e != cudaSuccess) {
    int dev = -1, maxs = -1;
    cudaGetDevice(&dev);
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    maxs = fa.maxDynamicSharedSizeBytes;
    fprintf(stderr, "tc_gemm: launch failed: %s (device %d, grid %d, smem %zu, max dynamic smem %d, params %zu)\n",
            cudaGetErrorString(e), dev, grid, smem, maxs, sizeof(DevParams));
  }
  return e;
}

// Status word of launches that pass none (one per device): a failed bounded wait records its code
// here, and every later launch on that device winds down at once until the host reads and clears
// it with tc_gemm_status(true).
__device__ int g_gemm_status = 0;

constexpr int kMaxDevices = 64;
std::mutex g_status_mutex;
int* g_status_ptr[kMaxDevices] = {};

int* default_status() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mutex);
  if (!g_status_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

}  // namespace

int tc_gemm_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_gemm_status, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

int* tc_gemm_default_status() { return default_status(); }

cudaError_t tc_gemm(const TcGemmArgs& a, cudaStream_t stream) {
  // The driver's tensor-map encoder needs the device's context current on this host thread; a
  // thread whose first CUDA work is this call (an autograd worker entering a backward) has not
  // bound it yet.  cudaFree(nullptr) binds it (once per thread).
  static thread_local bool bound = false;
  if (!bound) {
    (void)cudaFree(nullptr);
    bound = true;
  }
  DevParams dp{};
  dp.mode = a.mode;
  dp.M = a.M;
  dp.N = a.N;
  dp.K = a.K;
  dp.G = a.G;
  dp.offsets = a.offsets;
  dp.uniform_rows = a.mode == 1 ? a.uniform_rows : 0;
  dp.b2_k_split = a.b2_k_split;
  dp.situ = a.epi == 1 ? 1 : 0;
  dp.epi = a.epi;
  dp.out = a.out;
  dp.out_fp32 = a.out_fp32 ? 1 : 0;
  dp.ldc = a.ldc;
  dp.out_g = a.out_g;
  dp.out_u = a.out_u;
  dp.bg = a.bg;
  dp.bu = a.bu;
  dp.row_token = a.row_token;
  dp.row_weight = a.row_weight;
  dp.agg_tokens = a.agg_tokens;
  for (int r = 0; r < 8; ++r) dp.agg_peer[r] = reinterpret_cast<float*>(a.agg_peer[r]);
  if (a.agg_tokens > 0 && (a.epi != 2 || !a.agg_peer[0])) return cudaErrorInvalidValue;
  if (a.epi == 2 && (a.N % 4 || a.ldc % 4 || (reinterpret_cast<uintptr_t>(a.out) & 15))) return cudaErrorInvalidValue;
  dp.ag_world = a.ag_world;
  dp.ag_rows = a.ag_rows;
  dp.ag_rank = a.ag_rank;
  dp.ag_local = reinterpret_cast<uint8_t*>(const_cast<void*>(a.a));
  dp.ag_flags = a.ag_flags;
  dp.ag_epoch = a.ag_epoch;
  dp.ag_ld = a.a_ld * 2;
  for (int r = 0; r < 8; ++r) dp.ag_peer[r] = reinterpret_cast<const uint8_t*>(a.ag_peer[r]);
  if (a.ag_world > 0 && (a.ag_world > 8 || a.a_mn || a.mode != 0 || a.epi != 0 || a.comm_mode != 0 ||
                         a.ag_rows <= 0 || a.ag_rows % 128 || a.M != a.ag_world * a.ag_rows || a.a_rows != a.M ||
                         a.ag_rank < 0 || a.ag_rank >= a.ag_world || !a.ag_flags || !a.ag_epoch || !a.status ||
                         (a.a_ld * 2) % 16))
    return cudaErrorInvalidValue;
  dp.status = a.status ? a.status : default_status();
  if (!dp.status) return cudaErrorInvalidValue;
  dp.spin_limit = a.spin_limit > 0 ? a.spin_limit : tc::kSpinLimit;
  const int bn = a.epi == 1 ? 256 : a.bn;
  if (bn != 128 && bn != 256) return cudaErrorInvalidValue;
  if (a.epi == 1 && (a.a_mn || a.b_mn || !a.b2)) return cudaErrorInvalidValue;
  dp.ksplit = a.ksplit > 1 ? a.ksplit : 1;
  dp.debug = a.debug;
  dp.dbg = a.dbg;
  if ((a.debug & 6) && !a.dbg) return cudaErrorInvalidValue;
  dp.bias = a.bias;
  dp.resid = reinterpret_cast<const __nv_bfloat16*>(a.resid);
  dp.ldr = a.ldr;
  if (dp.ksplit > 1 && (a.mode != 0 || a.epi != 3 || a.comm_mode != 0 || a.ag_world > 0)) return cudaErrorInvalidValue;
  if (a.epi == 3 && (!a.out_fp32 || a.mode != 0 || a.comm_mode != 0)) return cudaErrorInvalidValue;
  if ((a.bias || a.resid) && (a.epi != 0 || a.mode != 0 || a.comm_mode != 0)) return cudaErrorInvalidValue;
  if (a.resid && (a.out_fp32 || a.ldr % 8 || (reinterpret_cast<uintptr_t>(a.resid) & 15))) return cudaErrorInvalidValue;
  // CTA pairs: dense non-comm launches of more than one 128-row block whose operands are both
  // K-major (pair = -1 picks this; measured on B200, an MN-major operand makes the leader's
  // per-stage copies small 64 x 64 boxes and the single-CTA 128 x 256 tile wins)
  const bool pair_ok = a.mode == 0 && a.comm_mode == 0 && a.ag_world == 0 && a.epi != 2;
  const bool pair = pair_ok && (a.pair > 0 || (a.pair < 0 && a.M > BM && !a.a_mn && !a.b_mn));
  if (a.pair > 0 && !pair_ok) return cudaErrorInvalidValue;
  // A: K-major storage [a_rows, a_cols=K]; MN-major storage [a_rows=K, a_cols=M]
  if (!a.a_mn) {
    if (!make_map_2d(&dp.map_a, a.a, a.a_cols, a.a_rows, a.a_ld * 2, 64, 128)) {
      if (debug_on()) fprintf(stderr, "tc_gemm: A tensor map failed\n");
      return cudaErrorInvalidValue;
    }
  } else {
    if (!make_map_2d(&dp.map_a, a.a, a.a_cols, a.a_rows, a.a_ld * 2, 64, 64)) return cudaErrorInvalidValue;
  }
  // B: K-major storage [G, N, K]; MN-major storage [G, K, N]
  const uint32_t bbox_rows = a.epi == 1 ? 128 : (uint32_t)(pair ? bn / 2 : bn);
  const void* bptrs[2] = {a.b, a.b2};
  CUtensorMap* bmaps[2] = {&dp.map_b, &dp.map_b2};
  for (int i = 0; i < 2; ++i) {
    if (!bptrs[i]) {
      dp.map_b2 = dp.map_b;
      continue;
    }
    bool ok;
    if (!a.b_mn)
      ok = make_map(bmaps[i], bptrs[i], a.b_cols, a.b_rows, a.b_groups, a.b_ld * 2, a.b_gstride * 2, 64, bbox_rows);
    else
      ok = make_map(bmaps[i], bptrs[i], a.b_cols, a.b_rows, a.b_groups, a.b_ld * 2, a.b_gstride * 2, 64, 64);
    if (!ok) {
      if (debug_on()) fprintf(stderr, "tc_gemm: B tensor map %d failed\n", i);
      return cudaErrorInvalidValue;
    }
  }
  if (a.seg_kind != 0) {
    // fused projection group: one map per segment; boundaries (prefix sums of the widths) must be
    // multiples of 32 (output columns) or 64 (A's K blocks / row boxes) except the last
    if (a.mode != 0 || a.comm_mode != 0 || a.ag_world != 0 || a.nseg < 1 || a.nseg > kMaxSegs || a.bias || a.resid ||
        a.epi == 1 || a.epi == 2 || (a.seg_kind == 1 && (a.epi != 0 || a.out_fp32)) ||
        (a.seg_kind == 2 && a.a_mn) || (a.seg_kind == 3 && !a.a_mn) || a.seg_kind > 3)
      return cudaErrorInvalidValue;
    const int align = a.seg_kind == 1 ? 32 : 64;
    dp.seg_kind = a.seg_kind;
    dp.nseg = a.nseg;
    dp.seg_start[0] = 0;
    for (int s = 0; s < a.nseg; ++s) {
      if (a.seg_width[s] <= 0 || !a.seg_ptr[s] || (reinterpret_cast<uintptr_t>(a.seg_ptr[s]) & 15) ||
          (a.seg_ld[s] * 2) % 16 || a.seg_ld[s] < a.seg_width[s])
        return cudaErrorInvalidValue;
      if (s + 1 < a.nseg && (dp.seg_start[s] + a.seg_width[s]) % align) return cudaErrorInvalidValue;
      dp.seg_start[s + 1] = dp.seg_start[s] + (int)a.seg_width[s];
      bool ok;
      if (a.seg_kind == 1) {
        // the TMA clips the right edge in 16-byte units: a ragged (last) segment writes its row padding
        // up to the next 8 columns, which its row stride must hold (those columns get zeros)
        const int64_t cols = (a.seg_width[s] + 7) / 8 * 8;
        ok = cols <= a.seg_ld[s] && make_store_map(&dp.seg_map[s], a.seg_ptr[s], (uint64_t)cols, (uint64_t)a.M,
                                                   (uint64_t)(a.seg_ld[s] * 2), false);
      }
      else if (a.seg_kind == 2)
        ok = make_map_2d(&dp.seg_map[s], a.seg_ptr[s], (uint64_t)a.seg_width[s], (uint64_t)a.M,
                         (uint64_t)(a.seg_ld[s] * 2), 64, 128);
      else
        ok = make_map_2d(&dp.seg_map[s], a.seg_ptr[s], (uint64_t)a.seg_width[s], (uint64_t)a.K,
                         (uint64_t)(a.seg_ld[s] * 2), 64, 64);
      if (!ok) return cudaErrorInvalidValue;
    }
    const int total_w = dp.seg_start[a.nseg];
    if ((a.seg_kind == 1 && total_w != a.N) || (a.seg_kind == 2 && total_w < a.K) || (a.seg_kind == 3 && total_w < a.M))
      return cudaErrorInvalidValue;
    if (a.seg_kind != 1) dp.map_a = dp.seg_map[0];  // map_a is prefetched; keep it a valid descriptor
    if (a.seg_kind == 1) {
      dp.map_c = dp.seg_map[0];
      dp.tma_store = 1;
    }
  }
  // Plain stores of dense / grouped-M products go through shared memory and TMA (full 32-byte
  // sectors, one instruction per 32 x 32 chunk); comm modes keep direct stores, which they fence
  // before signalling peers.
  {
    const size_t elt = a.out_fp32 ? 4 : 2;
    const int64_t out_rows = a.mode == 1 ? a.a_rows : a.M;
    if ((a.epi == 0 || (a.epi == 3 && a.out_fp32)) && (a.mode == 0 || a.mode == 1) && a.comm_mode == 0 &&
        a.ag_world == 0 && !(a.debug & 1) &&
        a.out && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0 && (a.ldc * elt) % 16 == 0 && a.ldc >= a.N &&
        (a.N * elt) % 16 == 0 &&  // the TMA clips the right edge in 16-byte units, not elements
        out_rows > 0 && make_store_map(&dp.map_c, a.out, (uint64_t)a.N, (uint64_t)out_rows, (uint64_t)(a.ldc * elt),
                                       a.out_fp32))
      dp.tma_store = 1;
  }
  int sms = a.num_sms > 0 ? a.num_sms : device_sms();
  if (a.comm_mode != 0) {
    CommParams& c = dp.cm;
    c.mode = a.comm_mode;
    c.rank = a.comm_rank;
    c.world = a.comm_world;
    c.rows_per_rank = a.comm_rows_per_rank;
    for (int q = 0; q < kMaxRanks; ++q) {
      c.part_peer[q] = a.part_peer[q];
      c.flags_peer[q] = a.flags_peer[q];
    }
    c.part_mc = a.part_mc;
    c.tiles_cap = a.tiles_cap;
    c.out = a.comm_out;
    c.ldo = a.comm_ldo;
    c.timeout_ns = a.timeout_ns;
    const bool ok = a.mode == 0 && a.epi == 0 && !a.out_fp32 && !a.a_mn && a.N % 8 == 0 && a.ldc == a.N &&
                    c.world >= 1 && c.world <= kMaxRanks && c.rank >= 0 && c.rank < c.world && a.status &&
                    a.comm_out && tc_gemm_tiles(a.M, a.N, bn) <= c.tiles_cap && a.out == (void*)c.part_peer[c.rank] &&
                    (c.mode == 1 || (c.mode == 2 && c.rows_per_rank > 0 && c.rows_per_rank % 128 == 0 &&
                                     c.rows_per_rank * c.world == a.M));
    if (!ok) return cudaErrorInvalidValue;
    if (bn == 256) {
      if (c.mode == 1) return a.b_mn ? launch<256, false, true, 1>(dp, sms, stream)
                                     : launch<256, false, false, 1>(dp, sms, stream);
      return a.b_mn ? launch<256, false, true, 2>(dp, sms, stream) : launch<256, false, false, 2>(dp, sms, stream);
    }
    if (c.mode == 1) return a.b_mn ? launch<128, false, true, 1>(dp, sms, stream)
                                   : launch<128, false, false, 1>(dp, sms, stream);
    return a.b_mn ? launch<128, false, true, 2>(dp, sms, stream) : launch<128, false, false, 2>(dp, sms, stream);
  }
  if (a.ag_world > 0)
    return (bn == 256 ? (a.b_mn ? launch<256, false, true, 3>(dp, sms, stream) : launch<256, false, false, 3>(dp, sms, stream))
                      : (a.b_mn ? launch<128, false, true, 3>(dp, sms, stream) : launch<128, false, false, 3>(dp, sms, stream)));
#define KIMI_TC_LAUNCH(BN_, AM_, BM_) return launch<BN_, AM_, BM_>(dp, sms, stream)
#define KIMI_TC_LAUNCH_PAIR(BN_, AM_, BM_) return launch<BN_, AM_, BM_, 0, true>(dp, sms, stream)
  if (pair) {
    if (bn == 256) {
      if (!a.a_mn && !a.b_mn) KIMI_TC_LAUNCH_PAIR(256, false, false);
      if (!a.a_mn && a.b_mn) KIMI_TC_LAUNCH_PAIR(256, false, true);
      if (a.a_mn && !a.b_mn) KIMI_TC_LAUNCH_PAIR(256, true, false);
      KIMI_TC_LAUNCH_PAIR(256, true, true);
    }
    if (!a.a_mn && !a.b_mn) KIMI_TC_LAUNCH_PAIR(128, false, false);
    if (!a.a_mn && a.b_mn) KIMI_TC_LAUNCH_PAIR(128, false, true);
    if (a.a_mn && !a.b_mn) KIMI_TC_LAUNCH_PAIR(128, true, false);
    KIMI_TC_LAUNCH_PAIR(128, true, true);
  }
  if (bn == 256) {
    if (!a.a_mn && !a.b_mn) KIMI_TC_LAUNCH(256, false, false);
    if (!a.a_mn && a.b_mn) KIMI_TC_LAUNCH(256, false, true);
    if (a.a_mn && !a.b_mn) KIMI_TC_LAUNCH(256, true, false);
    KIMI_TC_LAUNCH(256, true, true);
  }
  if (!a.a_mn && !a.b_mn) KIMI_TC_LAUNCH(128, false, false);
  if (!a.a_mn && a.b_mn) KIMI_TC_LAUNCH(128, false, true);
  if (a.a_mn && !a.b_mn) KIMI_TC_LAUNCH(128, true, false);
  KIMI_TC_LAUNCH(128, true, true);
#undef KIMI_TC_LAUNCH
#undef KIMI_TC_LAUNCH_PAIR
}

}  // namespace kimi
