// Expert-parallel dispatch and combine over NVLink peer memory: no NCCL, no host round trip.
//
// Every rank of the expert group holds one symmetric buffer (same layout on every rank, mapped
// into every peer) with: a flag block, a [world, E] count matrix, this rank's expert-input rows
// `xs` [r_max, L] (bf16, grouped by local expert in 128-row aligned segments) with their
// `row_token` (source rank * M + token) and `row_weight`, the fp32 aggregate `agg` [M, L], the
// published output gradient `dagg` [M, L], the expert-input gradient `dxs` [r_max, L] and the
// routing-weight gradients `dw_row` [r_max].
//
// Forward of one MoE layer (all ranks run the same launches in the same order):
//   ep_count     local per-expert counts; zero this rank's aggregate
//   ep_exchange  write the counts into every peer's count matrix, signal, wait for all peers;
//                every rank then derives the same segment layout of every owner, its own write
//                base inside each segment, and zeroes the padding rows of its own segments
//   ep_dispatch  one warp per (token, slot): the latent row goes STRAIGHT into the owner's `xs`
//                at its final grouped position (P2P stores over NVLink), with its token id and
//                routing weight; each CTA then releases a flag on every peer
//   ep_wait      the owner waits for every source's CTAs (bounded)
//   [gate|up] grouped GEMM with the SiTU epilogue on `xs`; down grouped GEMM whose epilogue adds
//   w * row into the SOURCE rank's aggregate over NVLink (system-scope atomics) -- the combine is
//   fused into the expert down-GEMM
//   ep_signal_wait  every rank's contributions have landed
// Backward:
//   publish dL/dagg into `dagg`, ep_signal_wait; ep_dy reads each row's token gradient from the
//   source's `dagg` (peer loads); local grouped GEMMs write dL/dxs into `dxs`; ep_signal_wait;
//   ep_slot_sum gathers each token's k slot gradients (and routing-weight gradients) from the
//   owners' `dxs` / `dw_row` (peer loads).
//
// Flags are counting semaphores (producers add, the waiter subtracts what it consumed), so the
// sequence replays inside a CUDA graph.  Every wait is bounded by `timeout_ns` and records
// status 6 on expiry; later launches of the sequence then skip their work.
//
// Parity: replaces the count all-to-all with its host read, the three dispatch all-to-alls and
// the return all-to-all of `training/distributed/expert_parallel.py:24-128` (reference); the
// math (no-drop routing, per-token weighted sum over slots) is the same.
#include <cstdint>

#include "common.cuh"
#include "device_info.h"
#include "kernels.h"

namespace kimi {
namespace {

constexpr int kEpTimeout = 6;

__device__ __forceinline__ uint64_t ep_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t ep_ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void ep_red_release(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void ep_fence() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ int ep_ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool ep_failed(const int* status) { return *reinterpret_cast<const volatile int*>(status); }

__device__ __forceinline__ uint32_t* flag_at(const EpPeers& p, int rank, int kind, int src) {
  return reinterpret_cast<uint32_t*>(p.flags[rank]) + kind * 8 + src;
}

// Wait until this rank's flag (kind, src) reaches `target` for every src, then consume it.
__device__ bool ep_wait_all(const EpPeers& p, int kind, uint32_t target) {
  const uint64_t t0 = ep_now();
  for (int s = 0; s < p.world; ++s) {
    uint32_t* f = flag_at(p, p.rank, kind, s);
    while (ep_ld_acquire(f) < target) {
      if (ep_failed(p.status)) return false;
      if ((int64_t)(ep_now() - t0) > p.timeout_ns) {
        atomicCAS(p.status, 0, kEpTimeout);
        return false;
      }
      __nanosleep(200);
    }
  }
  for (int s = 0; s < p.world; ++s) atomicSub_system(flag_at(p, p.rank, kind, s), target);
  return true;
}

__device__ void ep_signal_all(const EpPeers& p, int kind) {
  ep_fence();
  for (int r = 0; r < p.world; ++r) ep_red_release(flag_at(p, r, kind, p.rank), 1u);
}

__global__ void ep_count_kernel(const int64_t* __restrict__ sel, int64_t n, int E, int* __restrict__ cnt,
                                float* __restrict__ agg, int64_t agg_elems) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t i0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  for (int64_t i = i0; i < n; i += stride) {
    const int64_t e = sel[i];
    if (e >= 0 && e < E) atomicAdd(&cnt[e], 1);
  }
  float4* a4 = reinterpret_cast<float4*>(agg);
  for (int64_t i = i0; i < agg_elems / 4; i += stride) a4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// One CTA.  off[e]: start of expert e's segment in its owner's xs; base[e]: where this rank's rows
// for e start inside that segment.
__global__ void __launch_bounds__(1024) ep_exchange_kernel(EpPeers p, const int* __restrict__ cnt, int E, int per,
                                                           int L, int* __restrict__ offsets_local,
                                                           int* __restrict__ base, int* __restrict__ cursor) {
  __shared__ int tot[1024], pad[1024];
  __shared__ int ok;
  const int tid = threadIdx.x, me = p.rank, W = p.world;
  if (ep_failed(p.status)) {
    for (int j = tid; j <= per; j += blockDim.x) offsets_local[j] = 0;
    return;
  }
  for (int i = tid; i < W * E; i += blockDim.x) {
    const int r = i / E, e = i % E;
    asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p.counts[r] + me * E + e), "r"(cnt[e]) : "memory");
  }
  __syncthreads();
  if (tid == 0) {
    ep_signal_all(p, 0);
    ok = ep_wait_all(p, 0, 1u) ? 1 : 0;
  }
  __syncthreads();
  if (!ok) {
    for (int j = tid; j <= per; j += blockDim.x) offsets_local[j] = 0;
    return;
  }
  const int* cm = p.counts[me];
  for (int e = tid; e < E; e += blockDim.x) {
    int t = 0;
    for (int s = 0; s < W; ++s) t += ep_ld_relaxed(cm + s * E + e);
    tot[e] = t;
    pad[e] = (t + 127) / 128 * 128;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    const int owner0 = e / per * per;
    int off = 0;
    for (int j = owner0; j < e; ++j) off += pad[j];
    int before = 0;
    for (int s = 0; s < me; ++s) before += ep_ld_relaxed(cm + s * E + e);
    base[e] = off + before;
    cursor[e] = 0;
    if (e / per == me) {
      const int j = e - owner0;
      offsets_local[j] = off;
      if (j == per - 1) offsets_local[per] = off + pad[e];
    }
  }
  __syncthreads();
  // zero the padding rows of this rank's segments (rows [off + tot, off + pad))
  __nv_bfloat16* xs = static_cast<__nv_bfloat16*>(p.xs[me]);
  const int chunks = L / 8;
  for (int j = 0; j < per; ++j) {
    const int e = me * per + j;
    const int r0 = offsets_local[j] + tot[e], r1 = offsets_local[j] + pad[e];
    for (int i = tid; i < (r1 - r0) * chunks; i += blockDim.x) {
      const int r = r0 + i / chunks, c = i % chunks;
      reinterpret_cast<uint4*>(xs + (int64_t)r * L)[c] = make_uint4(0, 0, 0, 0);
      if (c == 0) {
        p.row_token[me][r] = -1;
        p.row_weight[me][r] = 0.f;
      }
    }
  }
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpPeers p, const __nv_bfloat16* __restrict__ latent,
                                                          const int64_t* __restrict__ sel,
                                                          const float* __restrict__ w, int M, int k, int E, int per,
                                                          int L, const int* __restrict__ base,
                                                          int* __restrict__ cursor, int* __restrict__ slot_pos) {
  const int lane = threadIdx.x & 31;
  const int64_t n = (int64_t)M * k;
  const bool failed = ep_failed(p.status);
  if (!failed) {
    const int chunks = L / 8;
    for (int64_t i = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; i < n;
         i += ((int64_t)gridDim.x * blockDim.x) >> 5) {
      const int64_t e = sel[i];
      if (e < 0 || e >= E) {
        if (lane == 0) slot_pos[i] = -1;
        continue;
      }
      const int dst = (int)(e / per), t = (int)(i / k);
      int pos = 0;
      if (lane == 0) pos = base[e] + atomicAdd(&cursor[e], 1);
      pos = __shfl_sync(0xffffffffu, pos, 0);
      const uint4* src = reinterpret_cast<const uint4*>(latent + (int64_t)t * L);
      uint4* out = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.xs[dst]) + (int64_t)pos * L);
      for (int c = lane; c < chunks; c += 32) out[c] = src[c];
      if (lane == 0) {
        p.row_token[dst][pos] = p.rank * M + t;
        p.row_weight[dst][pos] = w[i];
        slot_pos[i] = pos;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) ep_signal_all(p, 1);  // also after a failure, so no peer waits for nothing
}

__global__ void ep_wait_kernel(EpPeers p, int kind, uint32_t target) {
  if (threadIdx.x == 0) {
    ep_wait_all(p, kind, target);
    asm volatile("fence.proxy.async.global;" ::: "memory");  // peer-written rows feed TMA loads next
  }
}

__global__ void ep_signal_wait_kernel(EpPeers p, int kind) {
  if (threadIdx.x == 0) {
    ep_signal_all(p, kind);
    ep_wait_all(p, kind, 1u);
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
}

// One warp per expert row: dy = w * dagg[src][token] (bf16), dw_row = <dagg[src][token], y>.
__global__ void __launch_bounds__(256) ep_dy_kernel(EpPeers p, const int* __restrict__ offsets_total, int64_t r_max,
                                                    int M, int L, const __nv_bfloat16* __restrict__ y,
                                                    __nv_bfloat16* __restrict__ dy) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = min((int64_t)*offsets_total, r_max);
  const bool failed = ep_failed(p.status);
  const int* rt = p.row_token[p.rank];
  const float* rw = p.row_weight[p.rank];
  float* dw_row = p.dw_row[p.rank];
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    const int tok = failed ? -1 : rt[r];
    float acc = 0.f;
    if (tok >= 0) {
      const float wr = rw[r];
      const float* g = p.dagg[tok / M] + (int64_t)(tok % M) * L;
      for (int c = lane * 4; c < L; c += 128) {
        const float4 gv = *reinterpret_cast<const float4*>(g + c);
        const __nv_bfloat162* yv = reinterpret_cast<const __nv_bfloat162*>(y + r * L + c);
        const float2 y0 = __bfloat1622float2(yv[0]), y1 = __bfloat1622float2(yv[1]);
        acc += gv.x * y0.x + gv.y * y0.y + gv.z * y1.x + gv.w * y1.y;
        __nv_bfloat162* d = reinterpret_cast<__nv_bfloat162*>(dy + r * L + c);
        d[0] = __floats2bfloat162_rn(wr * gv.x, wr * gv.y);
        d[1] = __floats2bfloat162_rn(wr * gv.z, wr * gv.w);
      }
    } else {
      for (int c = lane * 4; c < L; c += 128) {
        __nv_bfloat162* d = reinterpret_cast<__nv_bfloat162*>(dy + r * L + c);
        d[0] = d[1] = __floats2bfloat162_rn(0.f, 0.f);
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) dw_row[r] = tok >= 0 ? acc : 0.f;
  }
}

// One warp per token: dlat[t] = sum_j dxs[owner_j][pos_j], dweights[t, j] = dw_row[owner_j][pos_j].
template <typename TO>
__global__ void __launch_bounds__(256) ep_slot_sum_kernel(EpPeers p, const int64_t* __restrict__ sel,
                                                          const int* __restrict__ slot_pos, int M, int k, int E,
                                                          int per, int L, TO* __restrict__ dlat,
                                                          float* __restrict__ dweights) {
  const int lane = threadIdx.x & 31;
  const bool failed = ep_failed(p.status);
  for (int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; t < M;
       t += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    for (int c = lane * 8; c < L; c += 256) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < k; ++j) {
        const int64_t e = sel[t * k + j];
        const int pos = slot_pos[t * k + j];
        if (failed || e < 0 || e >= E || pos < 0) continue;
        const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(p.dxs[e / per]) + (int64_t)pos * L + c;
        Vec<__nv_bfloat16> v;
        v.load(src);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += v.f(q);
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) dlat[t * L + c + q] = from_f<TO>(acc[q]);
    }
    if (lane < k) {
      const int64_t e = sel[t * k + lane];
      const int pos = slot_pos[t * k + lane];
      dweights[t * k + lane] = (failed || e < 0 || e >= E || pos < 0) ? 0.f : p.dw_row[e / per][pos];
    }
  }
}

int grid_for(int64_t warps) {
  int64_t b = (warps + 7) / 8;
  const int64_t cap = (int64_t)device_sms() * 8;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace

int ep_dispatch_grid(int64_t slots) { return grid_for(slots); }

cudaError_t ep_count(const int64_t* sel, int64_t n, int E, int* cnt, float* agg, int64_t agg_elems, cudaStream_t s) {
  if (E > 1024 || (agg_elems & 3)) return cudaErrorInvalidValue;
  if (cudaMemsetAsync(cnt, 0, sizeof(int) * E, s) != cudaSuccess) return cudaGetLastError();
  const int64_t work = n > agg_elems / 4 ? n : agg_elems / 4;
  int blocks = (int)((work + 255) / 256);
  {
    const int cap = device_sms() * 8;
    blocks = blocks < 1 ? 1 : (blocks > cap ? cap : blocks);
  }
  ep_count_kernel<<<blocks, 256, 0, s>>>(sel, n, E, cnt, agg, agg_elems);
  return cudaGetLastError();
}

cudaError_t ep_exchange(const EpPeers& p, const int* cnt, int E, int per, int L, int* offsets_local, int* base,
                        int* cursor, cudaStream_t s) {
  if (E > 1024 || per <= 0 || E % per || p.world * per != E || L % 8 || p.world > 8) return cudaErrorInvalidValue;
  ep_exchange_kernel<<<1, 1024, 0, s>>>(p, cnt, E, per, L, offsets_local, base, cursor);
  return cudaGetLastError();
}

cudaError_t ep_dispatch(const EpPeers& p, const void* latent, const int64_t* sel, const float* w, int M, int k, int E,
                        int per, int L, const int* base, int* cursor, int* slot_pos, cudaStream_t s) {
  if (L % 8) return cudaErrorInvalidValue;
  ep_dispatch_kernel<<<ep_dispatch_grid((int64_t)M * k), 256, 0, s>>>(
      p, static_cast<const __nv_bfloat16*>(latent), sel, w, M, k, E, per, L, base, cursor, slot_pos);
  return cudaGetLastError();
}

cudaError_t ep_wait(const EpPeers& p, int kind, uint32_t target, cudaStream_t s) {
  ep_wait_kernel<<<1, 32, 0, s>>>(p, kind, target);
  return cudaGetLastError();
}

cudaError_t ep_signal_wait(const EpPeers& p, int kind, cudaStream_t s) {
  ep_signal_wait_kernel<<<1, 32, 0, s>>>(p, kind);
  return cudaGetLastError();
}

cudaError_t ep_dy(const EpPeers& p, const int* offsets_total, int64_t r_max, int M, int L, const void* y, void* dy,
                  cudaStream_t s) {
  if (L % 4) return cudaErrorInvalidValue;
  ep_dy_kernel<<<grid_for(r_max), 256, 0, s>>>(p, offsets_total, r_max, M, L, static_cast<const __nv_bfloat16*>(y),
                                               static_cast<__nv_bfloat16*>(dy));
  return cudaGetLastError();
}

cudaError_t ep_slot_sum(const EpPeers& p, const int64_t* sel, const int* slot_pos, int M, int k, int E, int per, int L,
                        void* dlat, bool out_fp32, float* dweights, cudaStream_t s) {
  if (L % 8 || k > 32) return cudaErrorInvalidValue;
  if (out_fp32)
    ep_slot_sum_kernel<float><<<grid_for(M), 256, 0, s>>>(p, sel, slot_pos, M, k, E, per, L,
                                                          static_cast<float*>(dlat), dweights);
  else
    ep_slot_sum_kernel<__nv_bfloat16><<<grid_for(M), 256, 0, s>>>(p, sel, slot_pos, M, k, E, per, L,
                                                                  static_cast<__nv_bfloat16*>(dlat), dweights);
  return cudaGetLastError();
}

}  // namespace kimi
