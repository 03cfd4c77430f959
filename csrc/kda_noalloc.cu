// Allocation-free C entry point for the KDA chunked forward (declared in kda_noalloc.h).
//
// The two forward kernels (intra-chunk WY transform, then the chunk-to-chunk state scan)
// are the tcgen05 ones of kda_tc.cu; only where their intermediates live differs: here they
// are carved out of one file-scope device array instead of freshly allocated tensors.
#include <mutex>

#include "kda_noalloc.h"
#include "kernels.h"

namespace {

constexpr int kChunk = 64;                        // tokens per chunk (== head dim)
constexpr size_t kTile = 64 * 64;                 // floats in one per-chunk 64 x 64 tile
constexpr size_t kFloatsPerChunkHead = 8 * kTile + 64;  // W, U, P, Qg, Kend, states, Vp, A tiles + eGC row
constexpr size_t kScratchFloats = (size_t)KIMI_KDA_NOALLOC_MAX_CHUNK_HEADS * kFloatsPerChunkHead;

// The scratch array: 128 chunk-heads x 131,328 bytes = 16,809,984 bytes per device.
static __device__ __align__(256) float g_kda_scratch[kScratchFloats];
// Status word of this entry point's kernels (one per device, beside the scratch): a bounded wait
// inside a kernel that gives up writes its code here; kimi_kda_noalloc_last_status reads it.
static __device__ int g_noalloc_status = 0;

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
float* g_scratch_ptr[kMaxDevices] = {};  // device address of g_kda_scratch, per device
int* g_status_ptr[kMaxDevices] = {};     // device address of g_noalloc_status, per device

int scratch_for_current_device(float** out, int** status) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return KIMI_KDA_NOALLOC_BAD_SHAPE;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_kda_scratch);
    if (e != cudaSuccess) return (int)e;
    void* sp = nullptr;
    e = cudaGetSymbolAddress(&sp, g_noalloc_status);
    if (e != cudaSuccess) return (int)e;
    g_scratch_ptr[dev] = static_cast<float*>(p);
    g_status_ptr[dev] = static_cast<int*>(sp);
  }
  *out = g_scratch_ptr[dev];
  *status = g_status_ptr[dev];
  return KIMI_KDA_NOALLOC_OK;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int kimi_kda_chunk_fwd_noalloc(
    int dtype, const void* q, const void* k, const void* v, const float* g, const float* beta, const float* h0,
    void* o, float* ht, int batch, int tokens_padded, int heads, cudaStream_t stream) {
  if (batch <= 0 || heads <= 0 || tokens_padded <= 0 || tokens_padded % kChunk != 0 || dtype < 0 || dtype > 2 ||
      !q || !k || !v || !g || !beta || !o)
    return KIMI_KDA_NOALLOC_BAD_SHAPE;
  const long long chunk_heads = (long long)batch * heads * (tokens_padded / kChunk);
  if (chunk_heads > KIMI_KDA_NOALLOC_MAX_CHUNK_HEADS) return KIMI_KDA_NOALLOC_TOO_LARGE;
  float* base = nullptr;
  int* status = nullptr;
  const int st = scratch_for_current_device(&base, &status);
  if (st != KIMI_KDA_NOALLOC_OK) return st;
  const size_t tiles = (size_t)chunk_heads * kTile;
  kimi::KdaBuffers buf{base,             base + 1 * tiles, base + 2 * tiles, base + 3 * tiles,
                       base + 4 * tiles, base + 8 * tiles, base + 5 * tiles, base + 6 * tiles, base + 7 * tiles};
  return (int)kimi::kda_chunk_fwd(dtype, q, k, v, g, beta, h0, o, ht, buf, batch, tokens_padded, heads, stream,
                                  status);
}

extern "C" __attribute__((visibility("default"))) int kimi_kda_noalloc_last_status(void) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_noalloc_status, sizeof(int));
  if (e != cudaSuccess) return (int)e;
  if (v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_noalloc_status, &zero, sizeof(int));
    if (e != cudaSuccess) return (int)e;
    return KIMI_KDA_NOALLOC_WAIT_TIMEOUT;
  }
  return KIMI_KDA_NOALLOC_OK;
}

extern "C" __attribute__((visibility("default"))) const char* kimi_kda_noalloc_status_string(int status) {
  switch (status) {
    case KIMI_KDA_NOALLOC_OK:
      return "ok";
    case KIMI_KDA_NOALLOC_TOO_LARGE:
      return "kimi_kda_chunk_fwd_noalloc: batch * heads * (tokens_padded / 64) exceeds the fixed scratch array "
             "of 128 chunk-heads; split the batch into smaller calls";
    case KIMI_KDA_NOALLOC_WAIT_TIMEOUT:
      return "kimi_kda_chunk_fwd_noalloc: a kernel gave up waiting for its tensor-core work (bounded wait); "
             "the outputs of the calls since the last status check are not valid";
    case KIMI_KDA_NOALLOC_BAD_SHAPE:
      return "kimi_kda_chunk_fwd_noalloc: bad argument (tokens_padded must be a positive multiple of 64, dtype "
             "0..2, sizes positive, q/k/v/g/beta/o non-null)";
    default:
      return cudaGetErrorString(static_cast<cudaError_t>(status));
  }
}
