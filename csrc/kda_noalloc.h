// C entry point for the KDA chunked forward that allocates no device memory.
//
// This entry point has no counterpart in the reference implementation; it exists
// for callers that must not allocate device memory while they run:
//   * an inference server that reserves its whole memory pool up front and must not
//     see a cudaMalloc (or a caching allocator growing) once it is serving;
//   * code in a C or C++ host program that links only this library, owns its buffers,
//     and has no PyTorch caching allocator to borrow scratch from;
//   * a caller that already holds a lock or a memory budget it cannot exceed.
//
// The ordinary Python path (kimi_k3_b200.ops.kda_chunk) allocates its eight per-chunk
// intermediates through PyTorch's caching allocator.  This entry point instead keeps
// them in one fixed device array compiled into the library (KIMI_KDA_NOALLOC_MAX_CHUNK_HEADS
// chunk-heads, about 16 MiB), so a call only launches the two forward kernels.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Largest batch * heads * (tokens_padded / 64) the fixed scratch array holds.
#define KIMI_KDA_NOALLOC_MAX_CHUNK_HEADS 128

// Status codes returned besides cudaError_t values (which are all below 10000).
#define KIMI_KDA_NOALLOC_OK 0
#define KIMI_KDA_NOALLOC_TOO_LARGE 10001  // batch * heads * chunks exceeds the scratch array
#define KIMI_KDA_NOALLOC_BAD_SHAPE 10002  // tokens_padded not a positive multiple of 64, or another bad argument
#define KIMI_KDA_NOALLOC_WAIT_TIMEOUT 10003  // a kernel's bounded wait gave up (kimi_kda_noalloc_last_status)

// Chunked KDA forward, o = KDA(q, k, v, g, beta; h0), with head dims of 64.
//   dtype:        0 = float32, 1 = bfloat16, 2 = float16 (q, k, v and o)
//   q, k, v, o:   [batch, tokens_padded, heads, 64], contiguous
//   g:            float32 [batch, tokens_padded, heads, 64] log decays (cumulated inside)
//   beta:         float32 [batch, tokens_padded, heads]
//   h0:           float32 [batch, heads, 64, 64] initial state, or NULL for zeros
//   ht:           float32 [batch, heads, 64, 64] final state output, or NULL
//   stream:       the cudaStream_t to launch on (a stream of the current device)
// tokens_padded must be a multiple of 64; pad q, k, v, g with zeros and beta with zeros.
//
// Allocation: none.  The per-chunk intermediates live in one file-scope device array
// of KIMI_KDA_NOALLOC_MAX_CHUNK_HEADS chunk-heads; a larger problem returns
// KIMI_KDA_NOALLOC_TOO_LARGE before anything is launched (split the batch instead).
// The kernels write every scratch element they later read, so nothing there needs to
// start at zero.
//
// Set-up: the first call on each device looks up that device's copy of the scratch
// array (and the kernels raise their shared-memory limit once per process).  Make that
// first call, on every device you use, before any stream capture begins.
//
// Sharing: every call on one device uses the SAME scratch array.  Two calls that can
// run at the same time on that device (different streams, or different host threads
// without ordering) race on it and give wrong results; order them on one stream.
//
// Returns KIMI_KDA_NOALLOC_OK, one of the codes above, or a cudaError_t value.
int kimi_kda_chunk_fwd_noalloc(int dtype, const void* q, const void* k, const void* v, const float* g,
                               const float* beta, const float* h0, void* o, float* ht, int batch, int tokens_padded,
                               int heads, cudaStream_t stream);

// Status of the kernels launched by the calls above on the current device since the last check.
// The launch itself cannot report a wait that gives up inside a kernel (every wait in these kernels
// is bounded, so a broken tensor-core pipeline ends the kernel instead of hanging the GPU); the
// kernel records it in a status word that lives beside the scratch array.  Synchronize the stream
// first, then call this: it returns KIMI_KDA_NOALLOC_OK, or KIMI_KDA_NOALLOC_WAIT_TIMEOUT (and
// clears the word) when the outputs of those calls are not valid, or a cudaError_t value if the
// word could not be read.  It allocates nothing.
int kimi_kda_noalloc_last_status(void);

// Human-readable text for a status code returned above.
const char* kimi_kda_noalloc_status_string(int status);

#ifdef __cplusplus
}
#endif
