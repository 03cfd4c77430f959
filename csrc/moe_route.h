// Host interface of the device-side MoE routing kernels (moe_route.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace kimi {
cudaError_t moe_route_prep(const int64_t* sel, const float* w, int64_t M, int k, int E, int64_t r_max, int* counts,
                           int* offsets, int* cursor, int* row_token, float* row_weight, int* row_of,
                           cudaStream_t s);
cudaError_t moe_gather(const void* latent, const int* row_token, void* xs, int64_t r_max, int L, cudaStream_t s);
cudaError_t moe_dy(const float* dagg, const int* row_token, const float* row_weight, const void* y, void* dy,
                   float* dw_row, int64_t r_max, int L, cudaStream_t s);
cudaError_t moe_slot_sum(const void* dxs, const int* row_of, void* out, bool out_fp32, int64_t M, int k, int L,
                         cudaStream_t s);
cudaError_t situ_bwd_cat(const void* dh, const void* g, const void* u, void* dgu, int64_t rows, int H, float bg,
                         float bu, cudaStream_t s);
}  // namespace kimi
