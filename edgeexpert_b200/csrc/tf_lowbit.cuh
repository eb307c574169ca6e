// tf_lowbit.cuh -- 2/3-bit affine GEMV and routed decode phases (tf_lowbit.cu).
#pragma once

#include <cuda_runtime.h>

#include "tfcuda.h"

namespace tf {

// Batched 2/3-bit GEMV with tf_affine_gemv_batched's arguments; y32 != NULL
// selects fp32 output instead of y.
tf_status lowbit_gemv(tf_context* ctx, uint32_t bits, const void* W, const void* S, const void* B, uint64_t wbs,
                      uint64_t sbs, uint32_t batch, const void* x, uint32_t ntok, uint32_t xrs, void* y, float* y32,
                      uint32_t yrs, uint64_t ybs, uint32_t m, uint32_t n, tf_scale_type st, cudaStream_t stream,
                      const char* name);

tf_status lowbit_phase1(tf_context* ctx, uint32_t bits, const void* pool, uint64_t stride, uint32_t E, const void* ids,
                        const void* const* blobs, const tf_expert_offsets* off, const void* x, void* acts, uint32_t d,
                        uint32_t f, uint32_t top_k, tf_scale_type st, cudaStream_t stream, const char* name);

tf_status lowbit_phase2(tf_context* ctx, uint32_t bits, const void* pool, uint64_t stride, uint32_t E, const void* ids,
                        const void* const* blobs, const tf_expert_offsets* off, const void* acts, const void* rw,
                        const void* residual, void* y, uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st,
                        cudaStream_t stream, const char* name);

}  // namespace tf
