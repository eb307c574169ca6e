// tf_gemv_tc.cuh -- entry of the tensor-core one-token int4 GEMV (tf_gemv_tc.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/tfcuda.h"

struct tf_context;

namespace tf {

enum : int { kGemvStream = 0, kGemvTensorCore = 1 };

// Launches a ring-streamed GEMV for `batch` int4 matrices [m][n] sharing one
// fp16 activation vector: kind kGemvStream = integer mma.sync consumers,
// kGemvTensorCore = tcgen05 kind::i8 with the codes in TMEM.  Only when the
// shapes, alignments and shared memory allow it and (unless `force`) there are
// at least as many 128-row tiles as SMs.  Sets *used; returns TF_OK without
// launching when the path does not apply.
tf_status gemv_tc_try(tf_context* ctx, const void* W, const void* S, const void* B, uint64_t wbs, uint64_t sbs,
                      uint32_t batch, const void* x, void* y, uint64_t ybs, uint32_t m, uint32_t n,
                      tf_scale_type st, cudaStream_t stream, int kind, int force, bool* used, const char* name);

// One-token int4 GEMV [m][n] with fp32 output on the ring-streamed kernel
// (the LM head's logits); TF_ERR_UNSUPPORTED_SHAPE when the kernel cannot
// take the shape.
tf_status gemv_stream_f32(tf_context* ctx, const void* W, const void* S, const void* B, const void* x, float* y32,
                          uint32_t m, uint32_t n, tf_scale_type st, cudaStream_t stream, const char* name);

// Dense int4 GEMM [t][k] x [n][k]^T with fp32 output (tf_qmm.cu).
tf_status int4_qmm_f32(tf_context* ctx, const void* weights, const void* scales, const void* biases, const void* x,
                       float* y32, uint32_t t, uint32_t n, uint32_t k, uint32_t x_stride, uint32_t y_stride,
                       tf_scale_type st, cudaStream_t stream, const char* name);

// Grouped routed experts (gate/up + GELU, then down) on the ring-streamed
// grouped kernel (tf_grouped_stream.cu); TF_ERR_UNSUPPORTED_SHAPE when the
// shapes do not suit it.
tf_status grouped_stream(tf_context* ctx, const uint8_t* pool, uint64_t stride, uint32_t num_experts,
                         const tf_expert_offsets* off, const tf_token_expert_pair* pairs, const tf_moe_group* groups,
                         const uint32_t* n_groups, const __half* hidden, uint32_t hidden_stride, __half* acts,
                         __half* partials, uint32_t T, uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st,
                         cudaStream_t s, const char* name);

}  // namespace tf
