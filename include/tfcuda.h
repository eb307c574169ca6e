/*
 * tfcuda.h -- C ABI of the B200 (sm_100a) quantized-expert hot path for
 * TurboFieldfare (Gemma 4 26B-A4B MoE).
 *
 * Every entry point ENQUEUES work on the caller's CUDA stream (passed as
 * `void* stream`, a cudaStream_t; NULL = legacy default stream) and returns
 * immediately; none synchronises, none allocates device memory, so every call
 * is usable inside CUDA-graph capture once the context exists.  This mirrors
 * the reference's encoder style, where each `encode(commandBuffer:...)`
 * appends to a caller-owned MTLCommandBuffer
 * (Sources/TurboFieldfare/Kernels/Quant/DequantInt4GEMV.swift:84-127).
 *
 * Buffers are device pointers owned by the caller (byte offsets folded in).
 * Dimensions are uint32_t.  Weight layout is the reference's MLX-affine
 * format: codes packed LSB-first (int4: element k in byte k/2, low nibble =
 * even k), one scale and one bias per 64 elements along a row, stored as BF16
 * (TF_SCALE_BF16, the reference format) or fp16 (TF_SCALE_F16).  Activations
 * and outputs are fp16.
 *
 * Errors: a non-zero tf_status, never an abort.  The reference traps on
 * contract violations (precondition) and throws Swift errors for shape
 * mismatches; here both become status codes with a message readable through
 * tf_context_last_error().
 */
#ifndef TFCUDA_H
#define TFCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TF_API __attribute__((visibility("default")))
#else
#define TF_API
#endif

#define TFCUDA_VERSION_MAJOR 0
#define TFCUDA_VERSION_MINOR 1

typedef enum {
    TF_OK = 0,
    TF_ERR_INVALID_ARG = 1,       /* null pointer, zero or inconsistent dims */
    TF_ERR_MISALIGNED = 2,        /* pointer alignment the kernel cannot accept */
    TF_ERR_UNSUPPORTED_SHAPE = 3, /* N % 64 != 0, top_k / num_experts limits, ... */
    TF_ERR_CUDA = 4,              /* CUDA runtime error (launch, attribute, copy) */
    TF_ERR_NCCL = 5,              /* NCCL error in the expert-parallel layer */
    TF_ERR_TIMEOUT = 6,           /* a bounded device-side wait gave up */
    TF_ERR_NO_DEVICE = 7,         /* no usable sm_100 device */
    TF_ERR_GROUPING = 8           /* route metadata rejected (see tf_grouping_error) */
} tf_status;

typedef enum { TF_SCALE_BF16 = 0, TF_SCALE_F16 = 1 } tf_scale_type;

typedef struct tf_context tf_context;

/* ---- library / context ------------------------------------------------- */
TF_API const char* tf_status_string(tf_status s);
TF_API void tf_version(int* major, int* minor);

/* Replaces MetalContext (Sources/TurboFieldfare/Infrastructure/Metal/MetalContext.swift:98-210):
 * binds `device`, sizes the small device workspace (router logits, selection
 * ticket, device error word, decode activations) once. */
TF_API tf_status tf_context_create(int device, tf_context** out);
TF_API void tf_context_destroy(tf_context* ctx);
TF_API const char* tf_context_last_error(const tf_context* ctx);
/* Synchronises `stream`, returns the device error bits raised by bounded
 * waits or out-of-range expert ids since the last call (and clears them).
 * TF_ERR_TIMEOUT when a wait gave up. */
TF_API tf_status tf_context_check_device(tf_context* ctx, void* stream, uint32_t* flags_out);

/* ---- dense affine GEMV --------------------------------------------------- */
/* DequantInt4GEMV.encode / encodeTgx (Sources/TurboFieldfare/Kernels/Quant/DequantInt4GEMV.swift:84-180):
 * y[m] = sum_n (q*s+b)[m][n] * x[n] with fp32 accumulation, fp16 out.
 * W: m rows of n/2 bytes; scales/biases: m rows of n/64.  n % 64 == 0.
 * W must be at least 2-byte aligned (16-byte aligned takes the bulk-copy path). */
TF_API tf_status tf_int4_gemv(tf_context* ctx, const void* W, const void* scales, const void* biases,
                       const void* x, void* y, uint32_t m, uint32_t n, tf_scale_type st,
                       void* stream);

/* DequantInt8GEMV.encode (Sources/TurboFieldfare/Kernels/Quant/DequantInt8GEMV.swift:50-81). */
TF_API tf_status tf_int8_gemv(tf_context* ctx, const void* W, const void* scales, const void* biases,
                       const void* x, void* y, uint32_t m, uint32_t n, tf_scale_type st,
                       void* stream);

/* Batched form of the two above: `batch` matrices at W + i*w_stride_bytes
 * (scales/biases at + i*sb_stride_elems elements), a shared activation block
 * of `ntok` (1..8) tokens x[t*x_row_stride + k], outputs
 * y[i*y_batch_stride + t*y_row_stride + row].  bits in {2, 3, 4, 8}: 2- and
 * 3-bit rows are LSB-first packed, n/4 and 3n/8 bytes (the *_b3 GEMVs,
 * dequant_int4.metal:512-717; W 16-byte (2-bit) / 8-byte (3-bit) aligned).
 * (No single reference counterpart: it is the GemvBench loop,
 * Tests/TurboFieldfare/Core/Kernels/Quant/GemvBench.swift:20-107, and the
 * T-token repeated-GEMV path, PrefillSharedExpert.swift:43-58, in one launch.) */
TF_API tf_status tf_affine_gemv_batched(tf_context* ctx, uint32_t bits, const void* W, const void* scales,
                                 const void* biases, uint64_t w_stride_bytes, uint64_t sb_stride_elems,
                                 uint32_t batch, const void* x, uint32_t ntok, uint32_t x_row_stride,
                                 void* y, uint32_t y_row_stride, uint64_t y_batch_stride, uint32_t m,
                                 uint32_t n, tf_scale_type st, void* stream);

/* ---- router ------------------------------------------------------------- */
/* MoE.encodeRouterGemma4 (Sources/TurboFieldfare/Kernels/MoE/MoE.swift:147-197), both
 * encoders fused into one launch:
 *   logits[e] = sum_g s*sum(q*x~) + b*sum(x~),  x~_i = float(hidden_i)*float(eff_scale_i)
 *   top_k by logit (ties -> lower id), softmax over the k, w = half(p * per_expert_scale[e]).
 * W: int8 [num_experts][d]; eff_scale [d], per_expert_scale [num_experts] are BF16.
 * out_indices uint32[top_k], out_weights fp16[top_k] (device).
 * Limits: num_experts <= 256, 1 <= top_k <= 32, d % 64 == 0. */
TF_API tf_status tf_router_topk(tf_context* ctx, const void* W, const void* scales, const void* biases,
                         const void* hidden, const void* eff_scale, const void* per_expert_scale,
                         void* out_indices, void* out_weights, uint32_t num_experts, uint32_t d,
                         uint32_t top_k, tf_scale_type st, void* stream);

/* tf_router_topk plus a copy of the fp32 router logits, out_logits float[num_experts]
 * (device, 4-byte aligned), for parity checks of the accumulator and for
 * callers that log or post-process the logits.  The reference keeps them in
 * its internal 256-float buffer (Sources/TurboFieldfare/Kernels/MoE/MoE.swift:130-137,
 * written by router_gemv_gemma4_r4, Metal/MoE/moe.metal:78-133). */
TF_API tf_status tf_router_topk_with_logits(tf_context* ctx, const void* W, const void* scales, const void* biases,
                                            const void* hidden, const void* eff_scale, const void* per_expert_scale,
                                            void* out_indices, void* out_weights, void* out_logits,
                                            uint32_t num_experts, uint32_t d, uint32_t top_k, tf_scale_type st,
                                            void* stream);

/* Same computation as tf_router_topk, for callers that cannot allocate
 * device memory (a host application whose allocator owns every device byte,
 * or code that must not allocate after start-up).  No counterpart in the
 * reference.  Needs no tf_context and allocates nothing: its scratch (router
 * logits, selection ticket, error words; about 1 KB) is a fixed array in the
 * library that every GPU loading the library keeps until process exit.
 * Limit: num_experts <= 256 (TF_ERR_UNSUPPORTED_SHAPE beyond), other limits
 * as tf_router_topk.  The first call on a device, with that device current,
 * looks up the array's device address (it writes nothing); make that first
 * call before any stream capture, and do not call cudaDeviceReset between
 * calls.  All calls on a device share the array, so calls that overlap on the
 * GPU race: serialise them on one stream.  Device-side errors (a bounded wait
 * that gave up, a skipped misaligned access) are not visible in the return
 * code of the launch; read them with tf_router_topk_noalloc_check. */
TF_API tf_status tf_router_topk_noalloc(const void* W, const void* scales, const void* biases,
                                        const void* hidden, const void* eff_scale, const void* per_expert_scale,
                                        void* out_indices, void* out_weights, uint32_t num_experts, uint32_t d,
                                        uint32_t top_k, tf_scale_type st, void* stream);

/* Companion of tf_router_topk_noalloc (no counterpart in the reference): on
 * the current device, copies the fixed array's device error flags to the host
 * and clears them, ordered on `stream`, then synchronises `stream`.  Returns
 * TF_ERR_TIMEOUT (a bounded wait gave up), TF_ERR_MISALIGNED (an access was
 * skipped) or TF_OK; *flags_out (optional) receives the raw flag bits. */
TF_API tf_status tf_router_topk_noalloc_check(void* stream, uint32_t* flags_out);

/* ---- decode MoE ---------------------------------------------------------- */
/* MoEExpertOffsets (Sources/TurboFieldfare/Kernels/MoE/MoE.swift:4-29): byte offsets of
 * the nine sub-tensors inside one expert blob, identical for all experts. */
typedef struct {
    uint32_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b;
} tf_expert_offsets;

/* Routed experts are addressed either as an HBM-resident pool
 * (expert e at pool + e*expert_stride, ids read on the device from
 * `expert_ids`, uint32[top_k]) or, when expert_ids == NULL, through `blobs`,
 * a HOST array of top_k device pointers (the reference's RoutedBlobs).
 * top_k <= 8. */

/* MoE.encodeRoutedPersistentPhase1U16Load (MoE.swift:234-266; moe.metal:248-369):
 * acts[slot*f + j] = half(gelu_tanh(gate_slot[j].x) * (up_slot[j].x)), d % 64 == 0, f % 64 == 0. */
TF_API tf_status tf_moe_phase1(tf_context* ctx, const void* pool, uint64_t expert_stride, uint32_t num_experts,
                        const void* expert_ids, const void* const* blobs, const tf_expert_offsets* offsets,
                        const void* x, void* acts, uint32_t d, uint32_t f, uint32_t top_k,
                        tf_scale_type st, void* stream);

/* MoE.encodeRoutedPersistentPhase2Reduce (MoE.swift:312-362; moe.metal:475-511):
 * y[i] = half(residual[i] + sum_slot float(w_slot) * down_slot[i].acts_slot).
 * residual may be NULL (zero). */
TF_API tf_status tf_moe_phase2(tf_context* ctx, const void* pool, uint64_t expert_stride, uint32_t num_experts,
                        const void* expert_ids, const void* const* blobs, const tf_expert_offsets* offsets,
                        const void* acts, const void* routing_weights, const void* residual, void* y,
                        uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st, void* stream);

/* The same two phases for 2- and 3-bit routed experts (the rebits output):
 * MoE.encodeRoutedPersistentPhase1U16Load / encodeRoutedPersistentPhase2Reduce
 * with bits = 2 or 3 (MoE.swift:234-362; moe_phase1_gate_up_act_b2/_b3 and
 * moe_phase2_down_reduce_b2/_b3, moe.metal:644-1180).  Arguments and results
 * as tf_moe_phase1 / tf_moe_phase2; gate/up rows are d*bits/8 bytes and down
 * rows f*bits/8 bytes, LSB-first packed; weight sub-tensor offsets, pool,
 * stride and blobs 8-byte (3-bit) or 16-byte (2-bit) aligned.  bits = 4
 * calls tf_moe_phase1 / tf_moe_phase2. */
TF_API tf_status tf_moe_phase1_bits(tf_context* ctx, uint32_t bits, const void* pool, uint64_t expert_stride,
                                    uint32_t num_experts, const void* expert_ids, const void* const* blobs,
                                    const tf_expert_offsets* offsets, const void* x, void* acts, uint32_t d,
                                    uint32_t f, uint32_t top_k, tf_scale_type st, void* stream);
TF_API tf_status tf_moe_phase2_bits(tf_context* ctx, uint32_t bits, const void* pool, uint64_t expert_stride,
                                    uint32_t num_experts, const void* expert_ids, const void* const* blobs,
                                    const tf_expert_offsets* offsets, const void* acts, const void* routing_weights,
                                    const void* residual, void* y, uint32_t d, uint32_t f, uint32_t top_k,
                                    tf_scale_type st, void* stream);

/* SharedExpertProjection (Sources/TurboFieldfare/Kernels/MoE/SharedExpertInt8.swift:9-31). */
typedef struct {
    const void* weights;
    const void* scales;
    const void* biases;
    uint32_t rows, cols;
    uint32_t bits; /* 4 or 8 */
} tf_affine_matrix;

/* SharedExpertRuntime.encode (Sources/TurboFieldfare/Kernels/MoE/SharedExpertInt4.swift:97-137):
 * g = half(gate.x), u = half(up.x), act = half(gelu(g)*u), y = half(down.act).
 * scratch_act: caller-owned fp16[gate.rows] (the reference's scratchAct). */
TF_API tf_status tf_shared_expert(tf_context* ctx, const void* x, const tf_affine_matrix* gate,
                           const tf_affine_matrix* up, const tf_affine_matrix* down, void* y,
                           void* scratch_act, tf_scale_type st, void* stream);

/* One MoE FFN decode layer for one token (RealForwardRunner.produceToken's MoE
 * section, Sources/TurboFieldfare/Runtime/Inference/RealForwardRunner.swift:2480-2860,
 * without the SSD fetch: experts are HBM resident):
 *   router(router_x) -> top_k ids/weights (kept on the device)
 *   y = half(residual + sum_slot w_slot*routed_slot(x) + shared(x))
 * shared_* with rows == 0 disables the shared expert; residual may be NULL.
 * out_indices / out_weights (device, optional) receive the routing. */
typedef struct {
    const void* router_w;
    const void* router_s;
    const void* router_b;
    const void* eff_scale;        /* BF16 [d] */
    const void* per_expert_scale; /* BF16 [num_experts] */
    const void* expert_pool;
    uint64_t expert_stride;
    uint32_t num_experts;
    tf_expert_offsets offsets;
    tf_affine_matrix shared_gate, shared_up, shared_down;
    uint32_t d, f, top_k;
    tf_scale_type scale_type;
} tf_moe_layer;

TF_API tf_status tf_moe_decode_layer(tf_context* ctx, const tf_moe_layer* layer, const void* router_x,
                              const void* x, const void* residual, void* y, void* out_indices,
                              void* out_weights, void* stream);

/* PrefillRouter.encodeGemma4Block (Sources/TurboFieldfare/Kernels/Prefill/MoE/PrefillRouter.swift:37-89;
 * prefill_router_gemma4_block, Metal/Prefill/prefill.metal:478-573): the router for
 * T tokens at once, hidden[t * hidden_stride + k] (fp16).  Per token: int8
 * logits as tf_router_topk, top_k (1..64) by logit with ties to the lower id,
 * softmax over the k, times per_expert_scale.  out_indices uint32[T][top_k],
 * out_weights fp16[T][top_k] (device).  num_experts <= 256; W 16-byte aligned. */
TF_API tf_status tf_router_topk_batched(tf_context* ctx, const void* W, const void* scales, const void* biases,
                                        const void* hidden, uint32_t hidden_stride, const void* eff_scale,
                                        const void* per_expert_scale, void* out_indices, void* out_weights,
                                        uint32_t T, uint32_t num_experts, uint32_t d, uint32_t top_k,
                                        tf_scale_type st, void* stream);

/* tf_router_topk_batched plus a copy of every token's fp32 logits,
 * out_logits float[T][num_experts] (device, 4-byte aligned).  The reference
 * keeps them in the kernel's threadgroup memory (prefill.metal:478-573). */
TF_API tf_status tf_router_topk_batched_with_logits(tf_context* ctx, const void* W, const void* scales,
                                                    const void* biases, const void* hidden, uint32_t hidden_stride,
                                                    const void* eff_scale, const void* per_expert_scale,
                                                    void* out_indices, void* out_weights, void* out_logits, uint32_t T,
                                                    uint32_t num_experts, uint32_t d, uint32_t top_k,
                                                    tf_scale_type st, void* stream);

/* ---- token -> expert grouping ------------------------------------------------ */
/* PrefillTokenExpertPair (Sources/TurboFieldfare/Kernels/Prefill/MoE/PrefillRouter.swift:4-28):
 * weight_bits holds the fp16 routing weight in its low 16 bits. */
typedef struct { uint32_t token, expert, rank, weight_bits; } tf_token_expert_pair;
/* PrefillMoEGroup / PrefillMoETile (PrefillMoEGrouping.swift:3-29). */
typedef struct { uint32_t expert, pair_start, pair_count; } tf_moe_group;
typedef struct { uint32_t group_start, group_count, pair_start, pair_count; } tf_moe_tile;

/* PrefillMoEGroupingError cases (PrefillMoEGrouping.swift:52-88). */
typedef enum {
    TF_GROUPING_OK = 0,
    TF_GROUPING_INVALID_QUERY_COUNT = 1,
    TF_GROUPING_INVALID_TOP_K = 2,
    TF_GROUPING_INVALID_NUM_EXPERTS = 3,
    TF_GROUPING_INVALID_TILE_EXPERT_COUNT = 4,
    TF_GROUPING_PAIR_COUNT_MISMATCH = 5,
    TF_GROUPING_TOKEN_OUT_OF_RANGE = 6,
    TF_GROUPING_RANK_OUT_OF_RANGE = 7,
    TF_GROUPING_EXPERT_OUT_OF_RANGE = 8,
    TF_GROUPING_DUPLICATE_TOKEN_RANK = 9,
    TF_GROUPING_SORT_KEY_COUNT_MISMATCH = 10
} tf_grouping_code;
typedef struct { tf_grouping_code code; uint32_t a, b; } tf_grouping_error;

/* PrefillMoEGrouping.groupTokenExpertPairs (PrefillMoEGrouping.swift:91-192), HOST
 * memory, caller's thread: validates (first offending pair wins, in the
 * reference's check order), sorts by (sort key?, expert, token, rank) and builds
 * per-expert offsets (UINT32_MAX when empty) / counts (num_experts each), groups
 * and tiles (<= num_experts each).  TF_ERR_GROUPING with `error` filled on
 * rejected metadata. */
TF_API tf_status tf_group_token_expert_pairs(const tf_token_expert_pair* pairs, uint32_t n_pairs,
                                             int32_t query_count, int32_t top_k, int32_t num_experts,
                                             int32_t tile_expert_count, const uint64_t* sort_keys,
                                             uint32_t n_sort_keys, tf_token_expert_pair* sorted,
                                             uint32_t* offsets, uint32_t* counts, tf_moe_group* groups,
                                             uint32_t* n_groups, tf_moe_tile* tiles, uint32_t* n_tiles,
                                             tf_grouping_error* error);

/* The same grouping on the device for the GPU pipeline: the input is the
 * router's token-major routing (expert_ids uint32[T*K], weights fp16[T*K]),
 * the replacement for PrefillRouter.makeTokenExpertPairs + groupTokenExpertPairs
 * without the host round trip (RealForwardRunner.swift:1750-1822).  All
 * arrays are device memory; n_groups / n_tiles are device uint32 scalars.
 * sort_keys: device uint64[num_experts] or NULL.  num_experts <= 256.
 * Out-of-range expert ids are skipped and raise the context's device error bit,
 * except UINT32_MAX, which marks an empty slot and is skipped silently. */
TF_API tf_status tf_moe_route_sort(tf_context* ctx, const void* expert_ids, const void* weights, uint32_t T,
                                   uint32_t top_k, uint32_t num_experts, uint32_t tile_expert_count,
                                   const void* sort_keys, void* sorted_pairs, void* offsets, void* counts,
                                   void* groups, void* n_groups, void* tiles, void* n_tiles, void* stream);

/* ---- prefill GEMMs (tensor cores) -------------------------------------------------- */
/* PrefillInt4QMM.encode (Sources/TurboFieldfare/Kernels/Prefill/Primitives/PrefillPrimitives.swift:73-122;
 * prefill.metal:672-709) and MPPPrefillInt4QMM.encode (Kernels/TensorCore/MPPPrefillInt4QMM.swift:34-78):
 * Y[t][j] = half(sum_i w[j][i] * X[t][i]) for t < T, j < n, with w the int4
 * affine weight [n][k] dequantised to fp16 (fma(q, s, b), one rounding) and
 * an fp32 accumulator.  x_stride / y_stride in elements (0 = dense).
 * k % 64 == 0; weights and x 16-byte aligned; x_stride % 8 == 0. */
TF_API tf_status tf_int4_qmm(tf_context* ctx, const void* weights, const void* scales, const void* biases,
                             const void* x, void* y, uint32_t t, uint32_t n, uint32_t k, uint32_t x_stride,
                             uint32_t y_stride, tf_scale_type st, void* stream);

/* Prefill shared expert: per token the SharedExpertRuntime.encode arithmetic
 * (SharedExpertInt4.swift:97-137, g = half(gate.x), u = half(up.x),
 * act = half(gelu(g) * u), y = half(down.act)) over T tokens at once
 * (the reference loops T GEMVs, PrefillSharedExpert.swift:43-58).
 * act_scratch: fp16[T][gate.rows], 16-byte aligned.  int4 projections only. */
TF_API tf_status tf_prefill_shared_expert(tf_context* ctx, const void* x, uint32_t x_stride,
                                          const tf_affine_matrix* gate, const tf_affine_matrix* up,
                                          const tf_affine_matrix* down, void* act_scratch, void* y,
                                          uint32_t y_stride, uint32_t T, tf_scale_type st, void* stream);

/* PrefillGroupedRoutedMoE.encodeStreamedBatched
 * (Sources/TurboFieldfare/Kernels/Prefill/MoE/PrefillGroupedRoutedMoE.swift:446-527;
 * prefill.metal:336-440,598-670) over every group at once: for sorted pair p
 * = (token t, expert e, rank r)
 *   act_scratch[p][j]          = half(gelu(gate_e[j].x_t) * (up_e[j].x_t))
 *   route_partials[t*top_k+r][i] = half(down_e[i].act_scratch[p])
 * sorted_pairs / groups / n_groups are the device outputs of tf_moe_route_sort
 * (or the host grouping copied to the device).  act_scratch: fp16[T*top_k][f];
 * route_partials: fp16[T*top_k][d].  num_experts <= 256, d and f multiples of 64,
 * expert matrices 16-byte aligned inside the blob. */
TF_API tf_status tf_moe_grouped_routed(tf_context* ctx, const void* pool, uint64_t expert_stride,
                                       uint32_t num_experts, const tf_expert_offsets* offsets,
                                       const void* sorted_pairs, const void* groups, const void* n_groups,
                                       const void* hidden, uint32_t hidden_stride, void* act_scratch,
                                       void* route_partials, uint32_t T, uint32_t d, uint32_t f, uint32_t top_k,
                                       tf_scale_type st, void* stream);

/* tf_moe_grouped_routed with the caller's estimate of the pairs the groups
 * hold (0: all T*top_k).  The estimate only picks the kernel (the grouped
 * ring-streamed kernel up to 24 pairs per expert, the tcgen05 GEMMs above);
 * results are the same either way.  For rows whose slots mostly belong to
 * other ranks (expert parallelism: tf_ep_dispatch_unpack* marks them
 * UINT32_MAX), T*top_k overstates the work by the number of ranks.  No
 * reference counterpart beyond tf_moe_grouped_routed's. */
TF_API tf_status tf_moe_grouped_routed_expected(tf_context* ctx, const void* pool, uint64_t expert_stride,
                                                uint32_t num_experts, const tf_expert_offsets* offsets,
                                                const void* sorted_pairs, const void* groups, const void* n_groups,
                                                const void* hidden, uint32_t hidden_stride, void* act_scratch,
                                                void* route_partials, uint32_t T, uint32_t d, uint32_t f,
                                                uint32_t top_k, uint32_t expected_pairs, tf_scale_type st,
                                                void* stream);

/* PrefillMoE.encodeReduceTokenMajor (Sources/TurboFieldfare/Kernels/Prefill/MoE/PrefillMoE.swift:11-40;
 * prefill.metal:575-596): h2[t][i] = half(sum_r fma(w[t][r], partial[t*top_k+r][i])), rank order.
 * routing_weights fp16[T][top_k]; partials and h2 16-byte aligned, d % 8 == 0. */
TF_API tf_status tf_moe_reduce_token_major(tf_context* ctx, const void* route_partials, const void* routing_weights,
                                           void* h2, uint32_t T, uint32_t top_k, uint32_t d, void* stream);

/* ---- dense decode stack (the Gemma 4 decoder layer around the MoE FFN) ----------------------
 * RealForwardRunner.produceToken (Sources/TurboFieldfare/Runtime/Inference/RealForwardRunner.swift:2240-2480).
 * Norm weights are BF16 [d] (or [head_dim]); activations fp16; rows are tokens. */

/* rmsnorm_bf16w / rmsnorm_no_scale (Sources/TurboFieldfare/Metal/Primitives/rmsnorm.metal:32-150):
 * out[r][i] = half(x[r][i] * rsqrt(mean_i(x^2) + eps) * w[i]); weight NULL = no scale.
 * Strides in elements (0 = d). */
TF_API tf_status tf_rmsnorm(tf_context* ctx, const void* x, uint32_t x_stride, const void* weight, void* out,
                            uint32_t out_stride, uint32_t rows, uint32_t d, float eps, void* stream);

/* fused_qkv_epilogue (Sources/TurboFieldfare/Metal/Fusions/fused.metal:84-170), in place, for T
 * tokens: per head RMSNorm over head_dim (Q and K times the shared BF16 q/k
 * weight, V without scale), rounded to fp16, then NeoX RoPE at `position`
 * (freq = theta^(-2i/head_dim)) on the first rotated_pairs pairs of Q and K.
 * q[t*q_stride + h*head_dim + i]; k/v: the cache slots of this position,
 * token t at k + t*kv_stride elements.  head_dim even, <= 512. */
TF_API tf_status tf_qkv_epilogue(tf_context* ctx, void* q, uint32_t q_stride, void* k, void* v, uint64_t kv_stride,
                                 const void* q_weight, const void* k_weight, uint32_t head_dim, uint32_t num_q_heads,
                                 uint32_t num_kv_heads, uint32_t T, uint32_t position, float theta,
                                 uint32_t rotated_pairs, float eps, void* stream);

/* Split-KV GQA decode attention over an fp16 cache
 * (attention_decode_partial / _combine, Sources/TurboFieldfare/Metal/Attention/attention.metal:135-240;
 * the same online-softmax result as attention_decode_single :241-312):
 * out[t][h] = half(sum_p softmax_p(scale * q[t][h].k_p) v_p), p in [kv_start, seq_len),
 * kv head = h / (num_q_heads / num_kv_heads).  Caches are [seq][num_kv_heads][head_dim]
 * per token, token t at + t*seq_stride elements.  head_dim a multiple of 8 up to 256 (or 512);
 * at most 8 query heads per KV head.  workspace: caller-owned device scratch of
 * tf_attention_workspace_bytes (the reference's m/d/o partial buffers). */
TF_API size_t tf_attention_workspace_bytes(const tf_context* ctx, uint32_t T, uint32_t head_dim, uint32_t num_q_heads,
                                           uint32_t num_kv_heads, uint32_t seq_len);
TF_API tf_status tf_attention_decode(tf_context* ctx, const void* q, uint32_t q_stride, const void* k_cache,
                                     const void* v_cache, uint64_t seq_stride, void* out, uint32_t out_stride,
                                     uint32_t head_dim, uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t T,
                                     uint32_t seq_len, uint32_t kv_start, float scale, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* fused_post_attn_setup (Sources/TurboFieldfare/Metal/Fusions/fused.metal:190-269), per row:
 *   hidden = half(hidden + half(attn * inv(attn) * w_post_attn));
 *   dense_x = half(hidden * inv(hidden) * w_pre_ffn), routed_x = ... * w_pre_ffn2,
 *   router_x = half(hidden * inv(hidden)).  dense_x / routed_x / router_x may be NULL. */
TF_API tf_status tf_post_attn_setup(tf_context* ctx, void* hidden, const void* attn, void* dense_x, void* routed_x,
                                    void* router_x, const void* w_post_attn, const void* w_pre_ffn,
                                    const void* w_pre_ffn2, uint32_t rows, uint32_t d, float eps, void* stream);

/* The decoder-layer tail, the layer combine of the MoE FFN (fused_layer_tail,
 * Sources/TurboFieldfare/Metal/Fusions/fused.metal:271-375), per row, after the shared
 * expert's own post-FFN norm when w_post_ffn1 != NULL (RealForwardRunner.swift:191):
 *   h1n = half(h1 * inv(h1) * w_post_ffn1)          (h1n = h1 when w_post_ffn1 is NULL)
 *   h12 = half(h1n + half(h2 * inv(h2) * w_post_ffn2))
 *   hidden = half(half(hidden + half(h12 * inv(h12) * w_post_ffn)) * half(layer_scalar)). */
TF_API tf_status tf_layer_tail(tf_context* ctx, const void* h2, const void* h1, void* hidden, const void* w_post_ffn1,
                               const void* w_post_ffn2, const void* w_post_ffn, float layer_scalar, uint32_t rows,
                               uint32_t d, float eps, void* stream);

/* embed_lookup_int4 (Sources/TurboFieldfare/Metal/Quant/dequant_int4.metal:65-84) for T tokens:
 * out[t][i] = half((q * s + b) * out_scale) of row token_ids[t] (device uint32) of the int4
 * table [vocab][d].  An id >= vocab gives a zero row and the device error bit. */
TF_API tf_status tf_embed_int4(tf_context* ctx, const void* table, const void* scales, const void* biases,
                               const void* token_ids, uint32_t T, uint32_t vocab, uint32_t d, float out_scale,
                               void* out, uint32_t out_stride, tf_scale_type st, void* stream);

/* LMHeadChainInt4 (Sources/TurboFieldfare/Kernels/Fusions/LMHeadChainInt4.swift:1-135;
 * lm_head_greedy_int4_rows_chunk_raw / _reduce, Metal/Sampling/logit.metal:687-787):
 * x = rmsnorm_bf16w(hidden, norm_weight) -> fp32 logits = W x (int4 [vocab][d]) ->
 * out_tokens[t] = the row with the largest finite logit, ties to the lower row (0 when none).
 * Scratch (caller-owned): x_normed fp16 [T][d], logits float [T][vocab], 16-byte aligned.
 * T <= 256; one token streams the weights on the ring GEMV, more use the tcgen05 GEMM. */
TF_API tf_status tf_lm_head_greedy(tf_context* ctx, const void* hidden, uint32_t hidden_stride, const void* norm_weight,
                                   float eps, const void* W, const void* scales, const void* biases, uint32_t vocab,
                                   uint32_t d, uint32_t T, void* x_normed, void* logits, void* out_tokens,
                                   tf_scale_type st, void* stream);

/* ---- sampling (Sources/TurboFieldfare/Metal/Sampling/logit.metal:42-617;
 *      LogitSoftcapSoftmax / Sample / SampleTopK64, Kernels/Sampling/LogitOutput.swift) ---- */

/* logit_softcap_softmax: probs[r][i] = half(exp(z' - max z') / sum exp(z' - max z')),
 * z' = softcap * tanh(z / softcap), for `rows` (<= 256) rows of V logits
 * (fp32 when logits_fp32, else fp16). */
TF_API tf_status tf_softcap_softmax(tf_context* ctx, const void* logits, int logits_fp32, void* probs, uint32_t V,
                                    uint32_t rows, float softcap, void* stream);

/* Sample.encode (logit.metal:183-446) on one row of fp16 probabilities:
 * temperature <= 0: argmax (ties to the lower index); top_k == 0 and top_p
 * outside (0, 1): Gumbel-max over log(p)/T with the (seed, position, row)
 * counter draw; otherwise the top min(top_k or V, 256) by (p desc, index asc),
 * top-p against the full mass, p^(1/T), then the xorshift64* inverse-CDF draw.
 * out_token: device uint32.  V <= 262144. */
TF_API tf_status tf_sample(tf_context* ctx, const void* probs, uint32_t V, float temperature, uint32_t top_k,
                           float top_p, uint64_t seed, uint32_t position, void* out_token, void* stream);

/* SampleTopK64.encode (sample_topk64_stage1 / _reduce / _final, logit.metal:489-617):
 * the top 64 by (p desc, index asc), then the same truncating draw.  V <= 262144. */
TF_API tf_status tf_sample_topk64(tf_context* ctx, const void* probs, uint32_t V, float temperature, float top_p,
                                  uint64_t seed, void* out_token, void* stream);

/* ---- expert parallelism (routed experts sharded over GPUs) ------------------------------
 * No reference counterpart (the reference streams experts from SSD on one GPU).
 * Experts are sharded in contiguous id ranges of experts_per_rank; the
 * exchange itself is the caller's all-to-all (NCCL).
 * Every rank sends every other rank exactly `capacity` rows per layer, so the
 * all-to-all has equal splits known on the host in advance: no count readback,
 * no host synchronisation, and the whole step can be captured in a CUDA graph.
 * A row carries a token to an owner rank at most once, whatever the number of
 * its experts there.  Row layout: the token's d fp16 values, then this header
 * (row bytes = 2*d + 64): */
typedef struct {
    uint32_t local_expert[8]; /* per top-k slot: expert id on the owner, UINT32_MAX = not there */
    uint16_t weight_bits[8];  /* per slot: fp16 routing weight */
    uint32_t n_valid;         /* slots that live on the owner (0: payload not written) */
    uint32_t src_token;       /* token index on the sender */
    uint32_t reserved[2];
} tf_ep_row_header;

/* send[(r*capacity + t)] = token t of this rank for owner rank r (r < world,
 * t < capacity; t >= T gives an empty header).  expert_ids uint32[T][top_k]
 * and weights fp16[T][top_k] as tf_router_topk_batched writes them.
 * top_k <= 8, T <= capacity, send 16-byte aligned. */
TF_API tf_status tf_ep_dispatch_pack(tf_context* ctx, const void* hidden, uint32_t hidden_stride,
                                     const void* expert_ids, const void* weights, uint32_t T, uint32_t top_k,
                                     uint32_t num_experts, uint32_t experts_per_rank, uint32_t world,
                                     uint32_t capacity, uint32_t d, void* send, void* stream);

/* Owner side: the received rows' headers as token-major routing for
 * tf_moe_route_sort (which skips UINT32_MAX silently): expert_ids_out
 * uint32[rows][top_k], weights_out fp16[rows][top_k].  The received rows
 * themselves are the grouped GEMM's hidden input, stride (2*d + 64)/2 elements. */
TF_API tf_status tf_ep_dispatch_unpack(tf_context* ctx, const void* recv, uint32_t rows, uint32_t d, uint32_t top_k,
                                       void* expert_ids_out, void* weights_out, void* stream);

/* Owner side, after tf_moe_grouped_routed over the received rows:
 * out[i][:] (fp32) = sum over row i's slots on this rank, in slot order, of
 * fma(w, route_partials[i*top_k + slot][:]) -- the reference's token-major
 * reduce (prefill.metal:575-596) restricted to this rank's experts; 0 when the
 * row has none.  out 16-byte aligned. */
TF_API tf_status tf_ep_expert_combine(tf_context* ctx, const void* route_partials, const void* expert_ids,
                                      const void* weights, uint32_t rows, uint32_t top_k, uint32_t d, void* out,
                                      void* stream);

/* Sender side, after the return all-to-all (back fp32 [world][capacity][d]):
 * h2[t][:] = half(sum_r back[r][t][:]) in rank order, t < T.
 * h2_stride in elements (0 = d). */
TF_API tf_status tf_ep_return_reduce(tf_context* ctx, const void* back, uint32_t world, uint32_t capacity,
                                     uint32_t T, uint32_t d, void* h2, uint32_t h2_stride, void* stream);

/* ---- expert-parallel exchange over peer memory (no collective library on the data path) ----
 * The same fixed-capacity exchange with the two all-to-alls replaced by stores
 * into the peers' buffers over NVLink (CUDA IPC mappings of ordinary device
 * allocations; no multicast) and per-(sender, owner) arrival counters.  Each
 * rank allocates with tf_ep_ipc_alloc: recv (world*capacity rows of 2*d + 64
 * bytes), back (world*capacity*d floats) and flags (tf_ep_flag_bytes), shares
 * the 64-byte handles (e.g. an all-gather over the process group) and opens
 * its peers' with tf_ep_ipc_open.  peer_recv / peer_back / peer_flags are
 * DEVICE arrays of `world` pointers (entry r = rank r's buffer, this rank's
 * own at entry rank).  One layer:
 *   tf_ep_dispatch_p2p -> tf_ep_dispatch_unpack_p2p -> tf_moe_route_sort +
 *   tf_moe_grouped_routed (hidden = recv) -> tf_ep_combine_p2p -> tf_ep_return_reduce_p2p.
 * The waits are bounded (about 2 s); a timeout raises TF_ERR_TIMEOUT through
 * tf_context_check_device.  One process per GPU: every rank must run every
 * layer's five calls.  Buffers may be shared by consecutive layers. */
TF_API size_t tf_ep_flag_bytes(uint32_t world);
TF_API tf_status tf_ep_ipc_alloc(tf_context* ctx, size_t bytes, void** dev_ptr, void* ipc_handle /* 64 B out */);
TF_API tf_status tf_ep_ipc_open(tf_context* ctx, const void* ipc_handle, void** peer_ptr);
TF_API tf_status tf_ep_ipc_close(tf_context* ctx, void* peer_ptr);
TF_API tf_status tf_ep_ipc_free(tf_context* ctx, void* dev_ptr);
TF_API tf_status tf_ep_dispatch_p2p(tf_context* ctx, const void* hidden, uint32_t hidden_stride, const void* expert_ids,
                                    const void* weights, uint32_t T, uint32_t top_k, uint32_t num_experts,
                                    uint32_t experts_per_rank, uint32_t world, uint32_t rank, uint32_t capacity,
                                    uint32_t d, const void* peer_recv, const void* peer_flags, void* my_flags,
                                    void* stream);
TF_API tf_status tf_ep_dispatch_unpack_p2p(tf_context* ctx, const void* recv, const void* my_flags, uint32_t world,
                                           uint32_t capacity, uint32_t d, uint32_t top_k, void* expert_ids_out,
                                           void* weights_out, void* stream);
TF_API tf_status tf_ep_combine_p2p(tf_context* ctx, const void* route_partials, const void* expert_ids,
                                   const void* weights, uint32_t world, uint32_t rank, uint32_t capacity,
                                   uint32_t top_k, uint32_t d, const void* peer_back, const void* peer_flags,
                                   void* my_flags, void* stream);
TF_API tf_status tf_ep_return_reduce_p2p(tf_context* ctx, const void* back, const void* my_flags, uint32_t world,
                                         uint32_t capacity, uint32_t T, uint32_t d, void* h2, uint32_t h2_stride,
                                         void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TFCUDA_H */
