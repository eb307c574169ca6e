/*
 * oracle.h -- CPU restatement of TurboFieldfare's quantized-expert math.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in edgeexpert_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it.  Nothing in the
 * product path links or calls it.
 *
 * Every function cites the reference file:line (paths relative to the
 * TurboFieldfare project root) whose arithmetic it restates.
 *
 * Conventions
 *   - fp16 / bf16 values travel as uint16_t bit patterns.
 *   - scale_type: 0 = BF16 scale/bias (the reference format), 1 = fp16.
 *   - Weight rows are row-major, packed per Quantization.packCode.
 */
#ifndef TF_ORACLE_H
#define TF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- PRNG: Sources/TurboFieldfareValidation/Support/PRNG/SplitMix64.swift:11-23,
 *            SeedTree.swift:12-19 ---------------------------------------- */
uint64_t orc_sm64_next(uint64_t *state);
float    orc_sm64_uniform(uint64_t *state, float lo, float hi);
/* Box-Muller on top of SplitMix64 (not in the reference, which only has
 * uniforms; used for the BASELINE config distributions). */
double   orc_sm64_normal(uint64_t *state);
uint64_t orc_seedtree_seed(uint64_t root, const char *label);
void     orc_fill_uniform(uint64_t *state, float lo, float hi, float *out, size_t n);

/* BASELINE config inputs: q ~ U{0..2^bits-1}, scale = |N(0,0.02)|,
 * bias = -(2^bits/2)*scale + N(0,0.002) in the storage type; fp16 normals. */
void orc_fill_synthetic_affine(uint64_t *state, int rows, int cols, int bits, int scale_type,
                               uint8_t *packed, uint16_t *scales, uint16_t *biases);
void orc_fill_normal_f16(uint64_t *state, float sigma, uint16_t *out, size_t n);

/* ---- Number formats: Quantization.swift:16-28 ---------------------------- */
uint16_t orc_bf16_bits(float x);
float    orc_bf16_to_float(uint16_t b);
uint16_t orc_f16_bits(float x);          /* IEEE binary16, round-half-even */
float    orc_f16_to_float(uint16_t h);
float    orc_scale_to_float(uint16_t bits, int scale_type);
void     orc_f32_to_f16_array(const float *in, uint16_t *out, size_t n);
void     orc_f16_to_f32_array(const uint16_t *in, float *out, size_t n);

/* ---- Affine quantization: Quantization.swift:50-102,135-177,228-349 ----- */
size_t orc_packed_row_bytes(int n, int bits);
int    orc_unpack_code(const uint8_t *buf, size_t buf_len, int index, int bits);
void   orc_pack_code(uint8_t *buf, size_t buf_len, int code, int index, int bits);
/* rows x n floats -> packed [rows][row_bytes], scales/biases [rows][n/64]
 * (BF16 bits, exactly as quantizeAffine / quantizeInt8Affine). */
int    orc_quantize_affine(const float *w, int rows, int n, int bits,
                           uint8_t *packed, uint16_t *scales, uint16_t *biases);
void   orc_dequantize_affine(const uint8_t *packed, const uint16_t *scales,
                             const uint16_t *biases, int scale_type, int rows,
                             int n, int bits, float *out);

/* ---- GEMV references ---------------------------------------------------- */
/* DequantInt4GemvRef / DequantInt8GemvRef
 * (Sources/TurboFieldfareValidation/Support/Reference/Quant/DequantInt4Gemv.swift:12-43,
 *  DequantInt8Gemv.swift:12-41): dequantize each row to fp32, then a plain
 * sequential fp32 dot.  bits in {2,3,4,8}.  y is fp32. */
void orc_affine_gemv_ref(const uint8_t *W, const uint16_t *S, const uint16_t *B,
                         int scale_type, int bits, const float *x, float *y,
                         int m, int n, int nthreads);
/* Kernel-order restatement of dequant_int4_gemv_simd
 * (Sources/TurboFieldfare/Metal/Quant/dequant_int4.metal:95-174): 32 lanes,
 * 4-group blocks of 4 bytes per lane, fma chain, per-lane affine factoring,
 * butterfly lane sum.  x is fp16 bits; y_f32 receives the fp32 accumulator,
 * y_f16 the half-rounded output (either may be NULL). */
void orc_int4_gemv_kernel_order(const uint8_t *W, const uint16_t *S, const uint16_t *B,
                                int scale_type, const uint16_t *x_f16,
                                float *y_f32, uint16_t *y_f16, int m, int n,
                                int nthreads);
/* Kernel-order dequant_int8_gemv_simd (dequant_int8.metal:56-97). */
void orc_int8_gemv_kernel_order(const uint8_t *W, const uint16_t *S, const uint16_t *B,
                                int scale_type, const uint16_t *x_f16,
                                float *y_f32, uint16_t *y_f16, int m, int n);

/* ---- Router: moe.metal:78-185, RouterTopKTests.swift:72-97,
 *      prefill.metal:478-573 -------------------------------------------- */
/* logits[e] for one token.  x~_i = float(half h_i) * float(es_i) in fp32
 * (es scale_type as given).  logits_f32: kernel-order lanes (may be NULL);
 * logits_f64: the same x~ summed in double (may be NULL). */
void orc_router_logits(const uint8_t *W8, const uint16_t *S, const uint16_t *B,
                       int scale_type, const uint16_t *hidden_f16,
                       const uint16_t *eff_scale, int es_type,
                       float *logits_f32, double *logits_f64, int E, int D);
/* top-k by strict '>' with ties to the lower expert id; softmax over the k
 * selected; out_w = half(p * float(pes[e])). k in 1..64. */
void orc_router_topk(const float *logits, int E, const uint16_t *pes, int pes_type,
                     int k, uint32_t *out_idx, uint16_t *out_w_f16, float *out_w_f32);

/* ---- Activation: moe.metal:53-60 ---------------------------------------- */
float orc_gelu_tanh(float x);

/* ---- Decode MoE: moe.metal:248-337 (phase 1), 475-511 (phase 2),
 *      SharedExpertInt4.swift:30-94, dequant_int8.metal:99-154 ---------- */
/* Expert blob: one contiguous byte blob per expert; nine byte offsets
 * (MoE.swift:4-29) in the order gate{W,s,b}, up{W,s,b}, down{W,s,b}. */
typedef struct {
    uint32_t gate_w, gate_s, gate_b, up_w, up_s, up_b, down_w, down_s, down_b;
} orc_expert_offsets;

/* acts[slot*F+f] = half(gelu(g) * u), g/u fp32 dots (reference order:
 * dequantize, sequential dot). blobs[slot] points to each expert's blob. */
void orc_moe_phase1(const uint8_t *const *blobs, const orc_expert_offsets *off,
                    int scale_type, const uint16_t *x_f16, uint16_t *acts_f16,
                    int D, int F, int top_k, int nthreads);
/* y[d] = half(residual[d] + sum_slot float(half w_slot) * down_slot[d].act_slot) */
void orc_moe_phase2(const uint8_t *const *blobs, const orc_expert_offsets *off,
                    int scale_type, const uint16_t *acts_f16, const uint16_t *w_f16,
                    const uint16_t *residual_f16, uint16_t *y_f16, float *y_f32,
                    int D, int F, int top_k, int nthreads);
/* 2/3-bit kernel-order rows (moe.metal:644-757, dequant_int4.metal:512-583)
 * and the routed phases built on them (moe.metal:950-1180).  Rows are
 * LSB-first packed: 2-bit n/4 bytes, 3-bit 3n/8 bytes; bits in {2, 3}. */
void orc_lowbit_gemv_kernel_order(const uint8_t *W, const uint16_t *S, const uint16_t *B, int scale_type,
                                  int bits, const uint16_t *x_f16, float *y_f32, uint16_t *y_f16, int m, int n,
                                  int nthreads);
void orc_moe_phase1_bits(const uint8_t *const *blobs, const orc_expert_offsets *off, int scale_type, int bits,
                         const uint16_t *x_f16, uint16_t *acts_f16, int D, int F, int top_k, int nthreads);
void orc_moe_phase2_bits(const uint8_t *const *blobs, const orc_expert_offsets *off, int scale_type, int bits,
                         const uint16_t *acts_f16, const uint16_t *w_f16, const uint16_t *residual_f16,
                         uint16_t *y_f16, float *y_f32, int D, int F, int top_k, int nthreads);
/* Shared expert.  bits 4: g=half(gemv), u=half(gemv), act=half(gelu(g)*u),
 * y=half(down.act).  bits 8: same rounding of g/u (int8 fused kernel).
 * act_out (may be NULL) receives act as fp16 bits; y_f32 the unrounded y. */
void orc_shared_expert(const uint8_t *gW, const uint16_t *gS, const uint16_t *gB,
                       const uint8_t *uW, const uint16_t *uS, const uint16_t *uB,
                       const uint8_t *dW, const uint16_t *dS, const uint16_t *dB,
                       int scale_type, int bits, const uint16_t *x_f16,
                       uint16_t *act_out, uint16_t *y_f16, float *y_f32,
                       int D, int Fs, int nthreads);

/* ---- Prefill / batched path ---------------------------------------------- */
/* PrefillTokenExpertPair (PrefillRouter.swift:4-28): 16 bytes. */
typedef struct { uint32_t token, expert, rank, weight_bits; } orc_pair;
typedef struct { uint32_t expert, pair_start, pair_count; } orc_group;
typedef struct { uint32_t group_start, group_count, pair_start, pair_count; } orc_tile;

/* Error codes of PrefillMoEGroupingError (PrefillMoEGrouping.swift:52-88). */
enum {
    ORC_GROUP_OK = 0,
    ORC_GROUP_INVALID_QUERY_COUNT = 1,
    ORC_GROUP_INVALID_TOP_K = 2,
    ORC_GROUP_INVALID_NUM_EXPERTS = 3,
    ORC_GROUP_INVALID_TILE_EXPERT_COUNT = 4,
    ORC_GROUP_PAIR_COUNT_MISMATCH = 5,
    ORC_GROUP_TOKEN_OUT_OF_RANGE = 6,
    ORC_GROUP_RANK_OUT_OF_RANGE = 7,
    ORC_GROUP_EXPERT_OUT_OF_RANGE = 8,
    ORC_GROUP_DUPLICATE_TOKEN_RANK = 9,
    ORC_GROUP_SORT_KEY_COUNT_MISMATCH = 10
};
/* PrefillMoEGrouping.groupTokenExpertPairs (PrefillMoEGrouping.swift:91-192).
 * sort_keys may be NULL (num_sort_keys ignored then).  Outputs: sorted[n_pairs],
 * offsets[E] (UINT32_MAX when empty), counts[E], groups[<=E], tiles[<=E].
 * *n_groups / *n_tiles receive the counts.  err_a/err_b receive the
 * offending values for the error cases that carry them. */
int orc_group_pairs(const orc_pair *pairs, int n_pairs, int query_count, int top_k,
                    int num_experts, int tile_expert_count,
                    const uint64_t *sort_keys, int num_sort_keys,
                    orc_pair *sorted, uint32_t *offsets, uint32_t *counts,
                    orc_group *groups, int *n_groups, orc_tile *tiles, int *n_tiles,
                    uint32_t *err_a, uint32_t *err_b);

/* prefill_moe_reduce_token_major (prefill.metal:575-596):
 * h2[t,d] = half(sum_r fma(w[t,r], partial[t,r,d])). */
void orc_reduce_token_major(const uint16_t *partials_f16, const uint16_t *w_f16,
                            uint16_t *h2_f16, int T, int top_k, int D);

/* prefill_grouped_routed_moe_batched_phase1 + _down (prefill.metal:406-440,
 * 598-670) over already-sorted pairs and a pool of expert blobs
 * (pool + expert * stride):
 *   act = half(gelu(gate) * up)     (gate/up fp32, prefill row order)
 *   route_partials[(t*K+rank)*D + d] = half(down . act)              */
void orc_grouped_routed(const uint8_t *pool, uint64_t expert_stride,
                        const orc_expert_offsets *off, int scale_type,
                        const orc_pair *sorted, int n_pairs,
                        const uint16_t *hidden_f16, int hidden_stride,
                        uint16_t *route_partials_f16, int D, int F, int top_k,
                        int nthreads);

/* prefill_dequant_int4_qmm_f16_block (prefill.metal:672-709):
 * Y[t,n] = half(sum_k fma(fma(q,s,b), x[t,k], acc)), sequential k.
 * y_f32 (may be NULL) receives the unrounded accumulator. */
void orc_int4_qmm(const uint8_t *W, const uint16_t *S, const uint16_t *B, int scale_type,
                  const uint16_t *X_f16, uint16_t *Y_f16, float *Y_f32,
                  int T, int N, int K, int nthreads);

/* ---- Error metric: Tolerance/RelError.swift:7-16 ------------------------ */
float orc_rel_error(const float *actual, const float *ref, size_t n);

/* Number of OpenMP threads available (1 when built without OpenMP). */
int orc_max_threads(void);

/* ---- dense decode stack (oracle_decoder.c) -------------------------------- */
/* rmsnorm_bf16w / rmsnorm_no_scale (Metal/Primitives/rmsnorm.metal:32-150); w NULL = no scale. */
void orc_rmsnorm(const uint16_t *x, const uint16_t *w_bf16, uint16_t *out, int rows, int d, float eps);
/* fused_qkv_epilogue (Metal/Fusions/fused.metal:84-170), in place. */
void orc_qkv_epilogue(uint16_t *q, uint16_t *k, uint16_t *v, const uint16_t *qw, const uint16_t *kw, int hd,
                      int nq, int nkv, int position, float theta, int rotated_pairs, float eps);
/* attention_decode_single (Metal/Attention/attention.metal:241-312), K/V [seq][nkv][hd]. */
void orc_attention_decode(const uint16_t *q, const uint16_t *K, const uint16_t *V, uint16_t *out, float *out32,
                          int hd, int nq, int nkv, int seq_len, int kv_start, float scale);
/* fused_post_attn_setup (Metal/Fusions/fused.metal:190-269). */
void orc_post_attn_setup(uint16_t *hidden, const uint16_t *attn, uint16_t *dense_x, uint16_t *routed_x,
                         uint16_t *router_x, const uint16_t *w_post_attn, const uint16_t *w_pre_ffn,
                         const uint16_t *w_pre_ffn2, int rows, int d, float eps);
/* fused_layer_tail (Metal/Fusions/fused.metal:271-375) after the optional post-FFN-1 norm. */
void orc_layer_tail(const uint16_t *h2, const uint16_t *h1, uint16_t *hidden, const uint16_t *w_postffn1,
                    const uint16_t *w_postffn2, const uint16_t *w_postffn, float layer_scalar, int rows, int d,
                    float eps);
/* embed_lookup_int4 (Metal/Quant/dequant_int4.metal:65-84). */
void orc_embed_int4(const uint8_t *table, const uint16_t *S, const uint16_t *B, int st, const uint32_t *tokens,
                    int T, int d, float out_scale, uint16_t *out);
/* lm_head_greedy_int4_rows_chunk_raw + _reduce (Metal/Sampling/logit.metal:687-787). */
uint32_t orc_lm_head_greedy(const uint8_t *W, const uint16_t *S, const uint16_t *B, int st, const uint16_t *x_f16,
                            int vocab, int d, float *logits, int nthreads);

/* ---- sampling (Metal/Sampling/logit.metal:42-617) ---------------------------- */
void orc_softcap_softmax(const float *logits, uint16_t *probs, int V, float softcap);
float orc_gumbel(uint64_t seed, uint32_t position, uint32_t row);
uint32_t orc_sample(const uint16_t *probs, int V, float temperature, uint32_t top_k, float top_p, uint64_t seed,
                    uint32_t position);
uint32_t orc_sample_topk64(const uint16_t *probs, int V, float temperature, float top_p, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
