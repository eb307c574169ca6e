/*
 * oracle_moe.c -- router/top-k, GELU, decode MoE, shared expert, grouping,
 * token-major reduce, grouped routed prefill, dense int4 QMM.
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float hround(float v) { return orc_f16_to_float(orc_f16_bits(v)); }

/* DequantInt4GemvRef.apply for one row: dequantize, sequential fp32 dot
 * (DequantInt4Gemv.swift:26-40). */
static float row_dot_ref(const uint8_t *wr, const uint16_t *sr, const uint16_t *br,
                         int st, int bits, const float *x, int n) {
    const size_t rb = orc_packed_row_bytes(n, bits);
    float dot = 0.0f;
    for (int g = 0; g < n / 64; ++g) {
        float s = orc_scale_to_float(sr[g], st), b = orc_scale_to_float(br[g], st);
        for (int k = 0; k < 64; ++k) {
            int q = orc_unpack_code(wr, rb, g * 64 + k, bits);
            dot += ((float)q * s + b) * x[g * 64 + k];
        }
    }
    return dot;
}

/* ---------------- router (moe.metal:78-185) ------------------------------- */
void orc_router_logits(const uint8_t *W8, const uint16_t *S, const uint16_t *B, int st,
                       const uint16_t *h16, const uint16_t *es, int es_type,
                       float *l32, double *l64, int E, int D) {
    const int ng = D / 64;
    float *xt = (float *)malloc(sizeof(float) * (size_t)D);
    for (int i = 0; i < D; ++i)
        xt[i] = orc_f16_to_float(h16[i]) * orc_scale_to_float(es[i], es_type);
    for (int e = 0; e < E; ++e) {
        const uint8_t *wr = W8 + (size_t)e * D;
        const uint16_t *sr = S + (size_t)e * ng, *br = B + (size_t)e * ng;
        if (l32) {
            float acc[32];
            for (int lane = 0; lane < 32; ++lane) {
                float a = 0.0f;
                for (int g = 0; g < ng; ++g) {
                    float s = orc_scale_to_float(sr[g], st), b = orc_scale_to_float(br[g], st);
                    int idx = g * 64 + lane * 2;
                    float x0 = xt[idx], x1 = xt[idx + 1];
                    a = fmaf(s, (float)wr[idx] * x0 + (float)wr[idx + 1] * x1, a);
                    a = fmaf(b, x0 + x1, a);
                }
                acc[lane] = a;
            }
            for (int off = 16; off >= 1; off >>= 1)
                for (int l = 0; l < 32; ++l)
                    if ((l & off) == 0) acc[l] += acc[l | off];
            l32[e] = acc[0];
        }
        if (l64) {
            double a = 0.0;
            for (int g = 0; g < ng; ++g) {
                double s = orc_scale_to_float(sr[g], st), b = orc_scale_to_float(br[g], st);
                double dq = 0.0, sx = 0.0;
                for (int k = 0; k < 64; ++k) {
                    dq += (double)wr[g * 64 + k] * (double)xt[g * 64 + k];
                    sx += (double)xt[g * 64 + k];
                }
                a += s * dq + b * sx;
            }
            l64[e] = a;
        }
    }
    free(xt);
}

void orc_router_topk(const float *logits, int E, const uint16_t *pes, int pes_type, int k,
                     uint32_t *out_idx, uint16_t *out_w16, float *out_w32) {
    uint32_t ti[64];
    float ts[64];
    if (k < 1) return;
    if (k > 64) k = 64;
    for (int i = 0; i < k; ++i) { ti[i] = 0; ts[i] = -INFINITY; }
    for (int e = 0; e < E; ++e) {
        float s = logits[e];
        if (s <= ts[k - 1]) continue;
        int pos = k;
        for (int i = 0; i < k; ++i)
            if (s > ts[i] || (s == ts[i] && (uint32_t)e < ti[i])) { pos = i; break; }
        if (pos >= k) continue;
        for (int i = k - 1; i > pos; --i) { ti[i] = ti[i - 1]; ts[i] = ts[i - 1]; }
        ti[pos] = (uint32_t)e;
        ts[pos] = s;
    }
    float mx = ts[0], sum = 0.0f, ex[64];
    for (int i = 0; i < k; ++i) { ex[i] = expf(ts[i] - mx); sum += ex[i]; }
    for (int i = 0; i < k; ++i) {
        float w = ex[i] / sum * orc_scale_to_float(pes[ti[i]], pes_type);
        out_idx[i] = ti[i];
        if (out_w16) out_w16[i] = orc_f16_bits(w);
        if (out_w32) out_w32[i] = w;
    }
}

/* ---------------- GELU (moe.metal:53-60) ---------------------------------- */
float orc_gelu_tanh(float x) {
    const float x3 = x * x * x;
    float inner = 0.7978845608028654f * (x + 0.044715f * x3);
    if (inner < -20.0f) inner = -20.0f;
    if (inner > 20.0f) inner = 20.0f;
    return 0.5f * x * (1.0f + tanhf(inner));
}

/* ---------------- decode MoE ------------------------------------------------ */
#define BLOB_U16(base, off) ((const uint16_t *)((const uint8_t *)(base) + (off)))

void orc_moe_phase1(const uint8_t *const *blobs, const orc_expert_offsets *o, int st,
                    const uint16_t *x16, uint16_t *acts, int D, int F, int top_k,
                    int nthreads) {
    float *x = (float *)malloc(sizeof(float) * (size_t)D);
    orc_f16_to_f32_array(x16, x, (size_t)D);
    const int ng = D / 64;
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int rowg = 0; rowg < top_k * F; ++rowg) {
        int slot = rowg / F, f = rowg % F;
        const uint8_t *b = blobs[slot];
        float g = row_dot_ref(b + o->gate_w + (size_t)f * (D / 2), BLOB_U16(b, o->gate_s) + (size_t)f * ng,
                              BLOB_U16(b, o->gate_b) + (size_t)f * ng, st, 4, x, D);
        float u = row_dot_ref(b + o->up_w + (size_t)f * (D / 2), BLOB_U16(b, o->up_s) + (size_t)f * ng,
                              BLOB_U16(b, o->up_b) + (size_t)f * ng, st, 4, x, D);
        acts[(size_t)slot * F + f] = orc_f16_bits(orc_gelu_tanh(g) * u);
    }
    free(x);
}

void orc_moe_phase2(const uint8_t *const *blobs, const orc_expert_offsets *o, int st,
                    const uint16_t *acts16, const uint16_t *w16, const uint16_t *res16,
                    uint16_t *y16, float *y32, int D, int F, int top_k, int nthreads) {
    float *acts = (float *)malloc(sizeof(float) * (size_t)top_k * F);
    orc_f16_to_f32_array(acts16, acts, (size_t)top_k * F);
    const int ng = F / 64;
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int d = 0; d < D; ++d) {
        float acc = res16 ? orc_f16_to_float(res16[d]) : 0.0f;
        for (int s = 0; s < top_k; ++s) {
            const uint8_t *b = blobs[s];
            float v = row_dot_ref(b + o->down_w + (size_t)d * (F / 2), BLOB_U16(b, o->down_s) + (size_t)d * ng,
                                  BLOB_U16(b, o->down_b) + (size_t)d * ng, st, 4, acts + (size_t)s * F, F);
            acc += orc_f16_to_float(w16[s]) * v;
        }
        if (y32) y32[d] = acc;
        if (y16) y16[d] = orc_f16_bits(acc);
    }
    free(acts);
}

void orc_shared_expert(const uint8_t *gW, const uint16_t *gS, const uint16_t *gB,
                       const uint8_t *uW, const uint16_t *uS, const uint16_t *uB,
                       const uint8_t *dW, const uint16_t *dS, const uint16_t *dB,
                       int st, int bits, const uint16_t *x16, uint16_t *act_out,
                       uint16_t *y16, float *y32, int D, int Fs, int nthreads) {
    float *x = (float *)malloc(sizeof(float) * (size_t)D);
    float *act = (float *)malloc(sizeof(float) * (size_t)Fs);
    orc_f16_to_f32_array(x16, x, (size_t)D);
    const size_t rbD = orc_packed_row_bytes(D, bits), rbF = orc_packed_row_bytes(Fs, bits);
    const int ngD = D / 64, ngF = Fs / 64;
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int f = 0; f < Fs; ++f) {
        float g = hround(row_dot_ref(gW + rbD * f, gS + (size_t)f * ngD, gB + (size_t)f * ngD, st, bits, x, D));
        float u = hround(row_dot_ref(uW + rbD * f, uS + (size_t)f * ngD, uB + (size_t)f * ngD, st, bits, x, D));
        act[f] = hround(orc_gelu_tanh(g) * u);
    }
    if (act_out) orc_f32_to_f16_array(act, act_out, (size_t)Fs);
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int d = 0; d < D; ++d) {
        float v = row_dot_ref(dW + rbF * d, dS + (size_t)d * ngF, dB + (size_t)d * ngF, st, bits, act, Fs);
        if (y32) y32[d] = v;
        if (y16) y16[d] = orc_f16_bits(v);
    }
    free(x);
    free(act);
}

/* ---------------- grouping (PrefillMoEGrouping.swift:91-192) --------------- */
static const uint64_t *g_sort_keys;
static int pair_less(const orc_pair *a, const orc_pair *b) {
    if (g_sort_keys) {
        uint64_t ka = g_sort_keys[a->expert], kb = g_sort_keys[b->expert];
        if (ka != kb) return ka < kb ? -1 : 1;
    }
    if (a->expert != b->expert) return a->expert < b->expert ? -1 : 1;
    if (a->token != b->token) return a->token < b->token ? -1 : 1;
    if (a->rank != b->rank) return a->rank < b->rank ? -1 : 1;
    return 0;
}
static int pair_cmp(const void *a, const void *b) { return pair_less((const orc_pair *)a, (const orc_pair *)b); }
static int u64_cmp(const void *a, const void *b) {
    uint64_t x = *(const uint64_t *)a, y = *(const uint64_t *)b;
    return x < y ? -1 : (x > y ? 1 : 0);
}

int orc_group_pairs(const orc_pair *pairs, int n_pairs, int T, int K, int E, int tile_e,
                    const uint64_t *sort_keys, int n_keys, orc_pair *sorted,
                    uint32_t *offsets, uint32_t *counts, orc_group *groups, int *n_groups,
                    orc_tile *tiles, int *n_tiles, uint32_t *err_a, uint32_t *err_b) {
    *n_groups = 0;
    *n_tiles = 0;
    if (T < 0) { if (err_a) *err_a = (uint32_t)T; return ORC_GROUP_INVALID_QUERY_COUNT; }
    if (K <= 0) { if (err_a) *err_a = (uint32_t)K; return ORC_GROUP_INVALID_TOP_K; }
    if (E <= 0) { if (err_a) *err_a = (uint32_t)E; return ORC_GROUP_INVALID_NUM_EXPERTS; }
    if (tile_e < 1 || tile_e > 16) { if (err_a) *err_a = (uint32_t)tile_e; return ORC_GROUP_INVALID_TILE_EXPERT_COUNT; }
    if (sort_keys && n_keys != E) {
        if (err_a) *err_a = (uint32_t)E;
        if (err_b) *err_b = (uint32_t)n_keys;
        return ORC_GROUP_SORT_KEY_COUNT_MISMATCH;
    }
    if (n_pairs != T * K) {
        if (err_a) *err_a = (uint32_t)(T * K);
        if (err_b) *err_b = (uint32_t)n_pairs;
        return ORC_GROUP_PAIR_COUNT_MISMATCH;
    }
    uint64_t *seen = (uint64_t *)malloc(sizeof(uint64_t) * (size_t)(n_pairs ? n_pairs : 1));
    for (int i = 0; i < n_pairs; ++i) {
        const orc_pair *p = &pairs[i];
        /* checks in the reference's order, first offending pair wins */
        if (p->token >= (uint32_t)T) { if (err_a) *err_a = p->token; free(seen); return ORC_GROUP_TOKEN_OUT_OF_RANGE; }
        if (p->rank >= (uint32_t)K) { if (err_a) *err_a = p->rank; free(seen); return ORC_GROUP_RANK_OUT_OF_RANGE; }
        if (p->expert >= (uint32_t)E) { if (err_a) *err_a = p->expert; free(seen); return ORC_GROUP_EXPERT_OUT_OF_RANGE; }
        uint64_t key = ((uint64_t)p->token << 32) | p->rank;
        /* duplicate check against earlier pairs (set insertion order) */
        for (int j = 0; j < i; ++j)
            if (seen[j] == key) {
                if (err_a) *err_a = p->token;
                if (err_b) *err_b = p->rank;
                free(seen);
                return ORC_GROUP_DUPLICATE_TOKEN_RANK;
            }
        seen[i] = key;
    }
    (void)u64_cmp;
    free(seen);
    memcpy(sorted, pairs, sizeof(orc_pair) * (size_t)n_pairs);
    g_sort_keys = sort_keys;
    qsort(sorted, (size_t)n_pairs, sizeof(orc_pair), pair_cmp);   /* keys are total: stable not needed */
    g_sort_keys = NULL;
    for (int e = 0; e < E; ++e) { offsets[e] = 0xFFFFFFFFu; counts[e] = 0; }
    int ng = 0, i = 0;
    while (i < n_pairs) {
        uint32_t ex = sorted[i].expert;
        int start = i;
        while (i < n_pairs && sorted[i].expert == ex) ++i;
        offsets[ex] = (uint32_t)start;
        counts[ex] = (uint32_t)(i - start);
        groups[ng].expert = ex;
        groups[ng].pair_start = (uint32_t)start;
        groups[ng].pair_count = (uint32_t)(i - start);
        ++ng;
    }
    int nt = 0;
    for (int gs = 0; gs < ng; gs += tile_e) {
        int ge = gs + tile_e < ng ? gs + tile_e : ng;
        tiles[nt].group_start = (uint32_t)gs;
        tiles[nt].group_count = (uint32_t)(ge - gs);
        tiles[nt].pair_start = groups[gs].pair_start;
        tiles[nt].pair_count = groups[ge - 1].pair_start + groups[ge - 1].pair_count - groups[gs].pair_start;
        ++nt;
    }
    *n_groups = ng;
    *n_tiles = nt;
    return ORC_GROUP_OK;
}

/* ---------------- token-major reduce (prefill.metal:575-596) -------------- */
void orc_reduce_token_major(const uint16_t *part, const uint16_t *w, uint16_t *h2,
                            int T, int K, int D) {
    for (int t = 0; t < T; ++t)
        for (int d = 0; d < D; ++d) {
            float acc = 0.0f;
            for (int r = 0; r < K; ++r)
                acc = fmaf(orc_f16_to_float(w[t * K + r]),
                           orc_f16_to_float(part[((size_t)t * K + r) * D + d]), acc);
            h2[(size_t)t * D + d] = orc_f16_bits(acc);
        }
}

/* prefill_moe_int4_gemv_row_dev (prefill.metal:406-440): per group fma chain
 * over byte pairs, sum_x accumulated pairwise, then two fmas. */
static float prefill_row(const uint8_t *W, const uint16_t *S, const uint16_t *B, int st,
                         const float *x, int row, int N) {
    const int groups = N / 64;
    const uint8_t *wr = W + (size_t)row * (N / 2);
    const uint16_t *sr = S + (size_t)row * groups, *br = B + (size_t)row * groups;
    float acc = 0.0f;
    for (int g = 0; g < groups; ++g) {
        float sc = orc_scale_to_float(sr[g], st), bi = orc_scale_to_float(br[g], st);
        const uint8_t *wg = wr + g * 32;
        const float *xg = x + g * 64;
        float dq = 0.0f, sx = 0.0f;
        for (int k = 0; k < 32; ++k) {
            float x0 = xg[2 * k], x1 = xg[2 * k + 1];
            dq = fmaf((float)(wg[k] & 0x0F), x0, dq);
            dq = fmaf((float)(wg[k] >> 4), x1, dq);
            sx += x0 + x1;
        }
        acc = fmaf(sc, dq, acc);
        acc = fmaf(bi, sx, acc);
    }
    return acc;
}

void orc_grouped_routed(const uint8_t *pool, uint64_t stride, const orc_expert_offsets *o,
                        int st, const orc_pair *sorted, int n_pairs, const uint16_t *h16,
                        int hs, uint16_t *part, int D, int F, int K, int nthreads) {
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int p = 0; p < n_pairs; ++p) {
        const orc_pair pr = sorted[p];
        const uint8_t *b = pool + stride * pr.expert;
        float *x = (float *)malloc(sizeof(float) * (size_t)D);
        float *act = (float *)malloc(sizeof(float) * (size_t)F);
        for (int i = 0; i < D; ++i) x[i] = orc_f16_to_float(h16[(size_t)pr.token * hs + i]);
        for (int f = 0; f < F; ++f) {
            float g = prefill_row(b + o->gate_w, BLOB_U16(b, o->gate_s), BLOB_U16(b, o->gate_b), st, x, f, D);
            float u = prefill_row(b + o->up_w, BLOB_U16(b, o->up_s), BLOB_U16(b, o->up_b), st, x, f, D);
            act[f] = hround(orc_gelu_tanh(g) * u);
        }
        for (int d = 0; d < D; ++d) {
            float v = prefill_row(b + o->down_w, BLOB_U16(b, o->down_s), BLOB_U16(b, o->down_b), st, act, d, F);
            part[((size_t)pr.token * K + pr.rank) * D + d] = orc_f16_bits(v);
        }
        free(x);
        free(act);
    }
}

/* ---------------- dense int4 QMM (prefill.metal:672-709) ------------------ */
void orc_int4_qmm(const uint8_t *W, const uint16_t *S, const uint16_t *B, int st,
                  const uint16_t *X16, uint16_t *Y16, float *Y32, int T, int N, int K,
                  int nthreads) {
    const int groups = K / 64;
    float *X = (float *)malloc(sizeof(float) * (size_t)T * K);
    orc_f16_to_f32_array(X16, X, (size_t)T * K);
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for collapse(2) schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int t = 0; t < T; ++t)
        for (int n = 0; n < N; ++n) {
            const uint8_t *wr = W + (size_t)n * (K / 2);
            const float *xr = X + (size_t)t * K;
            float acc = 0.0f;
            for (int g = 0; g < groups; ++g) {
                float sc = orc_scale_to_float(S[(size_t)n * groups + g], st);
                float bi = orc_scale_to_float(B[(size_t)n * groups + g], st);
                for (int kk = 0; kk < 64; ++kk) {
                    int k = g * 64 + kk;
                    uint8_t pk = wr[k >> 1];
                    int q = (k & 1) == 0 ? (pk & 0x0F) : (pk >> 4);
                    acc = fmaf(fmaf((float)q, sc, bi), xr[k], acc);
                }
            }
            if (Y32) Y32[(size_t)t * N + n] = acc;
            if (Y16) Y16[(size_t)t * N + n] = orc_f16_bits(acc);
        }
    free(X);
}

/* ---------------- 2/3-bit routed decode (moe.metal:644-1180) --------------- */
/* Kernel-order row of moe_int2_gemv_row_simd_dev_vec / moe_int3_gemv_row_simd_dev_vec
 * (moe.metal:644-757; the same lane scheme as dequant_int4_gemv_simd_body_b3,
 * dequant_int4.metal:512-583): 32 lanes; full blocks of 4 groups where lane l
 * owns the 8 codes at blk*256 + 8l (2-bit: the u16 at blk*64 + 2l; 3-bit: the
 * 3 bytes at blk*96 + 3l), an fma chain for the dot, a left-to-right sum of
 * the 8 activations, acc = fma(s, dot, acc); acc = fma(b, sum, acc); the
 * groups past the last full block with 2 codes per lane; butterfly lane sum. */
static float lowbit_row_lanes(const uint8_t *wr, const uint16_t *sr, const uint16_t *br, int st, int bits,
                              const float *x, int n) {
    const int ng = n / 64, full = ng / 4;
    float acc[32];
    for (int lane = 0; lane < 32; ++lane) {
        float a = 0.0f;
        for (int blk = 0; blk < full; ++blk) {
            const int g = blk * 4 + (lane >> 3);
            const float s = orc_scale_to_float(sr[g], st), b = orc_scale_to_float(br[g], st);
            uint32_t v;
            if (bits == 2) {
                const int bb = blk * 64 + lane * 2;
                v = (uint32_t)wr[bb] | ((uint32_t)wr[bb + 1] << 8);
            } else {
                const int bb = blk * 96 + lane * 3;
                v = (uint32_t)wr[bb] | ((uint32_t)wr[bb + 1] << 8) | ((uint32_t)wr[bb + 2] << 16);
            }
            const uint32_t mask = (1u << bits) - 1u;
            const float *e = x + blk * 256 + lane * 8;
            float dot = 0.0f;
            for (int i = 0; i < 8; ++i) dot = fmaf((float)((v >> (bits * i)) & mask), e[i], dot);
            const float sum = e[0] + e[1] + e[2] + e[3] + e[4] + e[5] + e[6] + e[7];
            a = fmaf(s, dot, a);
            a = fmaf(b, sum, a);
        }
        for (int g = full * 4; g < ng; ++g) {
            const float s = orc_scale_to_float(sr[g], st), b = orc_scale_to_float(br[g], st);
            const int c0 = g * 64 + lane * 2;
            uint32_t q0, q1;
            if (bits == 2) {
                const uint8_t byte = wr[g * 16 + lane / 2];
                const int sh = 4 * (lane & 1);
                q0 = (byte >> sh) & 3u;
                q1 = (byte >> (sh + 2)) & 3u;
            } else {
                const int bbit = c0 * 3, b0 = bbit / 8, bsh = bbit % 8;
                const uint32_t v = (uint32_t)wr[b0] | ((uint32_t)wr[b0 + 1] << 8);
                q0 = (v >> bsh) & 7u;
                q1 = (v >> (bsh + 3)) & 7u;
            }
            const float x0 = x[c0], x1 = x[c0 + 1];
            float dot = fmaf((float)q0, x0, 0.0f);
            dot = fmaf((float)q1, x1, dot);
            a = fmaf(s, dot, a);
            a = fmaf(b, x0 + x1, a);
        }
        acc[lane] = a;
    }
    for (int off = 16; off >= 1; off >>= 1)
        for (int l = 0; l < 32; ++l)
            if ((l & off) == 0) acc[l] += acc[l | off];
    return acc[0];
}

void orc_lowbit_gemv_kernel_order(const uint8_t *W, const uint16_t *S, const uint16_t *B, int st, int bits,
                                  const uint16_t *x16, float *y32, uint16_t *y16, int m, int n, int nthreads) {
    float *x = (float *)malloc(sizeof(float) * (size_t)n);
    orc_f16_to_f32_array(x16, x, (size_t)n);
    const size_t rb = orc_packed_row_bytes(n, bits);
    const int ng = n / 64;
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int r = 0; r < m; ++r) {
        const float v = lowbit_row_lanes(W + rb * (size_t)r, S + (size_t)r * ng, B + (size_t)r * ng, st, bits, x, n);
        if (y32) y32[r] = v;
        if (y16) y16[r] = orc_f16_bits(v);
    }
    free(x);
}

/* moe_phase1_gate_up_act_b2/_b3 (moe.metal:950-1064): per (slot, f) the gate
 * and up rows in kernel order, acts = half(gelu_tanh(g) * u). */
void orc_moe_phase1_bits(const uint8_t *const *blobs, const orc_expert_offsets *o, int st, int bits,
                         const uint16_t *x16, uint16_t *acts, int D, int F, int top_k, int nthreads) {
    float *x = (float *)malloc(sizeof(float) * (size_t)D);
    orc_f16_to_f32_array(x16, x, (size_t)D);
    const int ng = D / 64;
    const size_t rb = orc_packed_row_bytes(D, bits);
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int rowg = 0; rowg < top_k * F; ++rowg) {
        const int slot = rowg / F, f = rowg % F;
        const uint8_t *b = blobs[slot];
        const float g = lowbit_row_lanes(b + o->gate_w + (size_t)f * rb, BLOB_U16(b, o->gate_s) + (size_t)f * ng,
                                         BLOB_U16(b, o->gate_b) + (size_t)f * ng, st, bits, x, D);
        const float u = lowbit_row_lanes(b + o->up_w + (size_t)f * rb, BLOB_U16(b, o->up_s) + (size_t)f * ng,
                                         BLOB_U16(b, o->up_b) + (size_t)f * ng, st, bits, x, D);
        acts[(size_t)slot * F + f] = orc_f16_bits(orc_gelu_tanh(g) * u);
    }
    free(x);
}

/* moe_phase2_down_reduce_b2/_b3 (moe.metal:1108-1180): partial[slot] =
 * float(w_slot) * down_slot[d].acts_slot (kernel-order row);
 * y[d] = half(residual[d] + partial[0] + partial[1] + ...). */
void orc_moe_phase2_bits(const uint8_t *const *blobs, const orc_expert_offsets *o, int st, int bits,
                         const uint16_t *acts16, const uint16_t *w16, const uint16_t *res16, uint16_t *y16,
                         float *y32, int D, int F, int top_k, int nthreads) {
    float *acts = (float *)malloc(sizeof(float) * (size_t)top_k * F);
    orc_f16_to_f32_array(acts16, acts, (size_t)top_k * F);
    const int ng = F / 64;
    const size_t rb = orc_packed_row_bytes(F, bits);
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int d = 0; d < D; ++d) {
        float acc = res16 ? orc_f16_to_float(res16[d]) : 0.0f;
        for (int s = 0; s < top_k; ++s) {
            const uint8_t *b = blobs[s];
            const float v = lowbit_row_lanes(b + o->down_w + (size_t)d * rb, BLOB_U16(b, o->down_s) + (size_t)d * ng,
                                             BLOB_U16(b, o->down_b) + (size_t)d * ng, st, bits,
                                             acts + (size_t)s * F, F);
            acc += orc_f16_to_float(w16[s]) * v;
        }
        if (y32) y32[d] = acc;
        if (y16) y16[d] = orc_f16_bits(acc);
    }
    free(acts);
}
