/*
 * oracle_decoder.c -- CPU restatement of the dense decode stack around the
 * MoE path: RMSNorms, the per-head Q/K/V epilogue with NeoX RoPE, split-KV
 * decode attention, the post-attention setup, the decoder-layer tail, the
 * int4 embedding lookup and the int4 LM head with greedy selection.
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  fp16 values travel as uint16_t
 * bits, weights of the norms are BF16 bits.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

static inline float h2f(uint16_t h) { return orc_f16_to_float(h); }
static inline uint16_t f2h(float v) { return orc_f16_bits(v); }

/* rms_block_inv (Sources/TurboFieldfare/Metal/Primitives/rmsnorm.metal:32-63):
 * inv = rsqrt(mean(x^2) + eps), fp32 sum of squares (sequential here). */
static float rms_inv(const float *x, int n, float eps) {
    float acc = 0.0f;
    for (int i = 0; i < n; ++i) acc = fmaf(x[i], x[i], acc);
    return 1.0f / sqrtf(acc / (float)n + eps);
}

/* rmsnorm_bf16w / rmsnorm_no_scale (rmsnorm.metal:70-98,128-150):
 * out = half(x * inv * w) (w = 1 when weight is NULL), per row. */
void orc_rmsnorm(const uint16_t *x, const uint16_t *w_bf16, uint16_t *out, int rows, int d, float eps) {
    float *xf = (float *)malloc(sizeof(float) * (size_t)d);
    for (int r = 0; r < rows; ++r) {
        for (int i = 0; i < d; ++i) xf[i] = h2f(x[(size_t)r * d + i]);
        const float inv = rms_inv(xf, d, eps);
        for (int i = 0; i < d; ++i) {
            float v = xf[i] * inv;
            if (w_bf16) v *= orc_bf16_to_float(w_bf16[i]);
            out[(size_t)r * d + i] = f2h(v);
        }
    }
    free(xf);
}

/* fused_rope_neox_pair (Sources/TurboFieldfare/Metal/Fusions/fused.metal:53-69). */
static void rope_pair(float *x0, float *x1, int pair, int hd, float pos, float theta) {
    const double exponent = -(double)(2 * pair) / (double)hd;
    const double freq = pow((double)theta, exponent);
    const double angle = (double)pos * freq;
    const float c = (float)cos(angle), s = (float)sin(angle);
    const float r0 = *x0 * c - *x1 * s;
    const float r1 = *x0 * s + *x1 * c;
    *x0 = r0;
    *x1 = r1;
}

/* fused_qkv_epilogue (fused.metal:84-170): per head, RMSNorm over head_dim
 * (Q, K: times the shared BF16 weight; V: no scale), rounded to half, then
 * NeoX RoPE on the first `rotated_pairs` pairs of Q and K.  In place. */
void orc_qkv_epilogue(uint16_t *q, uint16_t *k, uint16_t *v, const uint16_t *qw, const uint16_t *kw, int hd,
                      int nq, int nkv, int position, float theta, int rotated_pairs, float eps) {
    float *xf = (float *)malloc(sizeof(float) * (size_t)hd);
    float *nh = (float *)malloc(sizeof(float) * (size_t)hd);
    for (int head = 0; head < nq + 2 * nkv; ++head) {
        const int is_q = head < nq, is_k = !is_q && head < nq + nkv;
        uint16_t *dst = is_q ? q + (size_t)head * hd
                             : (is_k ? k + (size_t)(head - nq) * hd : v + (size_t)(head - nq - nkv) * hd);
        const uint16_t *w = is_q ? qw : kw;
        for (int i = 0; i < hd; ++i) xf[i] = h2f(dst[i]);
        const float inv = rms_inv(xf, hd, eps);
        for (int i = 0; i < hd; ++i) {
            float xv = xf[i] * inv;
            if (is_q || is_k) xv *= orc_bf16_to_float(w[i]);
            nh[i] = h2f(f2h(xv));
        }
        if (!is_q && !is_k) {
            for (int i = 0; i < hd; ++i) dst[i] = f2h(nh[i]);
            continue;
        }
        for (int pair = 0; pair < hd / 2; ++pair) {
            float x0 = nh[pair], x1 = nh[hd / 2 + pair];
            if (pair < rotated_pairs) rope_pair(&x0, &x1, pair, hd, (float)position, theta);
            dst[pair] = f2h(x0);
            dst[hd / 2 + pair] = f2h(x1);
        }
    }
    free(xf);
    free(nh);
}

/* attention_decode_single (Sources/TurboFieldfare/Metal/Attention/attention.metal:241-312):
 * per Q head, scores s_p = scale * (q . k_p) over p in [kv_start, seq_len),
 * softmax, out = half(sum_p softmax_p * v_p).  K/V are [seq][nkv][hd];
 * GQA: kv_head = q_head / (nq / nkv).  Two passes in double for the
 * reference value (the kernels use the online recurrence in fp32). */
void orc_attention_decode(const uint16_t *q, const uint16_t *K, const uint16_t *V, uint16_t *out, float *out32,
                          int hd, int nq, int nkv, int seq_len, int kv_start, float scale) {
    double *s = (double *)malloc(sizeof(double) * (size_t)(seq_len > 0 ? seq_len : 1));
    double *o = (double *)malloc(sizeof(double) * (size_t)hd);
    for (int h = 0; h < nq; ++h) {
        const int kvh = h / (nq / nkv);
        double m = -INFINITY;
        for (int p = kv_start; p < seq_len; ++p) {
            const uint16_t *kr = K + ((size_t)p * nkv + kvh) * hd;
            double acc = 0.0;
            for (int i = 0; i < hd; ++i) acc += (double)h2f(q[(size_t)h * hd + i]) * (double)h2f(kr[i]);
            s[p] = acc * scale;
            if (s[p] > m) m = s[p];
        }
        double dsum = 0.0;
        for (int i = 0; i < hd; ++i) o[i] = 0.0;
        for (int p = kv_start; p < seq_len; ++p) {
            const double e = exp(s[p] - m);
            dsum += e;
            const uint16_t *vr = V + ((size_t)p * nkv + kvh) * hd;
            for (int i = 0; i < hd; ++i) o[i] += e * (double)h2f(vr[i]);
        }
        for (int i = 0; i < hd; ++i) {
            const float val = dsum > 0.0 ? (float)(o[i] / dsum) : 0.0f;
            if (out) out[(size_t)h * hd + i] = f2h(val);
            if (out32) out32[(size_t)h * hd + i] = val;
        }
    }
    free(s);
    free(o);
}

/* fused_post_attn_setup (fused.metal:190-269), per row:
 *   hidden = half(hidden + half(attn * inv_a * w_post_attn))
 *   dense_x = half(hidden * inv_h * w_pre_ffn), routed_x = half(hidden * inv_h * w_pre_ffn2),
 *   router_x = half(hidden * inv_h). */
void orc_post_attn_setup(uint16_t *hidden, const uint16_t *attn, uint16_t *dense_x, uint16_t *routed_x,
                         uint16_t *router_x, const uint16_t *w_post_attn, const uint16_t *w_pre_ffn,
                         const uint16_t *w_pre_ffn2, int rows, int d, float eps) {
    float *a = (float *)malloc(sizeof(float) * (size_t)d);
    float *hh = (float *)malloc(sizeof(float) * (size_t)d);
    for (int r = 0; r < rows; ++r) {
        uint16_t *hr = hidden + (size_t)r * d;
        for (int i = 0; i < d; ++i) a[i] = h2f(attn[(size_t)r * d + i]);
        const float inv_a = rms_inv(a, d, eps);
        for (int i = 0; i < d; ++i) {
            const float an = h2f(f2h(a[i] * inv_a * orc_bf16_to_float(w_post_attn[i])));
            const uint16_t hb = f2h(h2f(hr[i]) + an);
            hr[i] = hb;
            hh[i] = h2f(hb);
        }
        const float inv_h = rms_inv(hh, d, eps);
        for (int i = 0; i < d; ++i) {
            const float h = hh[i] * inv_h;
            dense_x[(size_t)r * d + i] = f2h(h * orc_bf16_to_float(w_pre_ffn[i]));
            routed_x[(size_t)r * d + i] = f2h(h * orc_bf16_to_float(w_pre_ffn2[i]));
            router_x[(size_t)r * d + i] = f2h(h);
        }
    }
    free(a);
    free(hh);
}

/* The decoder-layer tail (fused_layer_tail, fused.metal:271-375), with the
 * shared expert's post-FFN norm applied first when w_postffn1 is given
 * (rmsnorm_bf16w(h1, post_feedforward_layernorm_1),
 * Sources/TurboFieldfare/Runtime/Inference/RealForwardRunner.swift:191), per row:
 *   h1n = half(h1 * inv1 * w_postffn1)                       (optional)
 *   h12 = half(h1n + half(h2 * inv2 * w_postffn2))
 *   hidden = half(hidden + half(h12 * inv12 * w_postffn)); hidden = half(hidden * half(layer_scalar)). */
void orc_layer_tail(const uint16_t *h2, const uint16_t *h1, uint16_t *hidden, const uint16_t *w_postffn1,
                    const uint16_t *w_postffn2, const uint16_t *w_postffn, float layer_scalar, int rows, int d,
                    float eps) {
    float *a = (float *)malloc(sizeof(float) * (size_t)d);
    float *b = (float *)malloc(sizeof(float) * (size_t)d);
    const float hs = h2f(f2h(layer_scalar));
    for (int r = 0; r < rows; ++r) {
        for (int i = 0; i < d; ++i) b[i] = h2f(h1[(size_t)r * d + i]);
        if (w_postffn1) {
            const float inv1 = rms_inv(b, d, eps);
            for (int i = 0; i < d; ++i) b[i] = h2f(f2h(b[i] * inv1 * orc_bf16_to_float(w_postffn1[i])));
        }
        for (int i = 0; i < d; ++i) a[i] = h2f(h2[(size_t)r * d + i]);
        const float inv2 = rms_inv(a, d, eps);
        for (int i = 0; i < d; ++i) {
            const float t = h2f(f2h(a[i] * inv2 * orc_bf16_to_float(w_postffn2[i])));
            a[i] = h2f(f2h(b[i] + t));
        }
        const float inv12 = rms_inv(a, d, eps);
        uint16_t *hr = hidden + (size_t)r * d;
        for (int i = 0; i < d; ++i) {
            const float t = h2f(f2h(a[i] * inv12 * orc_bf16_to_float(w_postffn[i])));
            const float hn = h2f(f2h(h2f(hr[i]) + t));
            hr[i] = f2h(hn * hs);
        }
    }
    free(a);
    free(b);
}

/* embed_lookup_int4 (Sources/TurboFieldfare/Metal/Quant/dequant_int4.metal:65-84):
 * out[t][i] = half((q * s + b) * out_scale) for row token_ids[t]. */
void orc_embed_int4(const uint8_t *table, const uint16_t *S, const uint16_t *B, int st, const uint32_t *tokens,
                    int T, int d, float out_scale, uint16_t *out) {
    const int ng = d / 64;
    for (int t = 0; t < T; ++t) {
        const uint32_t tok = tokens[t];
        const uint8_t *rq = table + (size_t)tok * (d / 2);
        for (int i = 0; i < d; ++i) {
            const uint8_t byte = rq[i >> 1];
            const int q = (i & 1) ? (byte >> 4) : (byte & 0xF);
            const float s = orc_scale_to_float(S[(size_t)tok * ng + i / 64], st);
            const float b = orc_scale_to_float(B[(size_t)tok * ng + i / 64], st);
            out[(size_t)t * d + i] = f2h(((float)q * s + b) * out_scale);
        }
    }
}

/* lm_head_greedy_int4_rows_chunk_raw + _reduce
 * (Sources/TurboFieldfare/Metal/Sampling/logit.metal:687-787): fp32 logit per
 * vocabulary row (factored sums, fp32), the largest finite logit wins, ties
 * to the lower row; token 0 when no row is finite.  logits (optional)
 * receives every row's fp32 value. */
uint32_t orc_lm_head_greedy(const uint8_t *W, const uint16_t *S, const uint16_t *B, int st, const uint16_t *x_f16,
                            int vocab, int d, float *logits, int nthreads) {
    float *y = logits ? logits : (float *)malloc(sizeof(float) * (size_t)vocab);
    orc_int4_gemv_kernel_order(W, S, B, st, x_f16, y, NULL, vocab, d, nthreads);
    float best = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (int r = 0; r < vocab; ++r)
        if (isfinite(y[r]) && (y[r] > best || (y[r] == best && (uint32_t)r < bi))) {
            best = y[r];
            bi = (uint32_t)r;
        }
    if (!logits) free(y);
    return bi == 0xFFFFFFFFu ? 0u : bi;
}

/* ---- sampling (Sources/TurboFieldfare/Metal/Sampling/logit.metal:42-617) ---- */

/* logit_softcap_softmax (logit.metal:52-146): z' = softcap * tanh(z / softcap),
 * p = half(exp(z' - max z') / sum exp(z' - max z')).  Two passes in double for
 * the reference value. */
void orc_softcap_softmax(const float *logits, uint16_t *probs, int V, float softcap) {
    double m = -INFINITY;
    double *z = (double *)malloc(sizeof(double) * (size_t)V);
    for (int i = 0; i < V; ++i) {
        z[i] = (double)softcap * tanh((double)logits[i] / (double)softcap);
        if (z[i] > m) m = z[i];
    }
    double d = 0.0;
    for (int i = 0; i < V; ++i) d += exp(z[i] - m);
    for (int i = 0; i < V; ++i) probs[i] = f2h((float)(exp(z[i] - m) / d));
    free(z);
}

/* xorshift64* and uniform01 (logit.metal:148-160). */
static uint64_t xorshift64(uint64_t *s) {
    *s ^= *s << 13;
    *s ^= *s >> 7;
    *s ^= *s << 17;
    return *s * 2685821657736338717ULL;
}
static float uniform01(uint64_t *s) {
    const uint32_t bits = (uint32_t)(xorshift64(s) >> 40);
    return (float)bits * (1.0f / 16777216.0f);
}
/* lmhead_splitmix64 / lmhead_gumbel_for (logit.metal:164-181). */
static uint64_t splitmix64_mix(uint64_t x) {
    x = x + 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
float orc_gumbel(uint64_t seed, uint32_t position, uint32_t row) {
    const uint64_t key = seed ^ ((uint64_t)position * 0xD2B74407B1CE6E93ull) ^ (uint64_t)row;
    const uint32_t bits = (uint32_t)(splitmix64_mix(key) >> 40);
    const float u = ((float)bits + 0.5f) * (1.0f / 16777216.0f);
    return -logf(-logf(u));
}

/* The truncating tail shared by `sample` (logit.metal:391-443) and
 * sample_topk64_final (:575-616): the candidates sorted by (p desc, index
 * asc); keep the finite ones, top-p against the full-vocabulary mass,
 * temperature p^(1/T), one xorshift step, then the inverse-CDF draw. */
static uint32_t truncated_draw(float *val, const uint32_t *idx, int count, int V, float temperature, float top_p,
                               uint64_t seed) {
    int kept = 0;
    while (kept < count && idx[kept] < (uint32_t)V && isfinite(val[kept])) kept++;
    if (top_p > 0.0f && top_p < 1.0f) {
        float cum = 0.0f;
        int cut = kept;
        for (int i = 0; i < kept; ++i) {
            cum += val[i];
            if (cum >= top_p) {
                cut = i + 1;
                break;
            }
        }
        kept = cut;
    }
    const float inv_t = 1.0f / temperature;
    for (int i = 0; i < kept; ++i)
        if (temperature != 1.0f) val[i] = powf(val[i], inv_t);
    float surviving = 0.0f;
    for (int i = 0; i < kept; ++i) surviving += val[i];
    uint64_t rng = seed;
    (void)xorshift64(&rng);
    const float u = uniform01(&rng) * surviving;
    float run = 0.0f;
    uint32_t picked = idx[0];
    for (int i = 0; i < kept; ++i) {
        run += val[i];
        if (u <= run) {
            picked = idx[i];
            break;
        }
    }
    return picked;
}

static int cand_cmp(const void *a, const void *b) {
    const float va = ((const float *)a)[0], vb = ((const float *)b)[0];
    const uint32_t ia = ((const uint32_t *)a)[1], ib = ((const uint32_t *)b)[1];
    if (va > vb) return -1;
    if (va < vb) return 1;
    return ia < ib ? -1 : (ia > ib);
}

/* sample (logit.metal:183-446): temperature <= 0 greedy argmax (ties to the
 * lower index); top_k == 0 and no top-p: Gumbel-max over inv_t * log p;
 * otherwise the top min(top_k or V, 256) candidates and truncated_draw. */
uint32_t orc_sample(const uint16_t *probs, int V, float temperature, uint32_t top_k, float top_p, uint64_t seed,
                    uint32_t position) {
    if (temperature <= 0.0f) {
        float best = -INFINITY;
        uint32_t bi = 0;
        for (int i = 0; i < V; ++i) {
            const float p = h2f(probs[i]);
            if (p > best) {
                best = p;
                bi = (uint32_t)i;
            }
        }
        return bi;
    }
    if (top_k == 0 && (top_p <= 0.0f || top_p >= 1.0f)) {
        const float inv_t = 1.0f / temperature;
        float best = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (int i = 0; i < V; ++i) {
            const float p = h2f(probs[i]);
            if (!(p > 0.0f)) continue;
            const float s = inv_t * logf(p) + orc_gumbel(seed, position, (uint32_t)i);
            if (s > best) {
                best = s;
                bi = (uint32_t)i;
            }
        }
        return bi == 0xFFFFFFFFu ? 0u : bi;
    }
    int k = top_k == 0 ? V : (int)top_k;
    if (k > 256) k = 256;
    if (k > V) k = V;
    float *c = (float *)malloc(sizeof(float) * 2 * (size_t)V);
    for (int i = 0; i < V; ++i) {
        c[2 * i] = h2f(probs[i]);
        ((uint32_t *)c)[2 * i + 1] = (uint32_t)i;
    }
    qsort(c, (size_t)V, 2 * sizeof(float), cand_cmp);
    float val[256];
    uint32_t idx[256];
    for (int i = 0; i < k; ++i) {
        val[i] = c[2 * i];
        idx[i] = ((uint32_t *)c)[2 * i + 1];
    }
    free(c);
    return truncated_draw(val, idx, k, V, temperature, top_p, seed);
}

/* SampleTopK64 (sample_topk64_stage1/_reduce/_final, logit.metal:489-617):
 * the top 64 by (p desc, index asc), then truncated_draw. */
uint32_t orc_sample_topk64(const uint16_t *probs, int V, float temperature, float top_p, uint64_t seed) {
    float *c = (float *)malloc(sizeof(float) * 2 * (size_t)V);
    for (int i = 0; i < V; ++i) {
        c[2 * i] = h2f(probs[i]);
        ((uint32_t *)c)[2 * i + 1] = (uint32_t)i;
    }
    qsort(c, (size_t)V, 2 * sizeof(float), cand_cmp);
    const int k = V < 64 ? V : 64;
    float val[64];
    uint32_t idx[64];
    for (int i = 0; i < k; ++i) {
        val[i] = c[2 * i];
        idx[i] = ((uint32_t *)c)[2 * i + 1];
    }
    free(c);
    return truncated_draw(val, idx, k, V, temperature, top_p, seed);
}
