/*
 * oracle_core.c -- PRNG, number formats, affine quantization, GEMV references.
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Built with -ffp-contract=off so
 * every fused multiply-add below is an explicit fmaf() where the reference
 * kernel writes fma(), and nothing else is contracted.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int orc_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---------------- PRNG (SplitMix64.swift:11-23, SeedTree.swift:12-19) ---- */
uint64_t orc_sm64_next(uint64_t *state) {
    *state += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *state;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

float orc_sm64_uniform(uint64_t *state, float lo, float hi) {
    /* Float(next() >> 40) / Float(1 << 24); lo + (hi - lo) * u */
    float u = (float)(orc_sm64_next(state) >> 40) / (float)(1 << 24);
    return lo + (hi - lo) * u;
}

double orc_sm64_normal(uint64_t *state) {
    /* Box-Muller (G. E. P. Box and M. E. Muller, 1958), cosine branch only.
     * u1 in (0,1] from 53 random bits so log() is finite. */
    double u1 = ((double)(orc_sm64_next(state) >> 11) + 1.0) * (1.0 / 9007199254740992.0);
    double u2 = (double)(orc_sm64_next(state) >> 11) * (1.0 / 9007199254740992.0);
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586476925 * u2);
}

uint64_t orc_seedtree_seed(uint64_t root, const char *label) {
    uint64_t h = 0xCBF29CE484222325ULL;          /* FNV-1a 64 */
    for (const unsigned char *p = (const unsigned char *)label; *p; ++p) {
        h ^= (uint64_t)*p;
        h *= 0x100000001B3ULL;
    }
    return root ^ h;
}

void orc_fill_uniform(uint64_t *state, float lo, float hi, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_sm64_uniform(state, lo, hi);
}

/* ---------------- number formats (Quantization.swift:16-28) -------------- */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t orc_bf16_bits(float x) {
    uint32_t bits = f2u(x);
    uint32_t lsb = (bits >> 16) & 1u;
    uint32_t rounded = (bits + 0x7FFFu + lsb) >> 16;   /* wrapping add, as &+ */
    return (uint16_t)rounded;
}

float orc_bf16_to_float(uint16_t b) { return u2f((uint32_t)b << 16); }

uint16_t orc_f16_bits(float x) {
    /* IEEE-754 binary32 -> binary16, round to nearest even, with subnormals,
     * overflow to inf and NaN propagation. */
    uint32_t u = f2u(x);
    uint32_t sign = (u >> 16) & 0x8000u;
    uint32_t exp = (u >> 23) & 0xFFu;
    uint32_t man = u & 0x7FFFFFu;
    if (exp == 0xFFu) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;                     /* 1 - e + 13 */
        uint32_t half = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1u);
        uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = ((uint32_t)e << 10) | (man >> 13);
    uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;   /* may carry into exp: correct */
    return (uint16_t)(sign | half);
}

float orc_f16_to_float(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    if (exp == 0) {
        if (man == 0) return u2f(sign);
        float v = (float)man * (1.0f / 16777216.0f);   /* man * 2^-24 */
        return sign ? -v : v;
    }
    if (exp == 31) return u2f(sign | 0x7F800000u | (man << 13));
    return u2f(sign | ((exp - 15 + 127) << 23) | (man << 13));
}

float orc_scale_to_float(uint16_t bits, int scale_type) {
    return scale_type == 1 ? orc_f16_to_float(bits) : orc_bf16_to_float(bits);
}

void orc_f32_to_f16_array(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f16_bits(in[i]);
}
void orc_f16_to_f32_array(const uint16_t *in, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f16_to_float(in[i]);
}

static inline float hround(float v) { return orc_f16_to_float(orc_f16_bits(v)); }

/* ---------------- affine quantization (Quantization.swift:228-349) ------- */
size_t orc_packed_row_bytes(int n, int bits) {
    if (bits == 8) return (size_t)n;
    return ((size_t)n * (size_t)bits + 7u) / 8u;
}

int orc_unpack_code(const uint8_t *buf, size_t len, int index, int bits) {
    switch (bits) {
    case 8: return buf[index];
    case 4: { uint8_t b = buf[index / 2]; return (index & 1) == 0 ? (b & 0x0F) : (b >> 4); }
    case 2: return (buf[index / 4] >> ((index % 4) * 2)) & 0x03;
    case 3: {
        size_t bit = (size_t)index * 3u, bi = bit / 8u;
        unsigned sh = (unsigned)(bit % 8u);
        uint32_t b0 = buf[bi];
        uint32_t b1 = bi + 1 < len ? buf[bi + 1] : 0u;
        uint32_t b2 = bi + 2 < len ? buf[bi + 2] : 0u;
        return (int)(((b0 | (b1 << 8) | (b2 << 16)) >> sh) & 0x07u);
    }
    default: return -1;
    }
}

void orc_pack_code(uint8_t *buf, size_t len, int code, int index, int bits) {
    switch (bits) {
    case 8: buf[index] = (uint8_t)code; break;
    case 4: {
        size_t bi = (size_t)index / 2u;
        uint8_t nib = (uint8_t)code & 0x0F;
        if ((index & 1) == 0) buf[bi] = (uint8_t)((buf[bi] & 0xF0) | nib);
        else buf[bi] = (uint8_t)((buf[bi] & 0x0F) | (nib << 4));
        break;
    }
    case 2: {
        size_t bi = (size_t)index / 4u;
        unsigned sh = (unsigned)((index % 4) * 2);
        buf[bi] = (uint8_t)((buf[bi] & ~(0x03u << sh)) | ((unsigned)(code & 0x03) << sh));
        break;
    }
    case 3: {
        size_t bit = (size_t)index * 3u, bi = bit / 8u;
        unsigned sh = (unsigned)(bit % 8u);
        uint16_t v = (uint16_t)((code & 0x07) << sh);
        buf[bi] |= (uint8_t)(v & 0xFF);
        if (bi + 1 < len) buf[bi + 1] |= (uint8_t)(v >> 8);
        break;
    }
    default: break;
    }
}

int orc_quantize_affine(const float *w, int rows, int n, int bits,
                        uint8_t *packed, uint16_t *scales, uint16_t *biases) {
    if (n % 64 != 0) return -1;
    if (!(bits == 2 || bits == 3 || bits == 4 || bits == 8)) return -2;
    const int qmax = (1 << bits) - 1;
    const int ng = n / 64;
    const size_t rb = orc_packed_row_bytes(n, bits);
    memset(packed, 0, rb * (size_t)rows);
    for (int r = 0; r < rows; ++r) {
        const float *row = w + (size_t)r * n;
        uint8_t *pr = packed + rb * (size_t)r;
        for (int g = 0; g < ng; ++g) {
            float wmin = INFINITY, wmax = -INFINITY;
            for (int k = 0; k < 64; ++k) {
                float v = row[g * 64 + k];
                if (v < wmin) wmin = v;
                if (v > wmax) wmax = v;
            }
            float sF, bF;
            if (wmax == wmin) { sF = 1.0f; bF = wmin; }
            else { sF = (wmax - wmin) / (float)qmax; bF = wmin; }
            uint16_t sb = orc_bf16_bits(sF), bb = orc_bf16_bits(bF);
            scales[(size_t)r * ng + g] = sb;
            biases[(size_t)r * ng + g] = bb;
            float s = orc_bf16_to_float(sb), b = orc_bf16_to_float(bb);
            float inv = s == 0.0f ? 0.0f : 1.0f / s;
            for (int k = 0; k < 64; ++k) {
                float v = row[g * 64 + k];
                long q = lroundf((v - b) * inv);     /* Swift .rounded(): half away from zero */
                if (q < 0) q = 0;
                if (q > qmax) q = qmax;
                orc_pack_code(pr, rb, (int)q, g * 64 + k, bits);
            }
        }
    }
    return 0;
}

void orc_dequantize_affine(const uint8_t *packed, const uint16_t *scales,
                           const uint16_t *biases, int st, int rows, int n,
                           int bits, float *out) {
    const int ng = n / 64;
    const size_t rb = orc_packed_row_bytes(n, bits);
    for (int r = 0; r < rows; ++r) {
        const uint8_t *pr = packed + rb * (size_t)r;
        for (int g = 0; g < ng; ++g) {
            float s = orc_scale_to_float(scales[(size_t)r * ng + g], st);
            float b = orc_scale_to_float(biases[(size_t)r * ng + g], st);
            for (int k = 0; k < 64; ++k) {
                int q = orc_unpack_code(pr, rb, g * 64 + k, bits);
                out[(size_t)r * n + g * 64 + k] = (float)q * s + b;
            }
        }
    }
}

/* ---------------- GEMV references --------------------------------------- */
void orc_affine_gemv_ref(const uint8_t *W, const uint16_t *S, const uint16_t *B,
                         int st, int bits, const float *x, float *y, int m, int n,
                         int nthreads) {
    const size_t rb = orc_packed_row_bytes(n, bits);
    const int ng = n / 64;
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int r = 0; r < m; ++r) {
        /* dequantizeAffine(row) then a sequential fp32 dot (vDSP_dotpr). */
        const uint8_t *pr = W + rb * (size_t)r;
        float dot = 0.0f;
        for (int g = 0; g < ng; ++g) {
            float s = orc_scale_to_float(S[(size_t)r * ng + g], st);
            float b = orc_scale_to_float(B[(size_t)r * ng + g], st);
            for (int k = 0; k < 64; ++k) {
                int q = orc_unpack_code(pr, rb, g * 64 + k, bits);
                float wv = (float)q * s + b;
                dot += wv * x[g * 64 + k];
            }
        }
        y[r] = dot;
    }
}

/* Butterfly sum of 32 lane partials (simd_sum order is not specified by
 * Metal; a xor-butterfly is the usual hardware tree). */
static float lane_sum32(float *v) {
    for (int off = 16; off >= 1; off >>= 1)
        for (int l = 0; l < 32; ++l)
            if ((l & off) == 0) v[l] = v[l] + v[l | off];
    return v[0];
}

void orc_int4_gemv_kernel_order(const uint8_t *W, const uint16_t *S, const uint16_t *B,
                                int st, const uint16_t *x16, float *y32, uint16_t *y16,
                                int m, int n, int nthreads) {
    const int ng = n / 64, rb = n / 2, full = ng / 4;
    (void)nthreads;
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int r = 0; r < m; ++r) {
        const uint8_t *wr = W + (size_t)r * rb;
        const uint16_t *sr = S + (size_t)r * ng, *br = B + (size_t)r * ng;
        float acc[32];
        for (int lane = 0; lane < 32; ++lane) {
            float a = 0.0f;
            for (int blk = 0; blk < full; ++blk) {
                int bb = blk * 128 + lane * 4;
                int g = blk * 4 + (lane >> 3);
                float s = orc_scale_to_float(sr[g], st), b = orc_scale_to_float(br[g], st);
                int elem = bb * 2;
                float e[8], sum = 0.0f, dot = 0.0f;
                for (int i = 0; i < 8; ++i) e[i] = orc_f16_to_float(x16[elem + i]);
                for (int i = 0; i < 4; ++i) {
                    uint8_t byte = wr[bb + i];
                    dot = fmaf((float)(byte & 0x0F), e[2 * i], dot);
                    dot = fmaf((float)(byte >> 4), e[2 * i + 1], dot);
                }
                sum = e[0] + e[1] + e[2] + e[3] + e[4] + e[5] + e[6] + e[7];
                a = fmaf(s, dot, a);
                a = fmaf(b, sum, a);
            }
            for (int g = full * 4; g < ng; ++g) {
                float s = orc_scale_to_float(sr[g], st), b = orc_scale_to_float(br[g], st);
                uint8_t byte = wr[g * 32 + lane];
                float x0 = orc_f16_to_float(x16[g * 64 + lane * 2]);
                float x1 = orc_f16_to_float(x16[g * 64 + lane * 2 + 1]);
                float dot = fmaf((float)(byte & 0x0F), x0, 0.0f);
                dot = fmaf((float)(byte >> 4), x1, dot);
                a = fmaf(s, dot, a);
                a = fmaf(b, x0 + x1, a);
            }
            acc[lane] = a;
        }
        float v = lane_sum32(acc);
        if (y32) y32[r] = v;
        if (y16) y16[r] = orc_f16_bits(v);
    }
}

void orc_int8_gemv_kernel_order(const uint8_t *W, const uint16_t *S, const uint16_t *B,
                                int st, const uint16_t *x16, float *y32, uint16_t *y16,
                                int m, int n) {
    const int ng = n / 64;
    for (int r = 0; r < m; ++r) {
        const uint8_t *wr = W + (size_t)r * n;
        float acc[32];
        for (int lane = 0; lane < 32; ++lane) {
            float a = 0.0f;
            for (int g = 0; g < ng; ++g) {
                float s = orc_scale_to_float(S[(size_t)r * ng + g], st);
                float b = orc_scale_to_float(B[(size_t)r * ng + g], st);
                int i0 = g * 64 + lane * 2;
                float x0 = orc_f16_to_float(x16[i0]), x1 = orc_f16_to_float(x16[i0 + 1]);
                float dq = (float)wr[i0] * x0 + (float)wr[i0 + 1] * x1;
                a = fmaf(s, dq, a);
                a = fmaf(b, x0 + x1, a);
            }
            acc[lane] = a;
        }
        float v = lane_sum32(acc);
        if (y32) y32[r] = v;
        if (y16) y16[r] = orc_f16_bits(v);
    }
}

float orc_rel_error(const float *a, const float *r, size_t n) {
    float md = 0.0f, rn = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float d = fabsf(a[i] - r[i]);
        if (d > md) md = d;
        if (fabsf(r[i]) > rn) rn = fabsf(r[i]);
    }
    return md / (rn > 1e-6f ? rn : 1e-6f);
}

float orc_hround_(float v) { return hround(v); }

/* ---------------- BASELINE synthetic inputs (config distributions) ------
 * codes q ~ U{0 .. 2^bits-1} from next() & mask, one draw per code;
 * scale = |N(0, 0.02)|, bias = -(2^bits / 2) * scale + N(0, 0.002), each
 * rounded to the storage type (BF16 or fp16);  x ~ N(0,1) rounded to fp16. */
void orc_fill_synthetic_affine(uint64_t *state, int rows, int cols, int bits, int scale_type,
                               uint8_t *packed, uint16_t *scales, uint16_t *biases) {
    const size_t rb = orc_packed_row_bytes(cols, bits);
    const int ng = cols / 64;
    const uint64_t mask = (1ull << bits) - 1ull;
    memset(packed, 0, rb * (size_t)rows);
    for (int r = 0; r < rows; ++r) {
        for (int k = 0; k < cols; ++k)
            orc_pack_code(packed + rb * (size_t)r, rb, (int)(orc_sm64_next(state) & mask), k, bits);
        for (int g = 0; g < ng; ++g) {
            float s = (float)fabs(orc_sm64_normal(state) * 0.02);
            float b = -(float)(1 << (bits - 1)) * s + (float)(orc_sm64_normal(state) * 0.002);
            scales[(size_t)r * ng + g] = scale_type == 1 ? orc_f16_bits(s) : orc_bf16_bits(s);
            biases[(size_t)r * ng + g] = scale_type == 1 ? orc_f16_bits(b) : orc_bf16_bits(b);
        }
    }
}

void orc_fill_normal_f16(uint64_t *state, float sigma, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = orc_f16_bits((float)(orc_sm64_normal(state) * sigma));
}
