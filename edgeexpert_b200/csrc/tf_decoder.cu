// tf_decoder.cu -- the dense decode stack around the MoE path (Gemma 4 decoder
// layer, RealForwardRunner.produceToken,
// Sources/TurboFieldfare/Runtime/Inference/RealForwardRunner.swift:2240-2480):
//   tf_rmsnorm            rmsnorm_bf16w / rmsnorm_no_scale (Metal/Primitives/rmsnorm.metal)
//   tf_qkv_epilogue       per-head Q/K/V RMSNorm + NeoX RoPE (fused_qkv_epilogue, fused.metal:84-170)
//   tf_attention_decode   split-KV GQA decode attention over an fp16 cache
//                         (attention_decode_partial/_combine, Metal/Attention/attention.metal:135-240)
//   tf_post_attn_setup    residual + pre-FFN / router norms (fused_post_attn_setup, fused.metal:190-269)
//   tf_layer_tail         the decoder-layer tail (fused_layer_tail, fused.metal:271-375)
//   tf_embed_int4         embed_lookup_int4 (Metal/Quant/dequant_int4.metal:65-84)
//   tf_lm_head_greedy     final norm + int4 LM head + greedy argmax
//                         (LMHeadChainInt4, Kernels/Fusions/LMHeadChainInt4.swift; logit.metal:687-787)
//
// All of these are HBM- or latency-bound small kernels: one CTA per row for
// the norms, a split-KV grid sized to the SM count for attention (each CTA
// reads one KV head's chunk once for all the query heads that share it), and
// the ring-streamed GEMV / tcgen05 GEMM with fp32 output for the LM head.
#include <initializer_list>

#include "tf_context.cuh"
#include "tf_gemv_tc.cuh"

using namespace tf;

namespace {

constexpr int kNormThreads = 256;
constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxChunk = 256;    // positions per split-KV chunk
constexpr int kAttnMaxGroup = 8;      // query heads per KV head
constexpr int kAttnMaxHeadDim = 512;

__device__ __forceinline__ float block_sum(float v, float* red) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();  // red may still be read from a previous call
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < nw ? red[lane] : 0.f;
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    return t;
}

__device__ __forceinline__ float rms_inv_of(float sumsq, int n, float eps) { return rsqrtf(sumsq / (float)n + eps); }

// out[r][i] = half(x[r][i] * inv * w[i]) (w == NULL: no scale)
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const __half* __restrict__ x, long long ldx,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __half* __restrict__ out, long long ldo, int d,
                                                               float eps) {
    __shared__ float red[32];
    const __half* xr = x + (long long)blockIdx.x * ldx;
    __half* orow = out + (long long)blockIdx.x * ldo;
    float acc = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = __half2float(xr[i]);
        acc = fmaf(v, v, acc);
    }
    const float inv = rms_inv_of(block_sum(acc, red), d, eps);
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        float v = __half2float(xr[i]) * inv;
        if (w) v *= __bfloat162float(w[i]);
        orow[i] = __float2half_rn(v);
    }
}

// One CTA per (token, head): heads [0, nq) are Q, [nq, nq+nkv) K, then V.
__global__ void __launch_bounds__(kNormThreads) qkv_epilogue_kernel(
    __half* __restrict__ q, long long ldq, __half* __restrict__ k, __half* __restrict__ v, long long ldkv,
    const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw, int hd, int nq, int nkv,
    float position, float theta, int rotated_pairs, float eps) {
    __shared__ float red[32];
    __shared__ float head[kAttnMaxHeadDim];
    const int t = blockIdx.y, hg = blockIdx.x;
    const bool is_q = hg < nq, is_k = !is_q && hg < nq + nkv;
    __half* dst = is_q ? q + (long long)t * ldq + (long long)hg * hd
                       : (is_k ? k + (long long)t * ldkv + (long long)(hg - nq) * hd
                               : v + (long long)t * ldkv + (long long)(hg - nq - nkv) * hd);
    const __nv_bfloat16* w = is_q ? qw : kw;
    float acc = 0.f;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        const float xv = __half2float(dst[i]);
        acc = fmaf(xv, xv, acc);
    }
    const float inv = rms_inv_of(block_sum(acc, red), hd, eps);
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float xv = __half2float(dst[i]) * inv;
        if (is_q || is_k) xv *= __bfloat162float(w[i]);
        head[i] = __half2float(__float2half_rn(xv));  // the norm's fp16 output boundary
    }
    __syncthreads();
    if (!is_q && !is_k) {
        for (int i = threadIdx.x; i < hd; i += blockDim.x) dst[i] = __float2half_rn(head[i]);
        return;
    }
    const int half_dim = hd / 2;
    for (int pair = threadIdx.x; pair < half_dim; pair += blockDim.x) {
        float x0 = head[pair], x1 = head[half_dim + pair];
        if (pair < rotated_pairs) {
            const float freq = powf(theta, -(float)(2 * pair) / (float)hd);
            float s, c;
            sincosf(position * freq, &s, &c);
            const float r0 = x0 * c - x1 * s;
            const float r1 = x0 * s + x1 * c;
            x0 = r0;
            x1 = r1;
        }
        dst[pair] = __float2half_rn(x0);
        dst[half_dim + pair] = __float2half_rn(x1);
    }
}

// Split-KV pass 1: CTA (chunk, kv head, token) scores the chunk's positions
// for the G query heads sharing the KV head, takes the chunk-local softmax
// and writes the un-normalised partial (m, d, o[hd]) per query head.
// Layout of the partials: md[((t*nq + h)*chunks + c)*2 + {0,1}], o[((t*nq + h)*chunks + c)*hd + i].
__global__ void __launch_bounds__(kAttnThreads) attention_partial_kernel(
    const __half* __restrict__ q, long long ldq, const __half* __restrict__ K, const __half* __restrict__ V,
    long long ld_seq, int hd, int nq, int nkv, int seq_len, int kv_start, int chunk_len, int chunks, float scale,
    float* __restrict__ md, float* __restrict__ po) {
    extern __shared__ __align__(16) float sm[];
    const int c = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
    const int G = nq / nkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* qs = sm;                            // [G][hd]
    float* sc = qs + G * hd;                   // [G][chunk_len]
    float* red = sc + G * kAttnMaxChunk;       // [warps][G][hd] (reused per 256-dim segment)
    const int p0 = kv_start + c * chunk_len;
    const int p1 = min(seq_len, p0 + chunk_len);
    const int np = max(0, p1 - p0);
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int g = i / hd, e = i - g * hd;
        qs[i] = __half2float(q[(long long)t * ldq + (long long)(kvh * G + g) * hd + e]);
    }
    __syncthreads();
    const __half* Kt = K + (long long)t * ld_seq + (long long)kvh * hd;
    const __half* Vt = V + (long long)t * ld_seq + (long long)kvh * hd;
    const long long pstride = (long long)nkv * hd;
    const int nseg = hd / 256 > 0 ? hd / 256 : 1;  // hd is a multiple of 256 or < 256
    const int seg_w = hd < 256 ? hd : 256;
    const bool lane_on = lane * 8 < seg_w;

    // scores: warp w takes positions w, w+8, ...; lane holds 8 consecutive
    // dims.  Four positions' rows are loaded before any is used, so each warp
    // keeps four 16-byte loads per lane in flight (the chunk is latency-bound
    // otherwise: one dependent round trip per position).
    constexpr int kPf = 4;
    for (int j0 = warp; j0 < np; j0 += kPf * kAttnWarps) {
        uint4 kv4[kPf][kAttnMaxHeadDim / 256];
#pragma unroll
        for (int k = 0; k < kPf; ++k) {
            const int j = j0 + k * kAttnWarps;
            const __half* kr = Kt + (long long)(p0 + min(j, np - 1)) * pstride;
#pragma unroll
            for (int seg = 0; seg < kAttnMaxHeadDim / 256; ++seg)
                kv4[k][seg] = (seg < nseg && lane_on && j < np)
                                  ? __ldcs(reinterpret_cast<const uint4*>(kr + seg * 256 + lane * 8))
                                  : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < kPf; ++k) {
            const int j = j0 + k * kAttnWarps;
            if (j >= np) break;
            float s[kAttnMaxGroup];
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; ++g) s[g] = 0.f;
#pragma unroll
            for (int seg = 0; seg < kAttnMaxHeadDim / 256; ++seg) {
                if (seg >= nseg || !lane_on) continue;
                const int e0 = seg * 256 + lane * 8;
                const __half2* kh = reinterpret_cast<const __half2*>(&kv4[k][seg]);
                float kf[8];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float2 f2 = __half22float2(kh[u]);
                    kf[2 * u] = f2.x;
                    kf[2 * u + 1] = f2.y;
                }
#pragma unroll
                for (int g = 0; g < kAttnMaxGroup; ++g) {
                    if (g >= G) break;
                    const float* qg = qs + g * hd + e0;
#pragma unroll
                    for (int u = 0; u < 8; ++u) s[g] = fmaf(qg[u], kf[u], s[g]);
                }
            }
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; ++g) {
                if (g >= G) break;
                float v = s[g];
                for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0) sc[g * kAttnMaxChunk + j] = v * scale;
            }
        }
    }
    __syncthreads();
    // chunk-local softmax: warp g < G owns head g
    __shared__ float s_m[kAttnMaxGroup], s_d[kAttnMaxGroup];
    if (warp < G) {
        float m = -INFINITY;
        for (int j = lane; j < np; j += 32) m = fmaxf(m, sc[warp * kAttnMaxChunk + j]);
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float dsum = 0.f;
        for (int j = lane; j < np; j += 32) {
            const float e = np ? __expf(sc[warp * kAttnMaxChunk + j] - m) : 0.f;
            sc[warp * kAttnMaxChunk + j] = e;
            dsum += e;
        }
        for (int o = 16; o; o >>= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, o);
        if (lane == 0) {
            s_m[warp] = m;
            s_d[warp] = dsum;
        }
    }
    __syncthreads();
    // o[g][i] = sum_p e[g][p] * V[p][i]: warp w takes positions w, w+8, ...
    for (int seg = 0; seg < nseg; ++seg) {
        float acc[kAttnMaxGroup][8];
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g)
#pragma unroll
            for (int u = 0; u < 8; ++u) acc[g][u] = 0.f;
        const int e0 = seg * 256 + lane * 8;
        if (lane_on) {
            for (int j0 = warp; j0 < np; j0 += kPf * kAttnWarps) {
                uint4 vv[kPf];  // four rows in flight, used in position order
#pragma unroll
                for (int k = 0; k < kPf; ++k) {
                    const int j = j0 + k * kAttnWarps;
                    vv[k] = j < np ? __ldcs(reinterpret_cast<const uint4*>(Vt + (long long)(p0 + j) * pstride + e0))
                                   : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int k = 0; k < kPf; ++k) {
                    const int j = j0 + k * kAttnWarps;
                    if (j >= np) break;
                    const __half2* vh = reinterpret_cast<const __half2*>(&vv[k]);
                    float vf[8];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const float2 f2 = __half22float2(vh[u]);
                        vf[2 * u] = f2.x;
                        vf[2 * u + 1] = f2.y;
                    }
#pragma unroll
                    for (int g = 0; g < kAttnMaxGroup; ++g) {
                        if (g >= G) break;
                        const float e = sc[g * kAttnMaxChunk + j];
#pragma unroll
                        for (int u = 0; u < 8; ++u) acc[g][u] = fmaf(e, vf[u], acc[g][u]);
                    }
                }
            }
        }
        __syncthreads();  // red is reused across segments
        if (lane_on) {
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; ++g) {
                if (g >= G) break;
                float4* r = reinterpret_cast<float4*>(red + ((size_t)warp * G + g) * 256 + lane * 8);
                r[0] = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
                r[1] = make_float4(acc[g][4], acc[g][5], acc[g][6], acc[g][7]);
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < G * seg_w; i += blockDim.x) {
            const int g = i / seg_w, e = i - g * seg_w;
            float v = 0.f;
            for (int w = 0; w < kAttnWarps; ++w) v += red[((size_t)w * G + g) * 256 + e];
            const long long row = ((long long)t * nq + kvh * G + g) * chunks + c;
            po[row * hd + seg * 256 + e] = v;
        }
    }
    if (threadIdx.x < G) {
        const long long row = ((long long)t * nq + kvh * G + threadIdx.x) * chunks + c;
        md[row * 2] = s_m[threadIdx.x];
        md[row * 2 + 1] = s_d[threadIdx.x];
    }
}

// Split-KV pass 1, streaming form (head_dim 64/128/256, at most 4 query
// heads per KV head): CTA (chunk, kv head, token) of 4 warps; a position's K
// and V rows are read by HD/8 lanes (8 dims each), so a warp covers 32/(HD/8)
// positions per step and keeps U steps of K and V rows (2U 16-byte loads per
// lane) in flight.  Each lane keeps an online softmax (m, d, o[8]) per query
// head over its positions: scores and values are read in one pass, with no
// score array in shared memory.  Lanes of other positions and the 4 warps
// are merged at the end: M = max m, d = sum d e^(m - M), o = sum o e^(m - M).
// The partial (m, d, o) goes to the same workspace rows as the two-pass form.
template <int HD, int G>
__global__ void __launch_bounds__(128, 4) attention_stream_kernel(
    const __half* __restrict__ q, long long ldq, const __half* __restrict__ K, const __half* __restrict__ V,
    long long ld_seq, int nq, int nkv, int seq_len, int kv_start, int chunk_len, int chunks, float scale,
    float* __restrict__ md, float* __restrict__ po) {
    constexpr int LPP = HD / 8;     // lanes per position
    constexpr int PPW = 32 / LPP;   // positions per warp step
    constexpr int NW = 4;
    constexpr int U = 4;            // warp steps in flight
    constexpr int STEP = NW * PPW;  // positions per CTA step
    __shared__ float s_m[NW][G], s_d[NW][G];
    __shared__ __align__(16) float s_o[NW][G][HD];
    const int c = blockIdx.x, kvh = blockIdx.y, t = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane / LPP, li = lane - sub * LPP;
    const int p0 = kv_start + c * chunk_len;
    const int np = max(0, min(seq_len, p0 + chunk_len) - p0);

    float qf[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const uint4 raw = *reinterpret_cast<const uint4*>(q + (long long)t * ldq + (long long)(kvh * G + g) * HD + li * 8);
        const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float2 f = __half22float2(h[u]);
            qf[g][2 * u] = f.x * scale;
            qf[g][2 * u + 1] = f.y * scale;
        }
    }
    float m[G], d[G], acc[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        d[g] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[g][e] = 0.f;
    }
    const long long pstride = (long long)nkv * HD;
    const __half* Kt = K + (long long)t * ld_seq + (long long)kvh * HD + li * 8 + (long long)p0 * pstride;
    const __half* Vt = V + (long long)t * ld_seq + (long long)kvh * HD + li * 8 + (long long)p0 * pstride;

    for (int base = warp * PPW; base < np; base += U * STEP) {  // warp-uniform bound
        uint4 kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = base + sub + u * STEP;
            kr[u] = make_uint4(0u, 0u, 0u, 0u);
            vr[u] = kr[u];
            if (j < np) {
                kr[u] = __ldcs(reinterpret_cast<const uint4*>(Kt + (long long)j * pstride));
                vr[u] = __ldcs(reinterpret_cast<const uint4*>(Vt + (long long)j * pstride));
            }
        }
        float s[U][G];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const __half2* kh = reinterpret_cast<const __half2*>(&kr[u]);
            float kf[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(kh[e]);
                kf[2 * e] = f.x;
                kf[2 * e + 1] = f.y;
            }
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float v = 0.f;
#pragma unroll
                for (int e = 0; e < 8; ++e) v = fmaf(qf[g][e], kf[e], v);
                s[u][g] = v;
            }
        }
#pragma unroll
        for (int o = LPP / 2; o; o >>= 1)
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int g = 0; g < G; ++g) s[u][g] += __shfl_xor_sync(0xffffffffu, s[u][g], o);
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (base + sub + u * STEP >= np)
#pragma unroll
                for (int g = 0; g < G; ++g) s[u][g] = -INFINITY;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mn = m[g];
#pragma unroll
            for (int u = 0; u < U; ++u) mn = fmaxf(mn, s[u][g]);
            if (mn == -INFINITY) continue;  // nothing valid yet for this lane
            const float corr = __expf(m[g] - mn);  // 0 when m is still -inf
            float p[U];
            float dsum = 0.f;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                p[u] = __expf(s[u][g] - mn);
                dsum += p[u];
            }
            d[g] = fmaf(d[g], corr, dsum);
            m[g] = mn;
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[g][e] *= corr;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const __half2* vh = reinterpret_cast<const __half2*>(&vr[u]);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(vh[e]);
                    acc[g][2 * e] = fmaf(p[u], f.x, acc[g][2 * e]);
                    acc[g][2 * e + 1] = fmaf(p[u], f.y, acc[g][2 * e + 1]);
                }
            }
        }
    }
    // merge the warp's position slots (lanes li, li + LPP, ...)
#pragma unroll
    for (int o = LPP; o < 32; o <<= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float mo = __shfl_xor_sync(0xffffffffu, m[g], o);
            const float dd = __shfl_xor_sync(0xffffffffu, d[g], o);
            const float mn = fmaxf(m[g], mo);
            const float a = mn == -INFINITY ? 0.f : __expf(m[g] - mn);
            const float b = mn == -INFINITY ? 0.f : __expf(mo - mn);
            d[g] = d[g] * a + dd * b;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const float ov = __shfl_xor_sync(0xffffffffu, acc[g][e], o);
                acc[g][e] = acc[g][e] * a + ov * b;
            }
            m[g] = mn;
        }
    }
    if (sub == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float4* r = reinterpret_cast<float4*>(&s_o[warp][g][li * 8]);
            r[0] = make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
            r[1] = make_float4(acc[g][4], acc[g][5], acc[g][6], acc[g][7]);
            if (li == 0) {
                s_m[warp][g] = m[g];
                s_d[warp][g] = d[g];
            }
        }
    }
    __syncthreads();
    // merge the warps in warp order and write the chunk's partial rows
    for (int i = threadIdx.x; i < G * HD; i += NW * 32) {
        const int g = i / HD, e = i - g * HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, s_m[w][g]);
        float D = 0.f, O = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < NW; ++w) {
                const float sc = __expf(s_m[w][g] - M);
                D = fmaf(s_d[w][g], sc, D);
                O = fmaf(s_o[w][g][e], sc, O);
            }
        }
        const long long row = ((long long)t * nq + kvh * G + g) * chunks + c;
        po[row * HD + e] = O;
        if (e == 0) {
            md[row * 2] = M;
            md[row * 2 + 1] = D;
        }
    }
}

// Split-KV pass 2: one CTA per (query head, token) merges the chunks:
// M = max m_c, D = sum d_c e^(m_c - M), out = half(sum o_c e^(m_c - M) / D).
__global__ void __launch_bounds__(kAttnThreads) attention_combine_kernel(const float* __restrict__ md,
                                                                          const float* __restrict__ po, int hd,
                                                                          int nq, int chunks, __half* __restrict__ out,
                                                                          long long ldo) {
    extern __shared__ __align__(16) float wts[];  // [chunks]
    __shared__ float s_D;
    const int h = blockIdx.x, t = blockIdx.y;
    const long long base = ((long long)t * nq + h) * chunks;
    if (threadIdx.x < 32) {
        float M = -INFINITY;
        for (int c = threadIdx.x; c < chunks; c += 32) M = fmaxf(M, md[(base + c) * 2]);
        for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        float D = 0.f;
        for (int c = threadIdx.x; c < chunks; c += 32) {
            const float m = md[(base + c) * 2];
            const float sc = (m == -INFINITY) ? 0.f : __expf(m - M);
            wts[c] = sc;
            D += md[(base + c) * 2 + 1] * sc;
        }
        for (int o = 16; o; o >>= 1) D += __shfl_xor_sync(0xffffffffu, D, o);
        if (threadIdx.x == 0) s_D = D;
    }
    __syncthreads();
    const float D = s_D;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float acc = 0.f;
        for (int c = 0; c < chunks; ++c) acc = fmaf(wts[c], po[(base + c) * hd + i], acc);
        out[(long long)t * ldo + (long long)h * hd + i] = __float2half_rn(D > 0.f ? acc / D : 0.f);
    }
}

// fused_post_attn_setup, one CTA per row; `sm` holds the row's fp16 hidden.
__global__ void __launch_bounds__(kNormThreads) post_attn_setup_kernel(
    __half* __restrict__ hidden, const __half* __restrict__ attn, __half* __restrict__ dense_x,
    __half* __restrict__ routed_x, __half* __restrict__ router_x, const __nv_bfloat16* __restrict__ w_post_attn,
    const __nv_bfloat16* __restrict__ w_pre_ffn, const __nv_bfloat16* __restrict__ w_pre_ffn2, int d, float eps) {
    extern __shared__ __align__(16) __half hs[];  // [d]
    __shared__ float red[32];
    const long long r = blockIdx.x;
    const __half* ar = attn + r * d;
    __half* hr = hidden + r * d;
    float acc = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = __half2float(ar[i]);
        acc = fmaf(v, v, acc);
    }
    const float inv_a = rms_inv_of(block_sum(acc, red), d, eps);
    acc = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float an = __half2float(__float2half_rn(__half2float(ar[i]) * inv_a * __bfloat162float(w_post_attn[i])));
        const __half h = __float2half_rn(__half2float(hr[i]) + an);
        hs[i] = h;
        hr[i] = h;
        const float hf = __half2float(h);
        acc = fmaf(hf, hf, acc);
    }
    const float inv_h = rms_inv_of(block_sum(acc, red), d, eps);
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float h = __half2float(hs[i]) * inv_h;
        if (dense_x) dense_x[r * d + i] = __float2half_rn(h * __bfloat162float(w_pre_ffn[i]));
        if (routed_x) routed_x[r * d + i] = __float2half_rn(h * __bfloat162float(w_pre_ffn2[i]));
        if (router_x) router_x[r * d + i] = __float2half_rn(h);
    }
}

// fused_layer_tail (+ the shared expert's post-FFN-1 norm when w1 != NULL), one CTA per row.
__global__ void __launch_bounds__(kNormThreads) layer_tail_kernel(
    const __half* __restrict__ h2, const __half* __restrict__ h1, __half* __restrict__ hidden,
    const __nv_bfloat16* __restrict__ w1, const __nv_bfloat16* __restrict__ w2, const __nv_bfloat16* __restrict__ w,
    float layer_scalar, int d, float eps) {
    extern __shared__ __align__(16) float tb[];  // [d] h1 (normed), then h12
    __shared__ float red[32];
    const long long r = blockIdx.x;
    const __half* h1r = h1 + r * d;
    const __half* h2r = h2 + r * d;
    __half* hr = hidden + r * d;
    float acc = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = __half2float(h1r[i]);
        tb[i] = v;
        acc = fmaf(v, v, acc);
    }
    if (w1) {
        const float inv1 = rms_inv_of(block_sum(acc, red), d, eps);
        for (int i = threadIdx.x; i < d; i += blockDim.x)
            tb[i] = __half2float(__float2half_rn(tb[i] * inv1 * __bfloat162float(w1[i])));
    }
    acc = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float v = __half2float(h2r[i]);
        acc = fmaf(v, v, acc);
    }
    const float inv2 = rms_inv_of(block_sum(acc, red), d, eps);
    acc = 0.f;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float tmp = __half2float(__float2half_rn(__half2float(h2r[i]) * inv2 * __bfloat162float(w2[i])));
        const float h12 = __half2float(__float2half_rn(tb[i] + tmp));
        tb[i] = h12;
        acc = fmaf(h12, h12, acc);
    }
    const float inv12 = rms_inv_of(block_sum(acc, red), d, eps);
    const float hs = __half2float(__float2half_rn(layer_scalar));
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        const float tmp = __half2float(__float2half_rn(tb[i] * inv12 * __bfloat162float(w[i])));
        const float hn = __half2float(__float2half_rn(__half2float(hr[i]) + tmp));
        hr[i] = __float2half_rn(hn * hs);
    }
}

// ---------------------------------------------------------------------------
// Register-resident forms of the three row norms for d % 8 == 0 and 16-byte
// aligned rows: a thread holds 8 consecutive elements of every operand (one
// 16-byte load each, issued together), so a row costs one memory round trip
// and the block reductions instead of one pass over memory per step.  Same
// element-wise arithmetic and roundings as the kernels above.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ld8h(const __half* p, bool on, float v[8]) {
    uint4 q = on ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0, 0, 0, 0);
    const __half2* h = reinterpret_cast<const __half2*>(&q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
    }
}
__device__ __forceinline__ void ld8b(const __nv_bfloat16* p, bool on, float v[8]) {
    uint4 q = on ? __ldg(reinterpret_cast<const uint4*>(p)) : make_uint4(0, 0, 0, 0);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        v[2 * j] = bf16_bits_to_float(w[j] & 0xFFFFu);
        v[2 * j + 1] = bf16_bits_to_float(w[j] >> 16);
    }
}
__device__ __forceinline__ void st8h(__half* p, const float v[8]) {
    uint4 q;
    __half2* h = reinterpret_cast<__half2*>(&q);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    *reinterpret_cast<uint4*>(p) = q;
}
__device__ __forceinline__ float rh(float v) { return __half2float(__float2half_rn(v)); }

__global__ void __launch_bounds__(1024) rmsnorm_vec_kernel(const __half* __restrict__ x, long long ldx,
                                                           const __nv_bfloat16* __restrict__ w,
                                                           __half* __restrict__ out, long long ldo, int d,
                                                           float eps) {
    __shared__ float red[32];
    const int i = threadIdx.x * 8;
    const bool on = i < d;
    float xv[8], wv[8];
    ld8h(x + (long long)blockIdx.x * ldx + i, on, xv);
    if (w) ld8b(w + i, on, wv);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(xv[j], xv[j], acc);
    const float inv = rms_inv_of(block_sum(acc, red), d, eps);
    if (!on) return;
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = w ? (xv[j] * inv) * wv[j] : xv[j] * inv;
    st8h(out + (long long)blockIdx.x * ldo + i, o);
}

__global__ void __launch_bounds__(1024) post_attn_setup_vec_kernel(
    __half* __restrict__ hidden, const __half* __restrict__ attn, __half* __restrict__ dense_x,
    __half* __restrict__ routed_x, __half* __restrict__ router_x, const __nv_bfloat16* __restrict__ w_post_attn,
    const __nv_bfloat16* __restrict__ w_pre_ffn, const __nv_bfloat16* __restrict__ w_pre_ffn2, int d, float eps) {
    __shared__ float red[32];
    const long long r = blockIdx.x;
    const int i = threadIdx.x * 8;
    const bool on = i < d;
    float a[8], h[8], wa[8], w1[8], w2[8];
    ld8h(attn + r * d + i, on, a);
    ld8h(hidden + r * d + i, on, h);
    ld8b(w_post_attn + i, on, wa);
    if (dense_x) ld8b(w_pre_ffn + i, on, w1);
    if (routed_x) ld8b(w_pre_ffn2 + i, on, w2);
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(a[j], a[j], acc);
    const float inv_a = rms_inv_of(block_sum(acc, red), d, eps);
    acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        h[j] = rh(h[j] + rh(a[j] * inv_a * wa[j]));
        acc = fmaf(h[j], h[j], acc);
    }
    const float inv_h = rms_inv_of(block_sum(acc, red), d, eps);
    if (!on) return;
    st8h(hidden + r * d + i, h);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] *= inv_h;
    if (dense_x) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = h[j] * w1[j];
        st8h(dense_x + r * d + i, o);
    }
    if (routed_x) {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = h[j] * w2[j];
        st8h(routed_x + r * d + i, o);
    }
    if (router_x) st8h(router_x + r * d + i, h);
}

__global__ void __launch_bounds__(1024) layer_tail_vec_kernel(
    const __half* __restrict__ h2, const __half* __restrict__ h1, __half* __restrict__ hidden,
    const __nv_bfloat16* __restrict__ w1, const __nv_bfloat16* __restrict__ w2, const __nv_bfloat16* __restrict__ w,
    float layer_scalar, int d, float eps) {
    __shared__ float red[32];
    const long long r = blockIdx.x;
    const int i = threadIdx.x * 8;
    const bool on = i < d;
    float t[8], v2[8], hv[8], a1[8], a2[8], a3[8];
    ld8h(h1 + r * d + i, on, t);
    ld8h(h2 + r * d + i, on, v2);
    ld8h(hidden + r * d + i, on, hv);
    if (w1) ld8b(w1 + i, on, a1);
    ld8b(w2 + i, on, a2);
    ld8b(w + i, on, a3);
    if (w1) {
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(t[j], t[j], acc);
        const float inv1 = rms_inv_of(block_sum(acc, red), d, eps);
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = rh(t[j] * inv1 * a1[j]);
    }
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(v2[j], v2[j], acc);
    const float inv2 = rms_inv_of(block_sum(acc, red), d, eps);
    acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        t[j] = rh(t[j] + rh(v2[j] * inv2 * a2[j]));
        acc = fmaf(t[j], t[j], acc);
    }
    const float inv12 = rms_inv_of(block_sum(acc, red), d, eps);
    if (!on) return;
    const float hs = rh(layer_scalar);
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = rh(hv[j] + rh(t[j] * inv12 * a3[j])) * hs;
    st8h(hidden + r * d + i, o);
}

// the register-resident kernels' preconditions: whole 16-byte vectors per row
inline bool vec_rows_ok(uint32_t d, std::initializer_list<const void*> ptrs, std::initializer_list<uint64_t> strides) {
    if (d % 8 || d > 8192) return false;
    for (const void* p : ptrs)
        if (p && (reinterpret_cast<uintptr_t>(p) & 15u)) return false;
    for (uint64_t st : strides)
        if (st % 8) return false;
    return true;
}
inline unsigned vec_threads(uint32_t d) { return (unsigned)(((d / 8) + 31) / 32 * 32); }

template <typename ST>
__global__ void embed_int4_kernel(const uint8_t* __restrict__ table, const ST* __restrict__ S,
                                  const ST* __restrict__ B, const uint32_t* __restrict__ tokens, int vocab, int d,
                                  float out_scale, __half* __restrict__ out, long long ldo, uint32_t* err) {
    const int t = blockIdx.y;
    const uint32_t tok = tokens[t];
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= d) return;
    if (tok >= (uint32_t)vocab) {
        out[t * ldo + i] = __float2half_rn(0.f);
        if (i == 0 && err) atomicOr(err, kErrBadExpert);
        return;
    }
    const uint8_t byte = table[(size_t)tok * (d / 2) + (i >> 1)];
    const int q = (i & 1) ? (byte >> 4) : (byte & 0xF);
    const float s = scale_to_float(S[(size_t)tok * (d / 64) + i / 64]);
    const float b = scale_to_float(B[(size_t)tok * (d / 64) + i / 64]);
    // multiply, add, multiply, each rounded once (no contraction), as the reference writes it
    out[t * ldo + i] = __float2half_rn(__fmul_rn(__fadd_rn(__fmul_rn((float)q, s), b), out_scale));
}

// Greedy argmax over fp32 logits [T][vocab] (finite values only; ties to the
// lower row).  Blocks fold into one 64-bit key per token with atomicMax: the
// high word is the order-preserving image of the float, the low word the
// complement of the row.  The last block of a token (ticket) writes the token
// (0 when no row is finite) and resets the key and the ticket.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t row) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - row);
}

__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ logits, long long ldl, int vocab,
                                                     unsigned long long* keys, unsigned int* tickets,
                                                     uint32_t* out_token) {
    const int t = blockIdx.y;
    const float* lr = logits + (long long)t * ldl;
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x) {
        const float v = lr[i];
        if (isfinite(v)) {
            const unsigned long long k = argmax_key(v, (uint32_t)i);
            best = k > best ? k : best;
        }
    }
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    __shared__ unsigned long long wb[8];
    __shared__ bool last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) wb[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = wb[w] > b ? wb[w] : b;
        if (b) atomicMax(&keys[t], b);
        __threadfence();
        last = atomicAdd(&tickets[t], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        const unsigned long long k = atomicExch(&keys[t], 0ull);
        out_token[t] = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
        tickets[t] = 0u;
    }
}

int attn_chunks(const tf_context* ctx, int T, int nkv, int seq_len) {
    if (seq_len <= 0) return 1;
    const int min_chunks = (seq_len + kAttnMaxChunk - 1) / kAttnMaxChunk;
    int want = (2 * ctx->num_sms + T * nkv - 1) / (T * nkv);  // about two CTAs per SM
    want = std::min(want, (seq_len + 31) / 32);               // at least 32 positions per chunk
    return std::max(min_chunks, std::max(1, want));
}

// The streaming form runs head_dim 64/128/256 with at most 4 query heads per
// KV head (TFCUDA_ATTN=split forces the two-pass form, read per call).
bool attn_streams(int G, int hd) {
    const char* e = getenv("TFCUDA_ATTN");
    if (e && strcmp(e, "split") == 0) return false;
    return G >= 1 && G <= 4 && (hd == 64 || hd == 128 || hd == 256);
}

// Chunks per (token, KV head) for the streaming form: the fewest whose CTAs
// fill the resident slots (4 CTAs per SM) to at least 90 % in their last
// wave, with at least 32 positions per chunk.  Independent of the live
// length except through that cap, so it never grows when kv_start does.
int attn_stream_chunks(const tf_context* ctx, int T, int nkv, int seq_len) {
    if (seq_len <= 0) return 1;
    const long long slots = 4LL * ctx->num_sms, pairs = (long long)T * nkv;
    const int maxc = std::max(1, (seq_len + 31) / 32);
    int best = 1;
    double best_eff = 0.0;
    for (int c = 1; c <= std::min(maxc, 1024); ++c) {
        const long long n = pairs * c;
        const double eff = (double)n / (double)(((n + slots - 1) / slots) * slots);
        if (eff >= 0.9) return c;
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = c;
        }
    }
    return best;
}

size_t attn_smem(int G, int hd) {
    return sizeof(float) * ((size_t)G * hd + (size_t)G * kAttnMaxChunk + (size_t)kAttnWarps * G * 256);
}

tf_status check(tf_context* ctx, const char* name) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "%s: cudaSetDevice failed", name);
    return TF_OK;
}

}  // namespace

extern "C" {

tf_status tf_rmsnorm(tf_context* ctx, const void* x, uint32_t x_stride, const void* weight, void* out,
                     uint32_t out_stride, uint32_t rows, uint32_t d, float eps, void* stream) {
    const char* name = "tf_rmsnorm";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (d == 0) return fail(ctx, TF_ERR_INVALID_ARG, "%s: d == 0", name);
    if (x_stride == 0) x_stride = d;
    if (out_stride == 0) out_stride = d;
    if (x_stride < d || out_stride < d) return fail(ctx, TF_ERR_INVALID_ARG, "%s: stride < d", name);
    if (rows == 0) return TF_OK;
    if (!x || !out) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned2(x) || !aligned2(out) || !aligned2(weight)) return fail(ctx, TF_ERR_MISALIGNED, "%s: misaligned", name);
    if (vec_rows_ok(d, {x, out, weight}, {x_stride, out_stride}))
        rmsnorm_vec_kernel<<<rows, vec_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const __half*>(x), x_stride, static_cast<const __nv_bfloat16*>(weight),
            static_cast<__half*>(out), out_stride, (int)d, eps);
    else
        rmsnorm_kernel<<<rows, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const __half*>(x), x_stride, static_cast<const __nv_bfloat16*>(weight),
            static_cast<__half*>(out), out_stride, (int)d, eps);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_qkv_epilogue(tf_context* ctx, void* q, uint32_t q_stride, void* k, void* v, uint64_t kv_stride,
                          const void* q_weight, const void* k_weight, uint32_t head_dim, uint32_t num_q_heads,
                          uint32_t num_kv_heads, uint32_t T, uint32_t position, float theta, uint32_t rotated_pairs,
                          float eps, void* stream) {
    const char* name = "tf_qkv_epilogue";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (head_dim == 0 || head_dim % 2 || head_dim > (uint32_t)kAttnMaxHeadDim || num_q_heads == 0 ||
        num_kv_heads == 0 || rotated_pairs > head_dim / 2)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: head_dim even and <= 512, heads > 0", name);
    if (q_stride == 0) q_stride = num_q_heads * head_dim;
    if (kv_stride == 0) kv_stride = (uint64_t)num_kv_heads * head_dim;
    if (T == 0) return TF_OK;
    if (!q || !k || !v || !q_weight || !k_weight) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    const dim3 grid(num_q_heads + 2 * num_kv_heads, T);
    qkv_epilogue_kernel<<<grid, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__half*>(q), q_stride, static_cast<__half*>(k), static_cast<__half*>(v), (long long)kv_stride,
        static_cast<const __nv_bfloat16*>(q_weight), static_cast<const __nv_bfloat16*>(k_weight), (int)head_dim,
        (int)num_q_heads, (int)num_kv_heads, (float)position, theta, (int)rotated_pairs, eps);
    return cuda_check(ctx, cudaGetLastError(), name);
}

size_t tf_attention_workspace_bytes(const tf_context* ctx, uint32_t T, uint32_t head_dim, uint32_t num_q_heads,
                                    uint32_t num_kv_heads, uint32_t seq_len) {
    if (!ctx || num_kv_heads == 0) return 0;
    const int G = (int)(num_q_heads / num_kv_heads);
    const int chunks = attn_streams(G, (int)head_dim)
                           ? attn_stream_chunks(ctx, (int)std::max(1u, T), (int)num_kv_heads, (int)seq_len)
                           : attn_chunks(ctx, (int)std::max(1u, T), (int)num_kv_heads, (int)seq_len);
    return sizeof(float) * (size_t)T * num_q_heads * chunks * (head_dim + 2);
}

tf_status tf_attention_decode(tf_context* ctx, const void* q, uint32_t q_stride, const void* k_cache,
                              const void* v_cache, uint64_t seq_stride, void* out, uint32_t out_stride,
                              uint32_t head_dim, uint32_t num_q_heads, uint32_t num_kv_heads, uint32_t T,
                              uint32_t seq_len, uint32_t kv_start, float scale, void* workspace,
                              size_t workspace_bytes, void* stream) {
    const char* name = "tf_attention_decode";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (head_dim == 0 || head_dim % 8 || (head_dim > 256 && head_dim % 256) || head_dim > (uint32_t)kAttnMaxHeadDim)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: head_dim a multiple of 8 up to 256, or of 256 up to 512", name);
    if (num_kv_heads == 0 || num_q_heads % num_kv_heads || num_q_heads / num_kv_heads > (uint32_t)kAttnMaxGroup)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: num_q_heads a multiple of num_kv_heads, at most 8 per KV head",
                    name);
    if (kv_start > seq_len) return fail(ctx, TF_ERR_INVALID_ARG, "%s: kv_start > seq_len", name);
    if (q_stride == 0) q_stride = num_q_heads * head_dim;
    if (out_stride == 0) out_stride = num_q_heads * head_dim;
    if (T == 0) return TF_OK;
    if (!q || !k_cache || !v_cache || !out || !workspace) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(k_cache) || !aligned16(v_cache) || (seq_stride * 2) % 16 || !aligned4(workspace))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: caches 16-byte aligned, sequence stride a multiple of 8", name);
    const int live = (int)(seq_len - kv_start);
    const int G = (int)(num_q_heads / num_kv_heads);
    const bool streams = attn_streams(G, (int)head_dim) && aligned16(q) && q_stride % 8 == 0;
    const int chunks = streams ? attn_stream_chunks(ctx, (int)T, (int)num_kv_heads, live)
                               : attn_chunks(ctx, (int)T, (int)num_kv_heads, live);
    const int chunk_len = live > 0 ? (live + chunks - 1) / chunks : 1;
    const size_t need = sizeof(float) * (size_t)T * num_q_heads * chunks * (head_dim + 2);
    if (workspace_bytes < need)
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: workspace of %zu bytes, %zu needed (tf_attention_workspace_bytes)",
                    name, workspace_bytes, need);
    float* md = static_cast<float*>(workspace);
    float* po = md + (size_t)T * num_q_heads * chunks * 2;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (streams) {
        const dim3 grid(chunks, num_kv_heads, T);
        const __half* qh = static_cast<const __half*>(q);
        const __half* kc = static_cast<const __half*>(k_cache);
        const __half* vc = static_cast<const __half*>(v_cache);
#define TF_ATTN_STREAM(HD, GG)                                                                                    \
    if ((int)head_dim == HD && G == GG)                                                                            \
        attention_stream_kernel<HD, GG><<<grid, 128, 0, cs>>>(qh, q_stride, kc, vc, (long long)seq_stride,         \
                                                              (int)num_q_heads, (int)num_kv_heads, (int)seq_len, \
                                                              (int)kv_start, chunk_len, chunks, scale, md, po);
        TF_ATTN_STREAM(64, 1) TF_ATTN_STREAM(64, 2) TF_ATTN_STREAM(64, 3) TF_ATTN_STREAM(64, 4)
        TF_ATTN_STREAM(128, 1) TF_ATTN_STREAM(128, 2) TF_ATTN_STREAM(128, 3) TF_ATTN_STREAM(128, 4)
        TF_ATTN_STREAM(256, 1) TF_ATTN_STREAM(256, 2) TF_ATTN_STREAM(256, 3) TF_ATTN_STREAM(256, 4)
#undef TF_ATTN_STREAM
        s = cuda_check(ctx, cudaGetLastError(), name);
        if (s) return s;
        attention_combine_kernel<<<dim3(num_q_heads, T), kAttnThreads, sizeof(float) * chunks, cs>>>(
            md, po, (int)head_dim, (int)num_q_heads, chunks, static_cast<__half*>(out), out_stride);
        return cuda_check(ctx, cudaGetLastError(), name);
    }
    const size_t smem = attn_smem(G, (int)head_dim);
    static bool configured[64] = {};
    if (!configured[ctx->device & 63]) {
        cudaError_t e = cudaFuncSetAttribute(attention_partial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)attn_smem(kAttnMaxGroup, kAttnMaxHeadDim));
        if (e != cudaSuccess) return cuda_check(ctx, e, name);
        configured[ctx->device & 63] = true;
    }
    attention_partial_kernel<<<dim3(chunks, num_kv_heads, T), kAttnThreads, smem, cs>>>(
        static_cast<const __half*>(q), q_stride, static_cast<const __half*>(k_cache),
        static_cast<const __half*>(v_cache), (long long)seq_stride, (int)head_dim, (int)num_q_heads,
        (int)num_kv_heads, (int)seq_len, (int)kv_start, chunk_len, chunks, scale, md, po);
    s = cuda_check(ctx, cudaGetLastError(), name);
    if (s) return s;
    attention_combine_kernel<<<dim3(num_q_heads, T), kAttnThreads, sizeof(float) * chunks, cs>>>(
        md, po, (int)head_dim, (int)num_q_heads, chunks, static_cast<__half*>(out), out_stride);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_post_attn_setup(tf_context* ctx, void* hidden, const void* attn, void* dense_x, void* routed_x,
                             void* router_x, const void* w_post_attn, const void* w_pre_ffn, const void* w_pre_ffn2,
                             uint32_t rows, uint32_t d, float eps, void* stream) {
    const char* name = "tf_post_attn_setup";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (d == 0 || d > 32768) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: 0 < d <= 32768", name);
    if (rows == 0) return TF_OK;
    if (!hidden || !attn || !w_post_attn || (dense_x && !w_pre_ffn) || (routed_x && !w_pre_ffn2))
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (vec_rows_ok(d, {hidden, attn, dense_x, routed_x, router_x, w_post_attn, w_pre_ffn, w_pre_ffn2}, {}))
        post_attn_setup_vec_kernel<<<rows, vec_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<__half*>(hidden), static_cast<const __half*>(attn), static_cast<__half*>(dense_x),
            static_cast<__half*>(routed_x), static_cast<__half*>(router_x),
            static_cast<const __nv_bfloat16*>(w_post_attn), static_cast<const __nv_bfloat16*>(w_pre_ffn),
            static_cast<const __nv_bfloat16*>(w_pre_ffn2), (int)d, eps);
    else
    post_attn_setup_kernel<<<rows, kNormThreads, sizeof(__half) * d, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__half*>(hidden), static_cast<const __half*>(attn), static_cast<__half*>(dense_x),
        static_cast<__half*>(routed_x), static_cast<__half*>(router_x),
        static_cast<const __nv_bfloat16*>(w_post_attn), static_cast<const __nv_bfloat16*>(w_pre_ffn),
        static_cast<const __nv_bfloat16*>(w_pre_ffn2), (int)d, eps);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_layer_tail(tf_context* ctx, const void* h2, const void* h1, void* hidden, const void* w_post_ffn1,
                        const void* w_post_ffn2, const void* w_post_ffn, float layer_scalar, uint32_t rows,
                        uint32_t d, float eps, void* stream) {
    const char* name = "tf_layer_tail";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (d == 0 || d > 16384) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: 0 < d <= 16384", name);
    if (rows == 0) return TF_OK;
    if (!h2 || !h1 || !hidden || !w_post_ffn2 || !w_post_ffn) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (vec_rows_ok(d, {h2, h1, hidden, w_post_ffn1, w_post_ffn2, w_post_ffn}, {}))
        layer_tail_vec_kernel<<<rows, vec_threads(d), 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const __half*>(h2), static_cast<const __half*>(h1), static_cast<__half*>(hidden),
            static_cast<const __nv_bfloat16*>(w_post_ffn1), static_cast<const __nv_bfloat16*>(w_post_ffn2),
            static_cast<const __nv_bfloat16*>(w_post_ffn), layer_scalar, (int)d, eps);
    else
    layer_tail_kernel<<<rows, kNormThreads, sizeof(float) * d, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(h2), static_cast<const __half*>(h1), static_cast<__half*>(hidden),
        static_cast<const __nv_bfloat16*>(w_post_ffn1), static_cast<const __nv_bfloat16*>(w_post_ffn2),
        static_cast<const __nv_bfloat16*>(w_post_ffn), layer_scalar, (int)d, eps);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_embed_int4(tf_context* ctx, const void* table, const void* scales, const void* biases,
                        const void* token_ids, uint32_t T, uint32_t vocab, uint32_t d, float out_scale, void* out,
                        uint32_t out_stride, tf_scale_type st, void* stream) {
    const char* name = "tf_embed_int4";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return fail(ctx, TF_ERR_INVALID_ARG, "%s: unknown scale type", name);
    if (d == 0 || d % 64) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d a positive multiple of 64", name);
    if (out_stride == 0) out_stride = d;
    if (T == 0) return TF_OK;
    if (!table || !scales || !biases || !token_ids || !out) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    const dim3 grid((d + 255) / 256, T);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (st == TF_SCALE_F16)
        embed_int4_kernel<__half><<<grid, 256, 0, cs>>>(
            static_cast<const uint8_t*>(table), static_cast<const __half*>(scales), static_cast<const __half*>(biases),
            static_cast<const uint32_t*>(token_ids), (int)vocab, (int)d, out_scale, static_cast<__half*>(out),
            out_stride, ctx->d_err);
    else
        embed_int4_kernel<__nv_bfloat16><<<grid, 256, 0, cs>>>(
            static_cast<const uint8_t*>(table), static_cast<const __nv_bfloat16*>(scales),
            static_cast<const __nv_bfloat16*>(biases), static_cast<const uint32_t*>(token_ids), (int)vocab, (int)d,
            out_scale, static_cast<__half*>(out), out_stride, ctx->d_err);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_lm_head_greedy(tf_context* ctx, const void* hidden, uint32_t hidden_stride, const void* norm_weight,
                            float eps, const void* W, const void* scales, const void* biases, uint32_t vocab,
                            uint32_t d, uint32_t T, void* x_normed, void* logits, void* out_tokens, tf_scale_type st,
                            void* stream) {
    const char* name = "tf_lm_head_greedy";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return fail(ctx, TF_ERR_INVALID_ARG, "%s: unknown scale type", name);
    if (d == 0 || d % 64 || vocab == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 64 == 0, vocab > 0", name);
    if (T > (uint32_t)kMaxLmTokens) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: at most %d tokens", name, kMaxLmTokens);
    if (T == 0) return TF_OK;
    if (!hidden || !W || !scales || !biases || !x_normed || !logits || !out_tokens)
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(x_normed) || !aligned16(logits) || !aligned4(out_tokens))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: x_normed / logits 16-byte aligned", name);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    s = tf_rmsnorm(ctx, hidden, hidden_stride, norm_weight, x_normed, d, T, d, eps, stream);
    if (s) return s;
    if (T == 1)
        s = gemv_stream_f32(ctx, W, scales, biases, x_normed, static_cast<float*>(logits), vocab, d, st, cs, name);
    else
        s = int4_qmm_f32(ctx, W, scales, biases, x_normed, static_cast<float*>(logits), T, vocab, d, d, vocab, st, cs,
                         name);
    if (s) return s;
    const int blocks = std::max(1, std::min((int)((vocab + 255) / 256), 2 * ctx->num_sms / (int)std::min(T, 2u)));
    argmax_kernel<<<dim3(blocks, T), 256, 0, cs>>>(static_cast<const float*>(logits), vocab, (int)vocab, ctx->d_lm_keys,
                                                   ctx->d_lm_tickets, static_cast<uint32_t*>(out_tokens));
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // extern "C"
