// tf_prefill_router.cu -- batched router for prefill / batched decode
// (prefill_router_gemma4_block, Sources/TurboFieldfare/Metal/Prefill/prefill.metal:478-573;
//  PrefillRouter.encodeGemma4Block, Kernels/Prefill/MoE/PrefillRouter.swift:37-89).
//
// Logits: a CTA serves 8 tokens and `tpc` 16-expert tiles.  x~ = float(half
// h) * float(bf16 es) is staged per token as two fp16 terms (hi, lo), giving
// 16 MMA columns (token t -> columns 2t, 2t+1) in two 8-column groups.  The
// CTA's warps take its tiles and split K between them; each streams the int8
// router rows from L2 straight into MMA fragments (codes exact in fp16),
// reusing each fragment for both column groups, and folds the per-group
// scale/bias in fp32; the K slices are added in slice order.  A second launch
// selects every token's top-k (logit desc, id asc -- the reference's
// insertion order), softmax over the k, times the per-expert gain.
#include <algorithm>

#include "tf_context.cuh"

using namespace tf;

namespace {

constexpr int kRtTok = 8;          // tokens per CTA
constexpr int kRtCG = kRtTok / 4;  // 8-column MMA groups
constexpr int kRtThreads = 256;
constexpr int kRtWarps = kRtThreads / 32;
constexpr int kRtMaxE = 256;
constexpr int kRtMaxK = 64;
constexpr int kRtSmemMax = 200 * 1024;  // d = 2816 needs ~104 KB: two CTAs per SM

template <typename ST>
__global__ void __launch_bounds__(kRtThreads) prefill_router_kernel(
    const uint8_t* __restrict__ W, const ST* __restrict__ S, const ST* __restrict__ B, const __half* __restrict__ H,
    int hstride, const __nv_bfloat16* __restrict__ es, float* __restrict__ logits_out, int T, int E, int D, int tpc) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int ws = x_words_stride(D);
    const int ng = D / kGroup;
    uint32_t* xs = reinterpret_cast<uint32_t*>(smem);            // [2*kRtTok][ws]
    float* xsum = reinterpret_cast<float*>(xs + 2 * kRtTok * ws);  // [kRtTok][ng]
    float* red = xsum + kRtTok * ng;                               // [warp][kRtTok][16] slice partials
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * kRtTok;
    const int ntok = min(kRtTok, T - t0);

    // stage hi/lo (columns 2t, 2t+1) in octet-pair order
    const bool hvec = ((reinterpret_cast<uintptr_t>(H) | reinterpret_cast<uintptr_t>(es)) & 15u) == 0 &&
                      (hstride & 7) == 0;
    for (int i = tid; i < kRtTok * (D / 8); i += blockDim.x) {
        const int t = i / (D / 8), q = i - t * (D / 8);
        __half hv[8];
        __nv_bfloat16 ev[8];
        if (t < ntok && hvec) {
            const uint4 hr = __ldg(reinterpret_cast<const uint4*>(H + (size_t)(t0 + t) * hstride + q * 8));
            const uint4 er = __ldg(reinterpret_cast<const uint4*>(es + q * 8));
            memcpy(hv, &hr, 16);
            memcpy(ev, &er, 16);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                hv[j] = t < ntok ? H[(size_t)(t0 + t) * hstride + q * 8 + j] : __float2half(0.f);
                ev[j] = es[q * 8 + j];
            }
        }
        __half hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float xt = t < ntok ? __half2float(hv[j]) * __bfloat162float(ev[j]) : 0.f;
            hi[j] = __float2half_rn(xt);
            lo[j] = __float2half_rn(xt - __half2float(hi[j]));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 a = __halves2half2(hi[j], hi[j + 4]);
            __half2 b = __halves2half2(lo[j], lo[j + 4]);
            xs[(2 * t) * ws + q * 4 + j] = *reinterpret_cast<uint32_t*>(&a);
            xs[(2 * t + 1) * ws + q * 4 + j] = *reinterpret_cast<uint32_t*>(&b);
        }
    }
    __syncthreads();
    // per (token, group) sum of the staged hi + lo terms: one thread per item
    // (eight 16-byte loads of each half, started at a thread-dependent chunk
    // so a quarter-warp reads distinct banks), no shuffle chains
    for (int i = tid; i < kRtTok * ng; i += blockDim.x) {
        const int t = i / ng, g = i - t * ng;
        const uint4* ha = reinterpret_cast<const uint4*>(xs + (2 * t) * ws + g * 32);
        const uint4* hb = reinterpret_cast<const uint4*>(xs + (2 * t + 1) * ws + g * 32);
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int q = (k + i) & 7;
            const uint4 a = ha[q], b = hb[q];
            const uint32_t wa[4] = {a.x, a.y, a.z, a.w}, wb[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&wa[j]));
                const float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&wb[j]));
                s += (fa.x + fb.x) + (fa.y + fb.y);
            }
        }
        xsum[t * ng + g] = s;
    }
    __syncthreads();

    // logits: this CTA's tpc 16-expert tiles, kRtWarps / tpc warps (K slices,
    // groups slice, slice + ksw, ...) per tile
    const int ksw = kRtWarps / tpc;
    const int tile = blockIdx.y * tpc + warp / ksw, slice = warp % ksw;
    const int g = lane >> 2, t = lane & 3;
    if (tile * 16 < E) {
        const int rA = tile * 16 + g, rB = rA + 8;
        const bool va = rA < E, vb = rB < E;
        const uint8_t* wA = W + (size_t)(va ? rA : 0) * D;
        const uint8_t* wB = W + (size_t)(vb ? rB : 0) * D;
        float accA[kRtCG], accB[kRtCG];  // (row g, token 4c+t), (row g+8, token 4c+t)
#pragma unroll
        for (int c = 0; c < kRtCG; ++c) accA[c] = accB[c] = 0.f;
        // software pipeline: the next group's weights and scales are loaded
        // (from L2) while the current group's MMAs run
        auto ldw = [&](int G, uint4& qa, uint4& qb, float sc[4]) {
            qa = __ldg(reinterpret_cast<const uint4*>(wA + G * 64 + t * 16));
            qb = __ldg(reinterpret_cast<const uint4*>(wB + G * 64 + t * 16));
            sc[0] = va ? scale_to_float(S[(size_t)rA * ng + G]) : 0.f;
            sc[1] = va ? scale_to_float(B[(size_t)rA * ng + G]) : 0.f;
            sc[2] = vb ? scale_to_float(S[(size_t)rB * ng + G]) : 0.f;
            sc[3] = vb ? scale_to_float(B[(size_t)rB * ng + G]) : 0.f;
        };
        uint4 qa = make_uint4(0, 0, 0, 0), qb = qa;
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        if (slice < ng) ldw(slice, qa, qb, sc);
        for (int G = slice; G < ng; G += ksw) {
            uint4 nqa = qa, nqb = qb;
            float nsc[4] = {0.f, 0.f, 0.f, 0.f};
            if (G + ksw < ng) ldw(G + ksw, nqa, nqb, nsc);
            uint32_t pa0[4], pa1[4], pb0[4], pb1[4];
            dq8(qa.x, qa.y, pa0);
            dq8(qa.z, qa.w, pa1);
            dq8(qb.x, qb.y, pb0);
            dq8(qb.z, qb.w, pb1);
#pragma unroll
            for (int cg = 0; cg < kRtCG; ++cg) {
                // B fragment: column g of group cg = token 4cg + g/2, part g%2
                const uint4* xp = reinterpret_cast<const uint4*>(xs + (cg * 8 + g) * ws + (G * 8 + 2 * t) * 4);
                const uint4 x0 = xp[0], x1 = xp[1];
                float c[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(c, pa0[0], pb0[0], pa0[1], pb0[1], x0.x, x0.y);
                mma16816(cb, pa0[2], pb0[2], pa0[3], pb0[3], x0.z, x0.w);
                mma16816(c, pa1[0], pb1[0], pa1[1], pb1[1], x1.x, x1.y);
                mma16816(cb, pa1[2], pb1[2], pa1[3], pb1[3], x1.z, x1.w);
                const float xsm = xsum[(4 * cg + t) * ng + G];
                // columns 2t (hi) and 2t+1 (lo) of this lane are token 4cg + t
                accA[cg] = fmaf(sc[0], (c[0] + cb[0]) + (c[1] + cb[1]), accA[cg]);
                accA[cg] = fmaf(sc[1], xsm, accA[cg]);
                accB[cg] = fmaf(sc[2], (c[2] + cb[2]) + (c[3] + cb[3]), accB[cg]);
                accB[cg] = fmaf(sc[3], xsm, accB[cg]);
            }
            qa = nqa;
            qb = nqb;
#pragma unroll
            for (int i = 0; i < 4; ++i) sc[i] = nsc[i];
        }
#pragma unroll
        for (int cg = 0; cg < kRtCG; ++cg) {
            red[(warp * kRtTok + 4 * cg + t) * 16 + g] = accA[cg];
            red[(warp * kRtTok + 4 * cg + t) * 16 + g + 8] = accB[cg];
        }
    }
    __syncthreads();
    // slices summed in slice order; logits [T][E] in global memory
    for (int i = tid; i < tpc * kRtTok * 16; i += blockDim.x) {
        const int tl = i / (kRtTok * 16), tok = (i / 16) % kRtTok, row = i % 16;
        const int e = (blockIdx.y * tpc + tl) * 16 + row;
        if (e >= E || tok >= ntok) continue;
        float v = 0.f;
        for (int sl = 0; sl < ksw; ++sl) v += red[((tl * ksw + sl) * kRtTok + tok) * 16 + row];
        logits_out[(size_t)(t0 + tok) * E + e] = v;
    }
}

// Per token (one warp each): top-k by (logit desc, id asc) -- the
// reference's insertion order -- softmax over the k, times the gain.
__global__ void __launch_bounds__(256) router_select_kernel(const float* __restrict__ logits, int T, int E, int K,
                                                            const __nv_bfloat16* __restrict__ pes, uint32_t* out_idx,
                                                            __half* out_w) {
    __shared__ float sv[8][kRtMaxK];
    __shared__ uint32_t si[8][kRtMaxK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tk = blockIdx.x * 8 + warp;
    if (tk >= T) return;
    float v[kRtMaxE / 32];
    uint32_t taken = 0;
#pragma unroll
    for (int j = 0; j < kRtMaxE / 32; ++j) {
        const int e = lane + 32 * j;
        v[j] = e < E ? logits[(size_t)tk * E + e] : 0.f;
        if (e >= E) taken |= 1u << j;
    }
    for (int r = 0; r < K; ++r) {
        float bv = 0.f;
        int be = -1;
#pragma unroll
        for (int j = 0; j < kRtMaxE / 32; ++j) {
            const int e = lane + 32 * j;
            if (!(taken >> j & 1u) && (be < 0 || v[j] > bv)) {  // e ascending: ties keep the lower id
                bv = v[j];
                be = e;
            }
        }
        for (int off = 16; off; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oe = __shfl_xor_sync(0xffffffffu, be, off);
            if (oe >= 0 && (be < 0 || ov > bv || (ov == bv && oe < be))) {
                bv = ov;
                be = oe;
            }
        }
        if (be >= 0 && (be & 31) == lane) taken |= 1u << (be >> 5);
        if (lane == 0) {
            sv[warp][r] = bv;
            si[warp][r] = (uint32_t)be;
        }
    }
    __syncwarp();
    const float vmax = sv[warp][0];
    float sum = 0.f;
    for (int j = 0; j < K; ++j) sum += expf(sv[warp][j] - vmax);
    for (int r = lane; r < K; r += 32) {
        const uint32_t e = si[warp][r];
        out_idx[(size_t)tk * K + r] = e;
        out_w[(size_t)tk * K + r] = __float2half_rn(expf(sv[warp][r] - vmax) / sum * __bfloat162float(pes[e]));
    }
}

}  // namespace

extern "C" {

static tf_status router_batched(tf_context* ctx, const void* W, const void* S, const void* B, const void* hidden,
                                uint32_t hidden_stride, const void* es, const void* pes, void* out_indices,
                                void* out_weights, float* out_logits, uint32_t T, uint32_t E, uint32_t d,
                                uint32_t top_k, tf_scale_type st, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    const char* name = "tf_router_topk_batched";
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return fail(ctx, TF_ERR_INVALID_ARG, "%s: unknown scale type", name);
    if (T == 0) return TF_OK;
    if (!W || !S || !B || !hidden || !es || !pes || !out_indices || !out_weights)
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (d == 0 || d % 64) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d must be a positive multiple of 64", name);
    if (E == 0 || E > (uint32_t)kRtMaxE) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: num_experts must be in 1..256", name);
    if (top_k == 0 || top_k > (uint32_t)kRtMaxK || top_k > E)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: top_k must be in 1..min(64, num_experts)", name);
    if (hidden_stride < d) return fail(ctx, TF_ERR_INVALID_ARG, "%s: hidden stride is too small", name);
    if ((reinterpret_cast<uintptr_t>(W) & 15u) || (d % 16) || !aligned2(S) || !aligned2(B) || !aligned2(hidden))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: router weights must be 16-byte aligned", name);
    const size_t smem = (size_t)2 * kRtTok * x_words_stride((int)d) * 4 + (size_t)kRtTok * (d / 64) * 4 +
                        (size_t)kRtWarps * kRtTok * 16 * 4;
    if (smem > (size_t)kRtSmemMax) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d too large", name);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    static bool configured[2][64] = {};
    const void* kfn = st == TF_SCALE_F16 ? reinterpret_cast<const void*>(&prefill_router_kernel<__half>)
                                         : reinterpret_cast<const void*>(&prefill_router_kernel<__nv_bfloat16>);
    if (!configured[st][ctx->device & 63]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kRtSmemMax);
        if (e != cudaSuccess) return cuda_check(ctx, e, name);
        configured[st][ctx->device & 63] = true;
    }
    // Logits go to the caller's array when given, else to the context's
    // scratch in token chunks that fit it.  Expert tiles are spread over
    // CTAs (tpc tiles each, the rest of the CTA's warps split K) until the
    // grid covers about two CTAs per SM.
    const int tiles = (int)((E + 15) / 16);
    const uint32_t chunk = out_logits ? T : (uint32_t)(kRtLogitsCap / E) / kRtTok * kRtTok;
    for (uint32_t c0 = 0; c0 < T; c0 += chunk) {
        const uint32_t Tc = std::min(chunk, T - c0);
        float* lg = out_logits ? out_logits : ctx->d_rt_logits;
        const long long gx = (Tc + kRtTok - 1) / kRtTok;
        int tpc = kRtWarps;
        while (tpc > 1 && gx * ((tiles + tpc - 1) / tpc) < 2ll * ctx->num_sms) tpc >>= 1;
        const dim3 grid((unsigned)gx, (unsigned)((tiles + tpc - 1) / tpc));
        const __half* h = static_cast<const __half*>(hidden) + (size_t)c0 * hidden_stride;
        float* lgc = lg + (out_logits ? (size_t)c0 * E : 0);
        if (st == TF_SCALE_F16)
            prefill_router_kernel<__half><<<grid, kRtThreads, smem, cs>>>(
                static_cast<const uint8_t*>(W), static_cast<const __half*>(S), static_cast<const __half*>(B), h,
                (int)hidden_stride, static_cast<const __nv_bfloat16*>(es), lgc, (int)Tc, (int)E, (int)d, tpc);
        else
            prefill_router_kernel<__nv_bfloat16><<<grid, kRtThreads, smem, cs>>>(
                static_cast<const uint8_t*>(W), static_cast<const __nv_bfloat16*>(S),
                static_cast<const __nv_bfloat16*>(B), h, (int)hidden_stride, static_cast<const __nv_bfloat16*>(es),
                lgc, (int)Tc, (int)E, (int)d, tpc);
        router_select_kernel<<<(Tc + 7) / 8, 256, 0, cs>>>(lgc, (int)Tc, (int)E, (int)top_k,
                                                            static_cast<const __nv_bfloat16*>(pes),
                                                            static_cast<uint32_t*>(out_indices) + (size_t)c0 * top_k,
                                                            static_cast<__half*>(out_weights) + (size_t)c0 * top_k);
    }
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_router_topk_batched(tf_context* ctx, const void* W, const void* S, const void* B, const void* hidden,
                                 uint32_t hidden_stride, const void* es, const void* pes, void* out_indices,
                                 void* out_weights, uint32_t T, uint32_t E, uint32_t d, uint32_t top_k,
                                 tf_scale_type st, void* stream) {
    return router_batched(ctx, W, S, B, hidden, hidden_stride, es, pes, out_indices, out_weights, nullptr, T, E, d,
                          top_k, st, stream);
}

tf_status tf_router_topk_batched_with_logits(tf_context* ctx, const void* W, const void* S, const void* B,
                                             const void* hidden, uint32_t hidden_stride, const void* es,
                                             const void* pes, void* out_indices, void* out_weights,
                                             void* out_logits, uint32_t T, uint32_t E, uint32_t d, uint32_t top_k,
                                             tf_scale_type st, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (!out_logits) return fail(ctx, TF_ERR_INVALID_ARG, "tf_router_topk_batched_with_logits: null out_logits");
    if (reinterpret_cast<uintptr_t>(out_logits) & 3u)
        return fail(ctx, TF_ERR_MISALIGNED, "tf_router_topk_batched_with_logits: out_logits must be 4-byte aligned");
    return router_batched(ctx, W, S, B, hidden, hidden_stride, es, pes, out_indices, out_weights,
                          static_cast<float*>(out_logits), T, E, d, top_k, st, stream);
}

}  // extern "C"
