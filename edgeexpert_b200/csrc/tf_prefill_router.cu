// tf_prefill_router.cu -- batched router for prefill / batched decode
// (prefill_router_gemma4_block, Sources/TurboFieldfare/Metal/Prefill/prefill.metal:478-573;
//  PrefillRouter.encodeGemma4Block, Kernels/Prefill/MoE/PrefillRouter.swift:37-89).
//
// One CTA serves 8 tokens.  x~ = float(half h) * float(bf16 es) is staged per
// token as two fp16 terms (hi, lo), giving 16 MMA columns (token t -> columns
// 2t, 2t+1) in two 8-column groups.  Each warp takes 16-expert tiles and
// streams the int8 router rows from L2 straight into MMA fragments (codes
// exact in fp16), reusing each fragment for both column groups, and folds the
// per-group scale/bias in fp32.  Then every token selects its top-k by rank
// (logit desc, id asc -- the reference's insertion order), softmax over the
// k, times the per-expert gain.
#include "tf_context.cuh"

using namespace tf;

namespace {

constexpr int kRtTok = 8;          // tokens per CTA
constexpr int kRtCG = kRtTok / 4;  // 8-column MMA groups
constexpr int kRtThreads = 256;
constexpr int kRtMaxE = 256;
constexpr int kRtMaxK = 64;
constexpr int kRtSmemMax = 200 * 1024;  // d = 2816 needs ~104 KB: two CTAs per SM

template <typename ST>
__global__ void __launch_bounds__(kRtThreads) prefill_router_kernel(
    const uint8_t* __restrict__ W, const ST* __restrict__ S, const ST* __restrict__ B, const __half* __restrict__ H,
    int hstride, const __nv_bfloat16* __restrict__ es, const __nv_bfloat16* __restrict__ pes, uint32_t* out_idx,
    __half* out_w, float* out_logits, int T, int E, int D, int K) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int ws = x_words_stride(D);
    const int ng = D / kGroup;
    uint32_t* xs = reinterpret_cast<uint32_t*>(smem);                         // [2*kRtTok][ws]
    float* xsum = reinterpret_cast<float*>(xs + 2 * kRtTok * ws);               // [kRtTok][ng]
    float* logits = xsum + kRtTok * ng;                                         // [kRtTok][256]
    float* sel = logits + kRtTok * kRtMaxE;                                     // [kRtTok][64] selected logits
    uint32_t* selid = reinterpret_cast<uint32_t*>(sel + kRtTok * kRtMaxK);      // [kRtTok][64]
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
    for (int i = warp; i < kRtTok * ng; i += blockDim.x / 32) {
        const int t = i / ng, g = i - t * ng;
        const uint32_t a = xs[(2 * t) * ws + g * 32 + lane], b = xs[(2 * t + 1) * ws + g * 32 + lane];
        const __half2 ha = *reinterpret_cast<const __half2*>(&a);
        const __half2 hb = *reinterpret_cast<const __half2*>(&b);
        float s = (__low2float(ha) + __low2float(hb)) + (__high2float(ha) + __high2float(hb));
        for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        if (lane == 0) xsum[t * ng + g] = s;
    }
    __syncthreads();

    // logits: warp per 16-expert tile
    const int g = lane >> 2, t = lane & 3;
    for (int tile = warp; tile * 16 < E; tile += blockDim.x / 32) {
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
        uint4 qa, qb;
        float sc[4];
        ldw(0, qa, qb, sc);
        for (int G = 0; G < ng; ++G) {
            uint4 nqa = qa, nqb = qb;
            float nsc[4] = {0.f, 0.f, 0.f, 0.f};
            if (G + 1 < ng) ldw(G + 1, nqa, nqb, nsc);
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
            if (va) logits[(4 * cg + t) * kRtMaxE + rA] = accA[cg];
            if (vb) logits[(4 * cg + t) * kRtMaxE + rB] = accB[cg];
            if (out_logits && 4 * cg + t < ntok) {  // optional caller copy, [T][E]
                if (va) out_logits[(size_t)(t0 + 4 * cg + t) * E + rA] = accA[cg];
                if (vb) out_logits[(size_t)(t0 + 4 * cg + t) * E + rB] = accB[cg];
            }
        }
    }
    __syncthreads();

    // per-token rank selection
    for (int i = tid; i < kRtTok * E; i += blockDim.x) {
        const int tk = i / E, e = i - tk * E;
        if (tk >= ntok) continue;
        const float v = logits[tk * kRtMaxE + e];
        int rank = 0;
        for (int j = 0; j < E; ++j) {
            const float o = logits[tk * kRtMaxE + j];
            rank += (o > v || (o == v && j < e)) ? 1 : 0;
        }
        if (rank < K) {
            sel[tk * kRtMaxK + rank] = v;
            selid[tk * kRtMaxK + rank] = (uint32_t)e;
        }
    }
    __syncthreads();
    for (int i = tid; i < kRtTok * K; i += blockDim.x) {
        const int tk = i / K, r = i - tk * K;
        if (tk >= ntok) continue;
        const float vmax = sel[tk * kRtMaxK];
        float sum = 0.f;
        for (int j = 0; j < K; ++j) sum += expf(sel[tk * kRtMaxK + j] - vmax);
        const uint32_t e = selid[tk * kRtMaxK + r];
        out_idx[(size_t)(t0 + tk) * K + r] = e;
        out_w[(size_t)(t0 + tk) * K + r] =
            __float2half_rn(expf(sel[tk * kRtMaxK + r] - vmax) / sum * __bfloat162float(pes[e]));
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
                        (size_t)kRtTok * kRtMaxE * 4 + (size_t)kRtTok * kRtMaxK * 8;
    const dim3 grid((T + kRtTok - 1) / kRtTok);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    auto run = [&](auto* kernel) -> tf_status {
        static bool configured[64] = {};
        if (!configured[ctx->device & 63]) {
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRtSmemMax);
            if (e != cudaSuccess) return cuda_check(ctx, e, name);
            configured[ctx->device & 63] = true;
        }
        if (smem > (size_t)kRtSmemMax) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d too large", name);
        return TF_OK;
    };
    tf_status s;
    if (st == TF_SCALE_F16) {
        s = run(prefill_router_kernel<__half>);
        if (s) return s;
        prefill_router_kernel<__half><<<grid, kRtThreads, smem, cs>>>(
            static_cast<const uint8_t*>(W), static_cast<const __half*>(S), static_cast<const __half*>(B),
            static_cast<const __half*>(hidden), (int)hidden_stride, static_cast<const __nv_bfloat16*>(es),
            static_cast<const __nv_bfloat16*>(pes), static_cast<uint32_t*>(out_indices), static_cast<__half*>(out_weights),
            out_logits, (int)T, (int)E, (int)d, (int)top_k);
    } else {
        s = run(prefill_router_kernel<__nv_bfloat16>);
        if (s) return s;
        prefill_router_kernel<__nv_bfloat16><<<grid, kRtThreads, smem, cs>>>(
            static_cast<const uint8_t*>(W), static_cast<const __nv_bfloat16*>(S), static_cast<const __nv_bfloat16*>(B),
            static_cast<const __half*>(hidden), (int)hidden_stride, static_cast<const __nv_bfloat16*>(es),
            static_cast<const __nv_bfloat16*>(pes), static_cast<uint32_t*>(out_indices), static_cast<__half*>(out_weights),
            out_logits, (int)T, (int)E, (int)d, (int)top_k);
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
