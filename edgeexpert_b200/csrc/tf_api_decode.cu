// tf_api_decode.cu -- C ABI: context, GEMVs, router, decode MoE layer.
#include <stdlib.h>

#include <algorithm>

#include "tf_context.cuh"
#include "tf_fused.cuh"
#include "tf_gemv_tc.cuh"
#include "tf_lowbit.cuh"

using namespace tf;

namespace {

template <class Fn>
tf_status dispatch_scale(tf_scale_type st, Fn&& fn) {
    if (st == TF_SCALE_F16) return fn(__half{});
    if (st == TF_SCALE_BF16) return fn(__nv_bfloat16{});
    return TF_ERR_INVALID_ARG;  // not a tf_scale_type value
}

tf_status check_ctx(tf_context* ctx) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    return TF_OK;
}

ExpertSource make_source(const void* pool, uint64_t stride, uint32_t E, const void* ids, const void* const* blobs,
                         const tf_expert_offsets* o, uint32_t top_k) {
    ExpertSource s;
    memset(&s, 0, sizeof(s));
    s.pool = static_cast<const uint8_t*>(pool);
    s.stride = stride;
    s.ids = static_cast<const uint32_t*>(ids);
    s.num_experts = (int)E;
    if (!ids && blobs)
        for (uint32_t i = 0; i < top_k && i < 8; ++i) s.blobs[i] = static_cast<const uint8_t*>(blobs[i]);
    const uint32_t off[9] = {o->gate_w, o->gate_s, o->gate_b, o->up_w, o->up_s, o->up_b, o->down_w, o->down_s, o->down_b};
    memcpy(s.off, off, sizeof(off));
    return s;
}

// TMA descriptors for one weight sub-tensor (byte offset `off` inside each
// expert blob) of all routed experts: one 3-D map over the pool, or one map
// per slot for explicit blobs.  False when any cannot be described.
bool source_maps(const ExpertSource& s, uint32_t top_k, uint32_t off, uint64_t rb, uint64_t rows, CUtensorMap* maps) {
    if (s.ids) return make_weight_map(&maps[0], s.pool + off, rb, rows, (uint64_t)s.num_experts, s.stride);
    bool ok = true;
    for (uint32_t i = 0; i < top_k; ++i) ok = make_weight_map(&maps[i], s.blobs[i] + off, rb, rows, 1, 0) && ok;
    return ok;
}

tf_status check_source(tf_context* ctx, const void* pool, const void* ids, const void* const* blobs,
                       const tf_expert_offsets* off, uint32_t E, uint32_t top_k, const char* name) {
    if (!off) return fail(ctx, TF_ERR_INVALID_ARG, "%s: offsets is NULL", name);
    if (top_k == 0 || top_k > 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: top_k must be in 1..8, got %u", name, top_k);
    if (ids) {
        if (!pool || E == 0) return fail(ctx, TF_ERR_INVALID_ARG, "%s: expert pool / num_experts missing", name);
    } else {
        if (!blobs) return fail(ctx, TF_ERR_INVALID_ARG, "%s: need expert_ids or blobs", name);
        for (uint32_t i = 0; i < top_k; ++i)
            if (!blobs[i]) return fail(ctx, TF_ERR_INVALID_ARG, "%s: blob %u is NULL", name, i);
    }
    const uint32_t o[9] = {off->gate_w, off->gate_s, off->gate_b, off->up_w, off->up_s, off->up_b, off->down_w, off->down_s, off->down_b};
    for (int i = 0; i < 9; ++i)
        if (o[i] & 1u) return fail(ctx, TF_ERR_MISALIGNED, "%s: expert sub-tensor offsets must be 2-byte aligned", name);
    return TF_OK;
}

// Batch-1 int4 work on the integer tensor path (activation as a 15-bit
// per-group integer in two int8 halves, mma.sync u8 x s8, 4 groups x {hi, lo}
// per 8 MMA columns).  The default for the GEMV and, with a helper warp per
// stage and load-batched staging, for the decode phases (measured faster on
// B200 than the fp16 path for both); TFCUDA_XINT=0 / 1 forces it off / on.
static bool xint_enabled(bool default_on) {
    const char* e = getenv("TFCUDA_XINT");
    if (e && e[0] == '1') return true;
    if (e && e[0] == '0') return false;
    return default_on;
}

static bool helpers_enabled() {
    const char* e = getenv("TFCUDA_HELPERS");
    return !(e && e[0] == '0');
}

tf_status gemv_common(tf_context* ctx, uint32_t bits, const void* W, const void* S, const void* B, uint64_t wbs,
                      uint64_t sbs, uint32_t batch, const void* x, uint32_t ntok, uint32_t xrs, void* y, uint32_t yrs,
                      uint64_t ybs, uint32_t m, uint32_t n, tf_scale_type st, void* stream, const char* name) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    if (!W || !S || !B || !x || !y) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (bits != 2 && bits != 3 && bits != 4 && bits != 8)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: bits must be 2, 3, 4 or 8", name);
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return fail(ctx, TF_ERR_INVALID_ARG, "%s: unknown scale type", name);
    if (m == 0 || n == 0 || batch == 0 || ntok == 0) return fail(ctx, TF_ERR_INVALID_ARG, "%s: zero dimension", name);
    if (n % 64) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: N must be a multiple of 64, got %u", name, n);
    if (ntok > 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: at most 8 tokens per call, got %u", name, ntok);
    if (!aligned2(W) || !aligned2(S) || !aligned2(B) || !aligned2(x) || !aligned2(y))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: buffers must be 2-byte aligned", name);
    if (bits == 2 || bits == 3)  // tf_lowbit.cu
        return lowbit_gemv(ctx, bits, W, S, B, wbs, sbs, batch, x, ntok, xrs, y, nullptr, yrs, ybs, m, n, st,
                           static_cast<cudaStream_t>(stream), name);
    // One token of int4 over at least one 128-row tile per SM: the ring-streamed
    // integer GEMV (tf_gemv_tc.cu).  TFCUDA_GEMV (read per call): "engine"
    // keeps the streaming engine, "stream" / "tc" force the integer / the
    // tcgen05 ring kernel for any tile count.
    if (bits == 4 && ntok == 1 && xint_enabled(true)) {
        const char* env = getenv("TFCUDA_GEMV");
        const bool eng = env && strcmp(env, "engine") == 0;
        const bool tc = env && strcmp(env, "tc") == 0;
        const bool forced = tc || (env && strcmp(env, "stream") == 0);
        if (!eng) {
            bool used = false;
            tf_status rc = gemv_tc_try(ctx, W, S, B, wbs, sbs, batch, x, y, ybs, m, n, st,
                                       static_cast<cudaStream_t>(stream), tc ? kGemvTensorCore : kGemvStream,
                                       forced ? 1 : 0, &used, name);
            if (rc || used) return rc;
        }
    }
    GemvParams p;
    memset(&p, 0, sizeof(p));
    p.W = static_cast<const uint8_t*>(W);
    p.S = S;
    p.B = B;
    p.w_bstride = (long long)wbs;
    p.sb_bstride = (long long)sbs;
    p.M = (int)m;
    p.K = (int)n;
    p.batch = (int)batch;
    p.bits = (int)bits;
    p.x = static_cast<const __half*>(x);
    p.x_row_stride = (int)xrs;
    p.ntok = (int)ntok;
    p.xint = (bits == 4 && ntok == 1 && xint_enabled(true)) ? 1 : 0;
    p.y = static_cast<__half*>(y);
    p.y_row_stride = (int)yrs;
    p.y_bstride = (long long)ybs;
    // TMA path when the weights can be described (16-byte aligned base and
    // batch stride); otherwise the synchronous 16-bit copy path.
    p.aligned = make_weight_map(&p.map, W, row_bytes((int)n, (int)bits), m, batch, wbs);
    p.x_aligned = aligned16(x) && (ntok == 1 || (xrs % 8) == 0);
    p.err = ctx->d_err;
    const int U = units_for_K((int)n, (int)bits);
    p.tiles = ((int)m + 15) / 16;
    p.sched = make_sched((int)batch * p.tiles, U, 0, 1, ctx->num_sms);
    const int sj = p.sched.S_total;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    return dispatch_scale(st, [&](auto tag) {
        using ST = decltype(tag);
        using Pol = GemvPolicy<ST>;
        // Tokens per launch: as many as the staged activations fit in shared memory.
        int tpl = (int)ntok;
        const size_t limit = engine_smem_limit<Pol, ST>(ctx);
        while (tpl > 1 && engine_fixed_smem() + Pol::x_bytes((int)n, tpl) + 1024 > limit) --tpl;
        for (int t0 = 0; t0 < (int)ntok; t0 += tpl) {
            GemvParams q = p;
            q.ntok = min(tpl, (int)ntok - t0);
            q.xint = (q.bits == 4 && q.ntok == 1 && xint_enabled(true)) ? 1 : 0;
            q.x = p.x + (size_t)t0 * xrs;
            q.y = p.y + (size_t)t0 * yrs;
            // one token on the integer path: a helper warp per stage
            // (TFCUDA_HELPERS=0 turns it off; read per call)
            tf_status rc = (q.xint && q.aligned && helpers_enabled())
                               ? launch_engine<Pol, ST, 1>(ctx, q, Pol::x_bytes((int)n, q.ntok), sj, cs, name)
                               : launch_engine<Pol, ST>(ctx, q, Pol::x_bytes((int)n, q.ntok), sj, cs, name);
            if (rc) return rc;
        }
        return TF_OK;
    });
}

}  // namespace

extern "C" {

const char* tf_status_string(tf_status s) {
    switch (s) {
    case TF_OK: return "ok";
    case TF_ERR_INVALID_ARG: return "invalid argument";
    case TF_ERR_MISALIGNED: return "misaligned pointer";
    case TF_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case TF_ERR_CUDA: return "CUDA error";
    case TF_ERR_NCCL: return "NCCL error";
    case TF_ERR_TIMEOUT: return "device wait timed out";
    case TF_ERR_NO_DEVICE: return "no usable sm_100 device";
    case TF_ERR_GROUPING: return "route grouping rejected";
    }
    return "unknown status";
}

void tf_version(int* major, int* minor) {
    if (major) *major = TFCUDA_VERSION_MAJOR;
    if (minor) *minor = TFCUDA_VERSION_MINOR;
}

tf_status tf_context_create(int device, tf_context** out) {
    if (!out) return TF_ERR_INVALID_ARG;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) return TF_ERR_NO_DEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return TF_ERR_NO_DEVICE;
    if (prop.major < 10) return TF_ERR_NO_DEVICE;  // built for sm_100a only
    if (cudaSetDevice(device) != cudaSuccess) return TF_ERR_CUDA;
    tf_context* ctx = new tf_context();
    ctx->device = device;
    ctx->num_sms = prop.multiProcessorCount;
    ctx->max_smem_optin = prop.sharedMemPerBlockOptin;
    cudaError_t e = cudaSuccess;
    e = e ? e : cudaMalloc(&ctx->d_err, 4 * sizeof(uint32_t));
    e = e ? e : cudaMalloc(&ctx->d_logits, sizeof(float) * kMaxRouterExperts * 64);
    e = e ? e : cudaMalloc(&ctx->d_rt_logits, sizeof(float) * kRtLogitsCap);
    e = e ? e : cudaMalloc(&ctx->d_qmm_part, sizeof(float) * kQmmPartCap);
    e = e ? e : cudaMalloc(&ctx->d_ticket, sizeof(unsigned int) * 64);
    e = e ? e : cudaMalloc(&ctx->d_flags, sizeof(unsigned int) * 32 * 1024);
    e = e ? e : cudaMalloc(&ctx->d_idx, sizeof(uint32_t) * kMaxTopKDecode);
    e = e ? e : cudaMalloc(&ctx->d_w, sizeof(__half) * kMaxTopKDecode);
    e = e ? e : cudaMalloc(&ctx->d_acts, sizeof(__half) * kMaxTopKDecode * kMaxF);
    e = e ? e : cudaMalloc(&ctx->d_shared_act, sizeof(__half) * kMaxFs);
    e = e ? e : cudaMalloc(&ctx->d_sort_cnt, sizeof(uint32_t) * kRouteSortChunks * 256);
    e = e ? e : cudaMalloc(&ctx->d_lm_keys, sizeof(unsigned long long) * kMaxLmTokens);
    e = e ? e : cudaMalloc(&ctx->d_lm_tickets, sizeof(unsigned int) * kMaxLmTokens);
    e = e ? e : cudaMemset(ctx->d_lm_keys, 0, sizeof(unsigned long long) * kMaxLmTokens);
    e = e ? e : cudaMalloc(&ctx->d_smx, sizeof(float) * kMaxLmTokens * 128 * 2);
    e = e ? e : cudaMalloc(&ctx->d_cand_v, sizeof(float) * 2 * kCandCap);
    e = e ? e : cudaMalloc(&ctx->d_cand_i, sizeof(uint32_t) * 2 * kCandCap);
    e = e ? e : cudaMemset(ctx->d_lm_tickets, 0, sizeof(unsigned int) * kMaxLmTokens);
    e = e ? e : cudaMemset(ctx->d_err, 0, 4 * sizeof(uint32_t));
    e = e ? e : cudaMemset(ctx->d_ticket, 0, sizeof(unsigned int) * 64);
    e = e ? e : cudaMemset(ctx->d_flags, 0, sizeof(unsigned int) * 32 * 1024);
    e = e ? e : cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        tf_context_destroy(ctx);
        return TF_ERR_CUDA;
    }
    *out = ctx;
    return TF_OK;
}

void tf_context_destroy(tf_context* ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaFree(ctx->d_err);
    cudaFree(ctx->d_logits);
    cudaFree(ctx->d_rt_logits);
    cudaFree(ctx->d_qmm_part);
    cudaFree(ctx->d_ticket);
    cudaFree(ctx->d_flags);
    cudaFree(ctx->d_idx);
    cudaFree(ctx->d_w);
    cudaFree(ctx->d_acts);
    cudaFree(ctx->d_shared_act);
    cudaFree(ctx->d_sort_cnt);
    cudaFree(ctx->d_lm_keys);
    cudaFree(ctx->d_lm_tickets);
    cudaFree(ctx->d_smx);
    cudaFree(ctx->d_cand_v);
    cudaFree(ctx->d_cand_i);
    delete ctx;
}

const char* tf_context_last_error(const tf_context* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

tf_status tf_context_check_device(tf_context* ctx, void* stream, uint32_t* flags_out) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    uint32_t words[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemcpyAsync(words, ctx->d_err, sizeof(words), cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cs);
    if (e == cudaSuccess) e = cudaMemsetAsync(ctx->d_err, 0, sizeof(words), cs);
    const uint32_t flags = words[0];
    if (e == cudaSuccess) e = cudaStreamSynchronize(cs);
    if (e != cudaSuccess) return cuda_check(ctx, e, "tf_context_check_device");
    if (flags_out) *flags_out = flags;
    if (flags & kErrMbarTimeout)
        return fail(ctx, TF_ERR_TIMEOUT, "a bounded device wait gave up (flags=0x%x, site %u, info 0x%08x)", flags,
                    words[1], words[2]);
    if (flags & kErrBadExpert) return fail(ctx, TF_ERR_INVALID_ARG, "an expert id was out of range (flags=0x%x)", flags);
    if (flags & kErrAlign)
        return fail(ctx, TF_ERR_MISALIGNED, "misaligned access skipped at site %u, address 0x%08x%08x", words[1],
                    words[3], words[2]);
    return TF_OK;
}

tf_status tf_int4_gemv(tf_context* ctx, const void* W, const void* S, const void* B, const void* x, void* y,
                       uint32_t m, uint32_t n, tf_scale_type st, void* stream) {
    return gemv_common(ctx, 4, W, S, B, 0, 0, 1, x, 1, n, y, m, 0, m, n, st, stream, "tf_int4_gemv");
}

tf_status tf_int8_gemv(tf_context* ctx, const void* W, const void* S, const void* B, const void* x, void* y,
                       uint32_t m, uint32_t n, tf_scale_type st, void* stream) {
    return gemv_common(ctx, 8, W, S, B, 0, 0, 1, x, 1, n, y, m, 0, m, n, st, stream, "tf_int8_gemv");
}

tf_status tf_affine_gemv_batched(tf_context* ctx, uint32_t bits, const void* W, const void* S, const void* B,
                                 uint64_t wbs, uint64_t sbs, uint32_t batch, const void* x, uint32_t ntok,
                                 uint32_t xrs, void* y, uint32_t yrs, uint64_t ybs, uint32_t m, uint32_t n,
                                 tf_scale_type st, void* stream) {
    return gemv_common(ctx, bits, W, S, B, wbs, sbs, batch, x, ntok, xrs, y, yrs, ybs, m, n, st, stream,
                       "tf_affine_gemv_batched");
}

// Router launch shared by tf_router_topk and the fused layer.
static tf_status router_launch(tf_context* ctx, const void* W, const void* S, const void* B, const void* hidden,
                               const void* es, const void* pes, void* out_idx, void* out_w, uint32_t E, uint32_t d,
                               uint32_t top_k, tf_scale_type st, cudaStream_t cs,
                               RouterParams* build_only = nullptr, float* out_logits = nullptr) {
    const char* name = "tf_router_topk";
    if (!W || !S || !B || !hidden || !es || !pes || !out_idx || !out_w) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return fail(ctx, TF_ERR_INVALID_ARG, "%s: unknown scale type", name);
    if (d == 0 || d % 64) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d must be a positive multiple of 64", name);
    if (E == 0 || E > (uint32_t)kMaxRouterExperts) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: num_experts must be in 1..256", name);
    if (top_k == 0 || top_k > 32 || top_k > E) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: top_k must be in 1..min(32, num_experts)", name);
    if (!aligned2(W) || !aligned2(S) || !aligned2(B) || !aligned2(hidden) || !aligned2(es) || !aligned2(pes) ||
        (reinterpret_cast<uintptr_t>(out_idx) & 3u))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: misaligned buffer", name);
    RouterParams p;
    memset(&p, 0, sizeof(p));
    p.W = static_cast<const uint8_t*>(W);
    p.S = S;
    p.B = B;
    p.hidden = static_cast<const __half*>(hidden);
    p.eff_scale = static_cast<const __nv_bfloat16*>(es);
    p.per_expert_scale = static_cast<const __nv_bfloat16*>(pes);
    p.E = (int)E;
    p.D = (int)d;
    p.top_k = (int)top_k;
    p.logits = ctx->d_logits;
    p.out_logits = out_logits;
    p.ticket = ctx->d_ticket;
    p.out_idx = static_cast<uint32_t*>(out_idx);
    p.out_w = static_cast<__half*>(out_w);
    p.aligned = make_weight_map(&p.map, W, d, E, 1, 0);
    p.err = ctx->d_err;
    p.sched = make_sched(((int)E + 15) / 16, units_for_K((int)d, 8), 0, 1, ctx->num_sms);
    const int sj = p.sched.S_total;
    if (build_only) {
        *build_only = p;
        return TF_OK;
    }
    return dispatch_scale(st, [&](auto tag) {
        using ST = decltype(tag);
        return launch_engine<RouterPolicy<ST>, ST>(ctx, p, RouterPolicy<ST>::x_bytes((int)d), sj, cs, name);
    });
}

tf_status tf_router_topk(tf_context* ctx, const void* W, const void* S, const void* B, const void* hidden,
                         const void* es, const void* pes, void* out_idx, void* out_w, uint32_t E, uint32_t d,
                         uint32_t top_k, tf_scale_type st, void* stream) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    return router_launch(ctx, W, S, B, hidden, es, pes, out_idx, out_w, E, d, top_k, st,
                         static_cast<cudaStream_t>(stream));
}

tf_status tf_router_topk_with_logits(tf_context* ctx, const void* W, const void* S, const void* B,
                                     const void* hidden, const void* es, const void* pes, void* out_idx, void* out_w,
                                     void* out_logits, uint32_t E, uint32_t d, uint32_t top_k, tf_scale_type st,
                                     void* stream) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    if (!out_logits) return fail(ctx, TF_ERR_INVALID_ARG, "tf_router_topk_with_logits: null out_logits");
    if (reinterpret_cast<uintptr_t>(out_logits) & 3u)
        return fail(ctx, TF_ERR_MISALIGNED, "tf_router_topk_with_logits: out_logits must be 4-byte aligned");
    return router_launch(ctx, W, S, B, hidden, es, pes, out_idx, out_w, E, d, top_k, st,
                         static_cast<cudaStream_t>(stream), nullptr, static_cast<float*>(out_logits));
}

static tf_status phase1_launch(tf_context* ctx, const ExpertSource& src, const void* x, void* acts, uint32_t d,
                               uint32_t f, uint32_t top_k, const tf_affine_matrix* sg, const tf_affine_matrix* su,
                               void* shared_act, tf_scale_type st, cudaStream_t cs, const char* name,
                               Phase1Params* build_only = nullptr, bool lazy_ids = false) {
    if (!x || (!acts && top_k)) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null activation pointer", name);
    if (d == 0 || d % 64 || f == 0 || f % 64) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d and f must be positive multiples of 64", name);
    if (f > (uint32_t)kMaxF * 4) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: f too large", name);
    Phase1Params p;
    memset(&p, 0, sizeof(p));
    p.src = src;
    p.D = (int)d;
    p.F = (int)f;
    p.top_k = (int)top_k;
    p.x = static_cast<const __half*>(x);
    p.acts = static_cast<__half*>(acts);
    bool aligned = true;
    if (top_k) {
        aligned = source_maps(src, top_k, src.off[0], d / 2, f, &p.map[0]) &&
                  source_maps(src, top_k, src.off[3], d / 2, f, &p.map[8]);
    }
    if (sg) {
        p.has_shared = 1;
        p.shared_bits = (int)sg->bits;
        p.Fs = (int)sg->rows;
        p.sg = AffineMat{static_cast<const uint8_t*>(sg->weights), sg->scales, sg->biases};
        p.su = AffineMat{static_cast<const uint8_t*>(su->weights), su->scales, su->biases};
        p.shared_act = static_cast<__half*>(shared_act);
        const uint64_t rb = row_bytes((int)d, (int)sg->bits);
        aligned = make_weight_map(&p.map[16], sg->weights, rb, sg->rows, 1, 0) &&
                  make_weight_map(&p.map[17], su->weights, rb, su->rows, 1, 0) && aligned;
    }
    p.aligned = aligned;
    p.x_aligned = aligned16(x);
    p.err = ctx->d_err;
    p.fjobs = (int)f / 8;
    p.lazy_ids = (lazy_ids && sg && top_k && src.ids != nullptr && !src.ids_in_smem) ? 1 : 0;
    p.xint = ((!sg || sg->bits == 4) && xint_enabled(true)) ? 1 : 0;
    if (p.lazy_ids)  // shared jobs first: they need no routing
        p.sched = make_sched((int)sg->rows / 8, units_for_K((int)d, (int)sg->bits), (int)top_k * p.fjobs,
                             units_for_K((int)d, 4), ctx->num_sms);
    else
        p.sched = make_sched((int)top_k * p.fjobs, units_for_K((int)d, 4), sg ? (int)sg->rows / 8 : 0,
                             sg ? units_for_K((int)d, (int)sg->bits) : 1, ctx->num_sms);
    const int sj = p.sched.S_total;
    if (build_only) {
        *build_only = p;
        return TF_OK;
    }
    return dispatch_scale(st, [&](auto tag) {
        using ST = decltype(tag);
        // integer path: a helper warp per stage halves each unit's latency
        const size_t xb1 = Phase1Policy<ST>::x_bytes((int)d);
        if (p.xint && p.aligned && helpers_enabled() &&
            engine_fixed_smem(1) + xb1 + 1024 <= engine_smem_limit<Phase1Policy<ST>, ST, 1>(ctx))
            return launch_engine<Phase1Policy<ST>, ST, 1>(ctx, p, xb1, sj, cs, name);
        return launch_engine<Phase1Policy<ST>, ST>(ctx, p, Phase1Policy<ST>::x_bytes((int)d), sj, cs, name);
    });
}

static tf_status phase2_launch(tf_context* ctx, const ExpertSource& src, const void* acts, const void* rw,
                               const void* residual, void* y, uint32_t d, uint32_t f, uint32_t top_k,
                               const tf_affine_matrix* sdn, const void* shared_act, tf_scale_type st, cudaStream_t cs,
                               const char* name, Phase2Params* build_only = nullptr) {
    if (!y || (top_k && (!acts || !rw))) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (d == 0 || d % 64 || f == 0 || f % 64) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d and f must be positive multiples of 64", name);
    if (acts && !aligned16(acts)) return fail(ctx, TF_ERR_MISALIGNED, "%s: acts must be 16-byte aligned", name);
    if (f % 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: f", name);
    Phase2Params p;
    memset(&p, 0, sizeof(p));
    p.src = src;
    p.D = (int)d;
    p.F = (int)f;
    p.top_k = (int)top_k;
    p.acts = static_cast<const __half*>(acts);
    p.routing_w = static_cast<const __half*>(rw);
    p.residual = static_cast<const __half*>(residual);
    p.y = static_cast<__half*>(y);
    bool aligned = top_k ? source_maps(src, top_k, src.off[6], f / 2, d, &p.map[0]) : true;
    size_t xb;
    if (sdn) {
        p.has_shared = 1;
        p.shared_bits = (int)sdn->bits;
        p.Fs = (int)sdn->cols;
        p.sd = AffineMat{static_cast<const uint8_t*>(sdn->weights), sdn->scales, sdn->biases};
        p.shared_act = static_cast<const __half*>(shared_act);
        aligned = make_weight_map(&p.map[8], sdn->weights, row_bytes((int)sdn->cols, (int)sdn->bits), sdn->rows, 1, 0) &&
                  aligned;
        if (!aligned16(shared_act)) return fail(ctx, TF_ERR_MISALIGNED, "%s: shared act must be 16-byte aligned", name);
    }
    p.aligned = aligned;
    p.xint = ((!sdn || sdn->bits == 4) && xint_enabled(true)) ? 1 : 0;
    p.err = ctx->d_err;
    const int U = (int)top_k * units_for_K((int)f, 4) + (sdn ? units_for_K((int)sdn->cols, (int)sdn->bits) : 0);
    p.upf = units_for_K((int)f, 4);
    p.sched = make_sched(((int)d + 15) / 16, U, 0, 1, ctx->num_sms);
    const int sj = p.sched.S_total;
    if (build_only) {
        *build_only = p;
        return TF_OK;
    }
    return dispatch_scale(st, [&](auto tag) {
        using ST = decltype(tag);
        xb = Phase2Policy<ST>::x_bytes((int)top_k, (int)f, sdn ? (int)sdn->cols : 0);
        // (when the activations still fit beside the helpers' larger reduction area)
        if (p.xint && p.aligned && helpers_enabled() &&
            engine_fixed_smem(1) + xb + 1024 <= engine_smem_limit<Phase2Policy<ST>, ST, 1>(ctx))
            return launch_engine<Phase2Policy<ST>, ST, 1>(ctx, p, xb, sj, cs, name);
        return launch_engine<Phase2Policy<ST>, ST>(ctx, p, xb, sj, cs, name);
    });
}

tf_status tf_moe_phase1(tf_context* ctx, const void* pool, uint64_t stride, uint32_t E, const void* ids,
                        const void* const* blobs, const tf_expert_offsets* off, const void* x, void* acts, uint32_t d,
                        uint32_t f, uint32_t top_k, tf_scale_type st, void* stream) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    s = check_source(ctx, pool, ids, blobs, off, E, top_k, "tf_moe_phase1");
    if (s) return s;
    ExpertSource src = make_source(pool, stride, E, ids, blobs, off, top_k);
    return phase1_launch(ctx, src, x, acts, d, f, top_k, nullptr, nullptr, nullptr, st,
                         static_cast<cudaStream_t>(stream), "tf_moe_phase1");
}

tf_status tf_moe_phase2(tf_context* ctx, const void* pool, uint64_t stride, uint32_t E, const void* ids,
                        const void* const* blobs, const tf_expert_offsets* off, const void* acts, const void* rw,
                        const void* residual, void* y, uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st,
                        void* stream) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    s = check_source(ctx, pool, ids, blobs, off, E, top_k, "tf_moe_phase2");
    if (s) return s;
    ExpertSource src = make_source(pool, stride, E, ids, blobs, off, top_k);
    return phase2_launch(ctx, src, acts, rw, residual, y, d, f, top_k, nullptr, nullptr, st,
                         static_cast<cudaStream_t>(stream), "tf_moe_phase2");
}

static tf_status check_shared(tf_context* ctx, const tf_affine_matrix* g, const tf_affine_matrix* u,
                              const tf_affine_matrix* dn, const char* name) {
    if (!g || !u || !dn) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null projection", name);
    if (g->rows != u->rows || g->cols != u->cols || dn->rows != g->cols || dn->cols != g->rows)
        return fail(ctx, TF_ERR_INVALID_ARG, "SharedExpert dimension mismatch: gate=(%u,%u) up=(%u,%u) down=(%u,%u)",
                    g->rows, g->cols, u->rows, u->cols, dn->rows, dn->cols);
    if (g->bits != u->bits || g->bits != dn->bits || (g->bits != 4 && g->bits != 8))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "SharedExpert unsupported weight bits: %u", g->bits);
    if (g->cols % 64 || g->rows % 64) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: dims must be multiples of 64", name);
    if (g->rows > (uint32_t)kMaxFs) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: intermediate too large", name);
    const tf_affine_matrix* m[3] = {g, u, dn};
    for (int i = 0; i < 3; ++i) {
        if (!m[i]->weights || !m[i]->scales || !m[i]->biases) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null weights", name);
        if (!aligned16(m[i]->weights)) return fail(ctx, TF_ERR_MISALIGNED, "%s: shared weights must be 16-byte aligned", name);
    }
    return TF_OK;
}

tf_status tf_shared_expert(tf_context* ctx, const void* x, const tf_affine_matrix* g, const tf_affine_matrix* u,
                           const tf_affine_matrix* dn, void* y, void* scratch_act, tf_scale_type st, void* stream) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    s = check_shared(ctx, g, u, dn, "tf_shared_expert");
    if (s) return s;
    if (!x || !y || !scratch_act) return fail(ctx, TF_ERR_INVALID_ARG, "tf_shared_expert: null pointer");
    if (!aligned16(scratch_act)) return fail(ctx, TF_ERR_MISALIGNED, "tf_shared_expert: scratch must be 16-byte aligned");
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    ExpertSource none;
    memset(&none, 0, sizeof(none));
    s = phase1_launch(ctx, none, x, nullptr, g->cols, 64, 0, g, u, scratch_act, st, cs, "tf_shared_expert");
    if (s) return s;
    return phase2_launch(ctx, none, nullptr, nullptr, nullptr, y, dn->rows, 64, 0, dn, scratch_act, st, cs,
                         "tf_shared_expert");
}

// Fused single-launch layer (tf_fused.cuh).  Builds the four phase
// parameter blocks with the same builders as the separate entry points.
static tf_status decode_layer_fused(tf_context* ctx, const tf_moe_layer* L, const void* router_x, const void* x,
                                    const void* residual, void* y, uint32_t* idx, __half* w, cudaStream_t cs) {
    const char* name = "tf_moe_decode_layer";
    const bool shared = L->shared_gate.rows != 0;
    LayerParams lp;
    memset(&lp, 0, sizeof(lp));
    tf_status s = router_launch(ctx, L->router_w, L->router_s, L->router_b, router_x, L->eff_scale,
                                L->per_expert_scale, idx, w, L->num_experts, L->d, L->top_k, L->scale_type, cs, &lp.r);
    if (s) return s;
    lp.r.fused = 1;
    lp.r.replicas = 16;  // d_logits holds 64 x 256 floats
    ExpertSource none;
    memset(&none, 0, sizeof(none));
    if (shared) {
        s = phase1_launch(ctx, none, x, nullptr, L->d, 64, 0, &L->shared_gate, &L->shared_up, ctx->d_shared_act,
                          L->scale_type, cs, name, &lp.sh);
        if (s) return s;
    }
    ExpertSource src = make_source(L->expert_pool, L->expert_stride, L->num_experts, idx, nullptr, &L->offsets, L->top_k);
    src.ids_in_smem = 1;
    s = phase1_launch(ctx, src, x, ctx->d_acts, L->d, L->f, L->top_k, nullptr, nullptr, nullptr, L->scale_type, cs,
                      name, &lp.p1);
    if (s) return s;
    s = phase2_launch(ctx, src, ctx->d_acts, w, residual, y, L->d, L->f, L->top_k, shared ? &L->shared_down : nullptr,
                      ctx->d_shared_act, L->scale_type, cs, name, &lp.p2);
    if (s) return s;
    lp.p2.rw_in_smem = 1;
    lp.has_shared = shared ? 1 : 0;
    lp.bar_count = ctx->d_ticket + 1;
    lp.bar_flags = ctx->d_flags;
    lp.out_idx = idx;
    lp.out_w = w;
    lp.err = ctx->d_err;
    return dispatch_scale(L->scale_type, [&](auto tag) -> tf_status {
        using ST = decltype(tag);
        size_t xb = RouterPolicy<ST>::x_bytes((int)L->d);
        xb = std::max(xb, Phase1Policy<ST>::x_bytes((int)L->d));
        xb = std::max(xb, Phase2Policy<ST>::x_bytes((int)L->top_k, (int)L->f, shared ? (int)L->shared_down.cols : 0));
        const size_t smem = engine_fixed_smem() + xb + 1024;
        static size_t static_smem = (size_t)-1;
        if (static_smem == (size_t)-1) {
            cudaFuncAttributes fa;
            cudaError_t e = cudaFuncGetAttributes(&fa, fused_layer_kernel<ST>);
            if (e != cudaSuccess) return cuda_check(ctx, e, name);
            static_smem = fa.sharedSizeBytes;
        }
        const size_t limit = ctx->max_smem_optin - static_smem;
        if (smem > limit) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: activations too large for shared memory", name);
        static bool configured[64] = {};
        if (!configured[ctx->device & 63]) {
            cudaError_t e = cudaFuncSetAttribute(fused_layer_kernel<ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)limit);
            if (e != cudaSuccess) return cuda_check(ctx, e, name);
            configured[ctx->device & 63] = true;
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)ctx->num_sms);
        cfg.blockDim = dim3(kWarps * 32);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = cs;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs co-resident: the grid barrier is safe
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cuda_check(ctx, cudaLaunchKernelEx(&cfg, fused_layer_kernel<ST>, lp), name);
    });
}

tf_status tf_moe_decode_layer(tf_context* ctx, const tf_moe_layer* L, const void* router_x, const void* x,
                              const void* residual, void* y, void* out_idx, void* out_w, void* stream) {
    tf_status s = check_ctx(ctx);
    if (s) return s;
    if (!L || !router_x || !x || !y) return fail(ctx, TF_ERR_INVALID_ARG, "tf_moe_decode_layer: null pointer");
    if (L->top_k == 0 || L->top_k > (uint32_t)kMaxTopKDecode)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "tf_moe_decode_layer: top_k must be in 1..8");
    if (L->f > (uint32_t)kMaxF) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "tf_moe_decode_layer: f too large");
    const bool shared = L->shared_gate.rows != 0;
    if (shared) {
        s = check_shared(ctx, &L->shared_gate, &L->shared_up, &L->shared_down, "tf_moe_decode_layer");
        if (s) return s;
        if (L->shared_gate.cols != L->d) return fail(ctx, TF_ERR_INVALID_ARG, "tf_moe_decode_layer: shared expert input dim != d");
    }
    s = check_source(ctx, L->expert_pool, ctx->d_idx, nullptr, &L->offsets, L->num_experts, L->top_k, "tf_moe_decode_layer");
    if (s) return s;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    uint32_t* idx = out_idx ? static_cast<uint32_t*>(out_idx) : ctx->d_idx;
    __half* w = out_w ? static_cast<__half*>(out_w) : ctx->d_w;
    // Three launches (router, phase 1, phase 2) by default: measured faster on
    // B200 than the single cooperative launch, which TFCUDA_FUSED=1 selects
    // (same arithmetic; read per call so one process can run both).
    const char* fz = getenv("TFCUDA_FUSED");
    if (fz && fz[0] == '1') return decode_layer_fused(ctx, L, router_x, x, residual, y, idx, w, cs);
    s = router_launch(ctx, L->router_w, L->router_s, L->router_b, router_x, L->eff_scale, L->per_expert_scale, idx, w,
                      L->num_experts, L->d, L->top_k, L->scale_type, cs);
    if (s) return s;
    ExpertSource src = make_source(L->expert_pool, L->expert_stride, L->num_experts, idx, nullptr, &L->offsets, L->top_k);
    s = phase1_launch(ctx, src, x, ctx->d_acts, L->d, L->f, L->top_k, shared ? &L->shared_gate : nullptr,
                      shared ? &L->shared_up : nullptr, ctx->d_shared_act, L->scale_type, cs, "tf_moe_decode_layer/phase1",
                      nullptr, /*lazy_ids=*/true);
    if (s) return s;
    return phase2_launch(ctx, src, ctx->d_acts, w, residual, y, L->d, L->f, L->top_k,
                         shared ? &L->shared_down : nullptr, ctx->d_shared_act, L->scale_type, cs,
                         "tf_moe_decode_layer/phase2");
}

}  // extern "C"

#ifdef TF_TRACE
extern "C" TF_API int tf_debug_trace(unsigned long long* out, int n) {
    return (int)cudaMemcpyFromSymbol(out, tf::g_tf_trace, sizeof(unsigned long long) * 16 * n);
}
#endif
