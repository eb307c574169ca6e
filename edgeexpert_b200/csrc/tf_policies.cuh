// tf_policies.cuh -- job/unit/epilogue policies for the streaming engine.
// Each policy maps the reference operator's output rows onto 16-row jobs.
//
// Policy interface:
//   Params                      kernel parameters; carry `Sched sched`,
//                               `aligned`, `err`
//   stage_pre(p, tid)           tiny per-CTA set-up needed to issue copies
//   stage_x(p, xa, tid, nt)     stage activations (all threads; may barrier)
//   unit(p, job, u, &sd, &c)    describe unit u of job (weights, rows, x)
//   epilogue(p, job, f, lane)   one warp writes the job's reduced outputs
#pragma once
#include "tf_engine.cuh"

namespace tf {

// (a CTA wider than kWarps warps carries helper warps and a larger reduction area)
__device__ __forceinline__ const uint8_t* engine_xarea() {
    return engine_smem_base() + engine_fixed_smem(blockDim.x > kWarps * 32 ? 1 : 0);
}

// ===========================================================================
// Plain affine GEMV, Y[tok][row] = sum_k W[row][k] * X[tok][k]
// (dequant_int4_gemv_simd / dequant_int8_gemv_simd; a batch of matrices with
// a common activation block of up to 8 tokens).
// ===========================================================================
struct GemvParams {
    CUtensorMap map;  // W as [batch][M][row_bytes], box 8 rows x 128 B
    const uint8_t* W;
    const void* S;
    const void* B;
    long long w_bstride;   // bytes between matrices
    long long sb_bstride;  // elements between scale blocks
    int M, K, batch, bits, tiles;
    const __half* x;
    int x_row_stride;  // elements between tokens
    int ntok;
    __half* y;
    int y_row_stride;     // elements between tokens of y
    long long y_bstride;  // elements between matrices of y
    int aligned, x_aligned;
    int xint;  // batch-1 int4: activation staged for the integer tensor path
    uint32_t* err;
    Sched sched;
};

template <typename ST>
struct GemvPolicy {
    using Params = GemvParams;
    static constexpr bool kWeightsIndependent = true;
    // engine hooks: schedule from the host Sched, activations staged once per CTA
    static constexpr bool kStagePerSuperjob = false;
    __device__ static int superjobs(const Params& p) { return p.sched.S_total; }
    __device__ static SuperJob superjob(const Params& p, int sjx) { return decode_superjob(p.sched, sjx); }
    __device__ static void stage_x_sj(const Params&, const SuperJob&, uint8_t*, int, int) {}
    __device__ static bool lazy(const Params&) { return false; }
    // [ntok][ws] words, [ntok][K/64] sums, [ntok][K/64] folded-offset corrections
    static size_t x_bytes(int K, int ntok) {
        return (size_t)ntok * x_words_stride(K) * 4 + 2 * (size_t)ntok * (K / kGroup) * 4;
    }
    __device__ static void stage_pre(const Params& p, int tid) {
        if (tid == 0 && p.aligned) prefetch_tmap(&p.map);
    }
    __device__ static void stage_x(const Params& p, uint8_t* xa, int tid, int nt) {
        uint32_t* xs = reinterpret_cast<uint32_t*>(xa);
        float* xsum = reinterpret_cast<float*>(xs + p.ntok * x_words_stride(p.K));
        float* xcorr = xsum + p.ntok * (p.K / kGroup);
        if (p.xint) {
            stage_x_int(p.x, p.K, xs, xsum, xcorr, tid, nt);
            return;
        }
        const bool fold = p.ntok == 1;
        stage_words(p.x, p.x_row_stride, p.ntok, p.K, xs, p.x_aligned, fold, tid, nt);
        __syncthreads();
        stage_xsum_smem(xs, x_words_stride(p.K), p.ntok, p.K, xsum, xcorr, fold, tid, nt);
    }
    __device__ static bool unit(const Params& p, int job, int u, SegDesc* d, int* chunk) {
        const int b = job / p.tiles, tile = job - b * p.tiles;
        const uint8_t* W = p.W + (size_t)b * p.w_bstride;
        const ST* S = reinterpret_cast<const ST*>(p.S) + (size_t)b * p.sb_bstride;
        const ST* B = reinterpret_cast<const ST*>(p.B) + (size_t)b * p.sb_bstride;
        d->WA = d->WB = W;
        d->mapA = d->mapB = &p.map;
        d->eA = d->eB = b;
        d->SA = d->SB = S;
        d->BA = d->BB = B;
        d->rowA = tile * 16;
        d->nA = max(0, min(8, p.M - d->rowA));
        d->rowB = d->rowA + 8;
        d->nB = max(0, min(8, p.M - d->rowB));
        d->K = p.K;
        d->bits = p.bits;
        const uint32_t* xs = reinterpret_cast<const uint32_t*>(engine_xarea());
        d->xs = xs;
        d->xsum = reinterpret_cast<const float*>(xs + p.ntok * x_words_stride(p.K));
        d->xcorr = d->xsum + p.ntok * (p.K / kGroup);
        d->xfold = p.xint ? 2 : (p.ntok == 1 ? 1 : 0);
        d->xws = x_words_stride(p.K);
        d->ntok = p.ntok;
        d->mult = 1.0f;
        *chunk = u;
        return true;
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int b = job / p.tiles, tile = job - b * p.tiles;
        const int g = lane >> 2, t = lane & 3;
        __half* y = p.y + (size_t)b * p.y_bstride;
        const int r0 = tile * 16 + g, r1 = r0 + 8;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int tok = 2 * t + j;
            if (tok >= p.ntok) continue;
            if (r0 < p.M) y[(size_t)tok * p.y_row_stride + r0] = __float2half_rn(f[j]);
            if (r1 < p.M) y[(size_t)tok * p.y_row_stride + r1] = __float2half_rn(f[2 + j]);
        }
    }
};

// ===========================================================================
// Expert source: HBM-resident pool indexed by device-side expert ids, or
// explicit per-slot blob pointers (the reference's RoutedBlobs, moe.metal:74-76).
// Offsets follow MoEExpertOffsets (MoE.swift:4-29).
// ===========================================================================
struct ExpertSource {
    const uint8_t* pool;
    unsigned long long stride;
    const uint32_t* ids;  // [top_k] expert ids (device); nullptr => use blobs
    int num_experts;
    const uint8_t* blobs[8];
    uint32_t off[9];  // gate_w gate_s gate_b up_w up_s up_b down_w down_s down_b
    int ids_in_smem;  // fused layer: ids already selected into ids_smem()
};

// Device expert ids are copied into shared memory once per CTA (stage_ids)
// so no bulk copy waits on a global load of its expert id.
__device__ __forceinline__ uint32_t* ids_smem() {
    __shared__ uint32_t ids[8];
    return ids;
}

// Routing weights of the fused layer, selected per CTA into shared memory.
__device__ __forceinline__ __half* rw_smem() {
    __shared__ __half rw[8];
    return rw;
}

__device__ __forceinline__ void stage_ids(const ExpertSource& es, int top_k, int tid) {
    if (es.ids != nullptr && !es.ids_in_smem && tid < top_k) ids_smem()[tid] = __ldg(es.ids + tid);
}

__device__ __forceinline__ const uint8_t* expert_blob(const ExpertSource& es, int slot, uint32_t* err) {
    if (es.ids == nullptr) return es.blobs[slot];
    const uint32_t e = ids_smem()[slot];
    if (e >= (uint32_t)es.num_experts) {
        if (err) atomicOr(err, kErrBadExpert);
        return nullptr;
    }
    return es.pool + (size_t)e * es.stride;
}

// Affine matrix handle for the shared expert (SharedExpertProjection,
// SharedExpertInt8.swift:9-31).
struct AffineMat {
    const uint8_t* W;
    const void* S;
    const void* B;
};

// ===========================================================================
// Decode MoE phase 1: routed gate/up/GELU for top_k experts
// (moe_phase1_gate_up_act_u16load, moe.metal:248-369) and, in the same
// launch, the shared expert gate/up/GELU (SharedExpertInt4.swift:60-85 /
// shared_int8_gate_up_act_simd, dequant_int8.metal:99-154).
// Job = 8 f-rows: stage rows 0-7 = gate rows, 8-15 = up rows of the same f,
// so one thread ends up holding gate and up of one output.
// ===========================================================================
struct Phase1Params {
    // pool mode: map[0] gate_w / map[8] up_w of all experts ([E][F][D/2]);
    // blob mode: map[slot] / map[8 + slot]; shared expert: map[16] / map[17].
    CUtensorMap map[18];
    ExpertSource src;
    int D, F, top_k, fjobs;  // fjobs = F / 8
    const __half* x;
    __half* acts;  // [top_k][F]
    int has_shared, shared_bits, Fs;
    AffineMat sg, su;
    __half* shared_act;  // [Fs]
    int aligned, x_aligned;
    // Decode layer only (its predecessor is the router): the shared expert's
    // jobs come first and start before the router has finished; a routed
    // unit waits for it (griddepcontrol.wait) and reads its expert id then;
    // epilogues write only after the wait.
    int lazy_ids;
    int xint;  // every consumer is int4: x staged for the integer tensor path
    uint32_t* err;
    Sched sched;
};

template <typename ST>
struct Phase1Policy {
    using Params = Phase1Params;
    static constexpr bool kWeightsIndependent = false;
    // engine hooks: schedule from the host Sched, activations staged once per CTA
    static constexpr bool kStagePerSuperjob = false;
    __device__ static int superjobs(const Params& p) { return p.sched.S_total; }
    __device__ static SuperJob superjob(const Params& p, int sjx) { return decode_superjob(p.sched, sjx); }
    __device__ static void stage_x_sj(const Params&, const SuperJob&, uint8_t*, int, int) {}
    __device__ static bool lazy(const Params& p) { return p.lazy_ids != 0; }
    static size_t x_bytes(int D) { return (size_t)x_words_stride(D) * 4 + 2 * (size_t)(D / kGroup) * 4; }
    // job -> routed job (>= 0) or shared job (>= 0); shared jobs first in lazy mode
    __device__ static void split(const Params& p, int job, int* rj, int* sj) {
        const int rjobs = p.top_k * p.fjobs;
        if (p.lazy_ids) {
            const int sjobs = p.has_shared ? p.Fs / 8 : 0;
            *sj = job < sjobs ? job : -1;
            *rj = job < sjobs ? -1 : job - sjobs;
        } else {
            *rj = job < rjobs ? job : -1;
            *sj = job < rjobs ? -1 : job - rjobs;
        }
    }
    __device__ static void stage_pre(const Params& p, int tid) {
        if (!p.lazy_ids) stage_ids(p.src, p.top_k, tid);
        if (!p.aligned) return;
        const bool pool = p.src.ids != nullptr;
        const int nm = p.top_k ? (pool ? 1 : p.top_k) : 0;
        if (tid < nm) prefetch_tmap(&p.map[tid]);
        else if (tid >= 32 && tid < 32 + nm) prefetch_tmap(&p.map[8 + tid - 32]);
        else if (p.has_shared && (tid == 64 || tid == 65)) prefetch_tmap(&p.map[16 + tid - 64]);
    }
    __device__ static void stage_x(const Params& p, uint8_t* xa, int tid, int nt) {
        uint32_t* xs = reinterpret_cast<uint32_t*>(xa);
        float* xsum = reinterpret_cast<float*>(xs + x_words_stride(p.D));
        if (p.xint) {
            stage_x_int(p.x, p.D, xs, xsum, xsum + p.D / kGroup, tid, nt);
            return;
        }
        stage_words(p.x, p.D, 1, p.D, xs, p.x_aligned, true, tid, nt);
        __syncthreads();
        stage_xsum_smem(xs, x_words_stride(p.D), 1, p.D, xsum, xsum + p.D / kGroup, true, tid, nt);
    }
    __device__ static bool unit(const Params& p, int job, int u, SegDesc* d, int* chunk) {
        const uint32_t* xs = reinterpret_cast<const uint32_t*>(engine_xarea());
        d->xs = xs;
        d->xsum = reinterpret_cast<const float*>(xs + x_words_stride(p.D));
        d->xcorr = d->xsum + p.D / kGroup;
        d->xfold = p.xint ? 2 : 1;
        d->xws = x_words_stride(p.D);
        d->ntok = 1;
        d->mult = 1.0f;
        d->K = p.D;
        int rj, sjb;
        split(p, job, &rj, &sjb);
        if (rj >= 0) {
            const int slot = rj / p.fjobs, f0 = (rj - slot * p.fjobs) * 8;
            const uint8_t* b;
            uint32_t eid = 0;
            if (p.lazy_ids) {
                griddep_wait();  // the router that writes the ids has finished
                eid = __ldcg(p.src.ids + slot);
                b = eid < (uint32_t)p.src.num_experts ? p.src.pool + (size_t)eid * p.src.stride : nullptr;
                if (!b && p.err) atomicOr(p.err, kErrBadExpert);
            } else {
                b = expert_blob(p.src, slot, p.err);
                if (p.src.ids != nullptr) eid = ids_smem()[slot];
            }
            d->bits = 4;
            d->rowA = d->rowB = f0;
            d->nA = d->nB = b ? 8 : 0;
            if (!b) b = p.src.pool ? p.src.pool : p.src.blobs[0];
            const bool pool = p.src.ids != nullptr;
            d->mapA = &p.map[pool ? 0 : slot];
            d->mapB = &p.map[pool ? 8 : 8 + slot];
            d->eA = d->eB = (pool && b) ? (int)eid : 0;
            d->WA = b + p.src.off[0];
            d->SA = b + p.src.off[1];
            d->BA = b + p.src.off[2];
            d->WB = b + p.src.off[3];
            d->SB = b + p.src.off[4];
            d->BB = b + p.src.off[5];
        } else {
            const int f0 = sjb * 8;
            d->bits = p.shared_bits;
            d->rowA = d->rowB = f0;
            d->nA = d->nB = 8;
            d->mapA = &p.map[16];
            d->mapB = &p.map[17];
            d->eA = d->eB = 0;
            d->WA = p.sg.W;
            d->SA = p.sg.S;
            d->BA = p.sg.B;
            d->WB = p.su.W;
            d->SB = p.su.S;
            d->BB = p.su.B;
        }
        *chunk = u;
        return true;
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int g = lane >> 2, t = lane & 3;
        if (p.lazy_ids) griddep_wait();  // outputs are written after the router
        if (t != 0) return;  // token 0 lives in column 0: lanes with t == 0
        int rj, sjb;
        split(p, job, &rj, &sjb);
        if (rj >= 0) {
            const int slot = rj / p.fjobs, f0 = (rj - slot * p.fjobs) * 8;
            // routed: g and u stay fp32 (moe.metal:368)
            p.acts[(size_t)slot * p.F + f0 + g] = __float2half_rn(gelu_tanh(f[0]) * f[2]);
        } else {
            const int f0 = sjb * 8;
            // shared: g and u rounded to half first (gelu_mul_fp16 on half
            // GEMV outputs, utility.metal:6-18; dequant_int8.metal:150-152)
            const float gh = __half2float(__float2half_rn(f[0]));
            const float uh = __half2float(__float2half_rn(f[2]));
            p.shared_act[f0 + g] = __float2half_rn(gelu_tanh(gh) * uh);
        }
    }
};

// ===========================================================================
// Decode MoE phase 2: y[d] = half(residual[d] + sum_slot w_slot * down_slot[d].act_slot
//                                 [+ shared_down[d].shared_act])
// (moe_phase2_down_reduce_k8, moe.metal:475-511; shared down GEMV,
// SharedExpertInt4.swift:87-93).  Job = 16 consecutive d rows.
// x area: routed acts as a token block [top_k][ws(F)] words, their sums
// [top_k][F/64], then the shared act words [ws(Fs)] and sums [Fs/64].
// ===========================================================================
struct Phase2Params {
    // pool mode: map[0] down_w of all experts ([E][D][F/2]); blob mode:
    // map[slot]; shared expert down: map[8].
    CUtensorMap map[9];
    ExpertSource src;
    int D, F, top_k, upf;     // upf = units per routed down row (F)
    const __half* acts;       // [top_k][F]
    const __half* routing_w;  // [top_k] fp16
    const __half* residual;   // [D] or nullptr
    __half* y;                // [D]
    int has_shared, shared_bits, Fs;
    AffineMat sd;
    const __half* shared_act;  // [Fs]
    int rw_in_smem;            // fused layer: routing weights in rw_smem()
    int xint;                  // every consumer is int4: acts staged for the integer tensor path
    int aligned;
    uint32_t* err;
    Sched sched;
};

template <typename ST>
struct Phase2Policy {
    using Params = Phase2Params;
    static constexpr bool kWeightsIndependent = false;
    // engine hooks: schedule from the host Sched, activations staged once per CTA
    static constexpr bool kStagePerSuperjob = false;
    __device__ static int superjobs(const Params& p) { return p.sched.S_total; }
    __device__ static SuperJob superjob(const Params& p, int sjx) { return decode_superjob(p.sched, sjx); }
    __device__ static void stage_x_sj(const Params&, const SuperJob&, uint8_t*, int, int) {}
    __device__ static bool lazy(const Params&) { return false; }
    __host__ __device__ static size_t routed_words(int top_k, int F) { return (size_t)top_k * x_words_stride(F); }
    // routed: [top_k][ws] words, [top_k][F/64] sums, [top_k][F/64] corrections;
    // shared (16-byte aligned): [ws] words, [Fs/64] sums, [Fs/64] corrections
    __host__ __device__ static size_t shared_off(int top_k, int F) {
        return ((routed_words(top_k, F) * 4 + 2 * (size_t)top_k * (F / kGroup) * 4) + 15) / 16 * 16;
    }
    static size_t x_bytes(int top_k, int F, int Fs) {
        return shared_off(top_k, F) + (Fs > 0 ? (size_t)x_words_stride(Fs) * 4 + 2 * (size_t)(Fs / kGroup) * 4 : 0);
    }
    __device__ static void stage_pre(const Params& p, int tid) {
        stage_ids(p.src, p.top_k, tid);
        if (!p.aligned) return;
        const int nm = p.top_k ? (p.src.ids != nullptr ? 1 : p.top_k) : 0;
        if (tid < nm) prefetch_tmap(&p.map[tid]);
        else if (p.has_shared && tid == 32) prefetch_tmap(&p.map[8]);
    }
    __device__ static void stage_x(const Params& p, uint8_t* xa, int tid, int nt) {
        uint32_t* xs = reinterpret_cast<uint32_t*>(xa);
        float* xsum = reinterpret_cast<float*>(xs + routed_words(p.top_k, p.F));
        uint32_t* xss = reinterpret_cast<uint32_t*>(xa + shared_off(p.top_k, p.F));
        float* xsums = reinterpret_cast<float*>(xss + x_words_stride(p.Fs));
        if (p.xint) {
            const int ngF = p.F / kGroup;
            if (p.top_k)
                stage_x_int_rows(p.acts, p.F, p.top_k, p.F, xs, x_words_stride(p.F), xsum, xsum + p.top_k * ngF, tid,
                                 nt);
            if (p.has_shared) stage_x_int(p.shared_act, p.Fs, xss, xsums, xsums + p.Fs / kGroup, tid, nt);
            return;
        }
        if (p.top_k) stage_words(p.acts, p.F, p.top_k, p.F, xs, true, true, tid, nt);
        if (p.has_shared) stage_words(p.shared_act, p.Fs, 1, p.Fs, xss, true, true, tid, nt);
        __syncthreads();
        if (p.top_k)
            stage_xsum_smem(xs, x_words_stride(p.F), p.top_k, p.F, xsum, xsum + p.top_k * (p.F / kGroup), true, tid,
                            nt);
        if (p.has_shared)
            stage_xsum_smem(xss, x_words_stride(p.Fs), 1, p.Fs, xsums, xsums + p.Fs / kGroup, true, tid, nt);
    }
    __device__ static bool unit(const Params& p, int job, int u, SegDesc* d, int* chunk) {
        const uint8_t* xa = engine_xarea();
        const int d0 = job * 16;
        d->rowA = d0;
        d->rowB = d0 + 8;
        d->ntok = 1;
        const int nr = p.top_k * p.upf;
        if (u < nr) {
            const int s = p.upf == 1 ? u : u / p.upf;
            *chunk = u - s * p.upf;
            const uint8_t* b = expert_blob(p.src, s, p.err);
            const bool ok = b != nullptr;
            if (!b) b = p.src.pool ? p.src.pool : p.src.blobs[0];
            d->nA = ok ? max(0, min(8, p.D - d0)) : 0;
            d->nB = ok ? max(0, min(8, p.D - d0 - 8)) : 0;
            const bool pool = p.src.ids != nullptr;
            d->mapA = d->mapB = &p.map[pool ? 0 : s];
            d->eA = d->eB = pool ? (int)ids_smem()[s] : 0;
            d->WA = d->WB = b + p.src.off[6];
            d->SA = d->SB = b + p.src.off[7];
            d->BA = d->BB = b + p.src.off[8];
            d->K = p.F;
            d->bits = 4;
            const uint32_t* xs = reinterpret_cast<const uint32_t*>(xa);
            d->xs = xs + (size_t)s * x_words_stride(p.F);
            d->xsum = reinterpret_cast<const float*>(xs + routed_words(p.top_k, p.F)) + s * (p.F / kGroup);
            d->xcorr = d->xsum + p.top_k * (p.F / kGroup);
            d->xfold = p.xint ? 2 : 1;
            d->xws = x_words_stride(p.F);
            d->mult = __half2float(p.rw_in_smem ? rw_smem()[s] : p.routing_w[s]);
        } else {
            *chunk = u - nr;
            d->nA = max(0, min(8, p.D - d0));
            d->nB = max(0, min(8, p.D - d0 - 8));
            d->mapA = d->mapB = &p.map[8];
            d->eA = d->eB = 0;
            d->WA = d->WB = p.sd.W;
            d->SA = d->SB = p.sd.S;
            d->BA = d->BB = p.sd.B;
            d->K = p.Fs;
            d->bits = p.shared_bits;
            const uint32_t* xss = reinterpret_cast<const uint32_t*>(xa + shared_off(p.top_k, p.F));
            d->xs = xss;
            d->xsum = reinterpret_cast<const float*>(xss + x_words_stride(p.Fs));
            d->xcorr = d->xsum + p.Fs / kGroup;
            d->xfold = p.xint ? 2 : 1;
            d->xws = x_words_stride(p.Fs);
            d->mult = 1.0f;
        }
        return true;
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int g = lane >> 2, t = lane & 3;
        if (t != 0) return;
        const int r0 = job * 16 + g, r1 = r0 + 8;
        if (r0 < p.D) {
            const float res = p.residual ? __half2float(p.residual[r0]) : 0.f;
            p.y[r0] = __float2half_rn(res + f[0]);
        }
        if (r1 < p.D) {
            const float res = p.residual ? __half2float(p.residual[r1]) : 0.f;
            p.y[r1] = __float2half_rn(res + f[2]);
        }
    }
};

// ===========================================================================
// Router: logits[e] = sum_g s*sum(q*x~) + b*sum(x~), x~_i = float(half h_i) *
// float(bf16 es_i) (router_gemv_gemma4_r4, moe.metal:78-133), then top-k +
// softmax over the k + per-expert gain (router_topk_select_k8, moe.metal:135-185),
// fused: the CTA that finishes the last expert tile runs the selection.
// x~ is an fp32 product; it is staged as two fp16 terms hi + lo (token
// columns 0 and 1) so the tensor-core dot keeps ~22 bits of x~.
// ===========================================================================
struct RouterParams {
    CUtensorMap map;  // W as [1][E][D], box 8 rows x 128 B
    const uint8_t* W;
    const void* S;
    const void* B;
    const __half* hidden;
    const __nv_bfloat16* eff_scale;
    const __nv_bfloat16* per_expert_scale;
    int E, D, top_k;
    float* logits;        // [E] workspace
    float* out_logits;    // optional caller copy of the fp32 logits [E] (NULL = none)
    unsigned int* ticket; // workspace counter, left at 0
    uint32_t* out_idx;
    __half* out_w;
    int fused;  // fused layer: write the logits only (selection runs per CTA later)
    int replicas;  // copies of the logits written 256 floats apart (each CTA reads one)
    int aligned;
    uint32_t* err;
    Sched sched;
};

__device__ __forceinline__ void warp_topk_softmax(const float* logits, int E, int k,
                                                  const __nv_bfloat16* pes, uint32_t* out_idx,
                                                  __half* out_w, int lane) {
    // Selection order = sort by (logit desc, expert id asc): identical to the
    // reference's insertion with strict '>' and ties to the lower id.
    constexpr int kPer = 8;  // E <= 256
    // lane holds experts lane*8 .. lane*8+7: two 16-byte loads per lane
    // (`logits` has room for 256 entries)
    float v[kPer];
    {
        const float4 a = __ldcg(reinterpret_cast<const float4*>(logits) + lane * 2);
        const float4 b = __ldcg(reinterpret_cast<const float4*>(logits) + lane * 2 + 1);
        const float t[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < kPer; ++i) v[i] = lane * kPer + i < E ? t[i] : -INFINITY;
    }
    float my_exp = 0.f;
    int my_e = -1;
    float vmax = 0.f;
    float sum = 0.f;
    for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int e = lane * kPer + i;
            if (e < E && (v[i] > bv || (v[i] == bv && e < be))) {
                bv = v[i];
                be = e;
            }
        }
        for (int off = 16; off; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
            const int oe = __shfl_xor_sync(0xffffffffu, be, off);
            if (ov > bv || (ov == bv && oe < be)) {
                bv = ov;
                be = oe;
            }
        }
        if (r == 0) vmax = bv;
        const float ex = expf(bv - vmax);
        sum += ex;
        if (lane == r) {
            my_e = be;
            my_exp = ex;
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i)
            if (lane * kPer + i == be) v[i] = -INFINITY;
        if (be >= E) break;
    }
    if (lane < k && my_e >= 0) {
        out_idx[lane] = (uint32_t)my_e;
        out_w[lane] = __float2half_rn(my_exp / sum * __bfloat162float(pes[my_e]));
    }
}

// CTA-parallel selection for E <= 256 experts (threads 0..255 take part;
// every thread of the CTA must call it).  Expert e's rank = number of experts
// ordered before it by (logit desc, id asc), the same order as the
// reference's insertion (moe.metal:152-169).  Experts with rank < k are the
// selection, in rank order; softmax over them, times the per-expert gain.
// `scratch` = 256 floats of shared memory.
__device__ __forceinline__ void cta_topk_softmax(const float* logits, int E, int k, const __nv_bfloat16* pes,
                                                 uint32_t* out_idx, __half* out_w, float* scratch) {
    const int e = threadIdx.x;
    float v = -INFINITY;
    if (e < 256) {
        v = e < E ? __ldcg(logits + e) : -INFINITY;
        scratch[e] = v;
    }
    __syncthreads();
    int rank = 0;
    if (e < E) {
        for (int j = 0; j < E; ++j) {
            const float o = scratch[j];
            rank += (o > v || (o == v && j < e)) ? 1 : 0;
        }
    }
    __syncthreads();  // everyone done reading scratch
    if (e < E && rank < k) {
        out_idx[rank] = (uint32_t)e;
        scratch[rank] = v;  // selected logits in rank order
    }
    __syncthreads();
    if (e < k) {
        const float vmax = scratch[0];
        float sum = 0.f;
        for (int r = 0; r < k; ++r) sum += expf(scratch[r] - vmax);
        const uint32_t ex = out_idx[e];
        out_w[e] = __float2half_rn(expf(scratch[e] - vmax) / sum * __bfloat162float(pes[ex]));
    }
    __syncthreads();
}

template <typename ST>
struct RouterPolicy {
    using Params = RouterParams;
    static constexpr bool kWeightsIndependent = true;
    // engine hooks: schedule from the host Sched, activations staged once per CTA
    static constexpr bool kStagePerSuperjob = false;
    __device__ static int superjobs(const Params& p) { return p.sched.S_total; }
    __device__ static SuperJob superjob(const Params& p, int sjx) { return decode_superjob(p.sched, sjx); }
    __device__ static void stage_x_sj(const Params&, const SuperJob&, uint8_t*, int, int) {}
    __device__ static bool lazy(const Params&) { return false; }
    static size_t x_bytes(int D) { return (size_t)2 * x_words_stride(D) * 4 + (size_t)2 * (D / kGroup) * 4; }
    __device__ static void stage_pre(const Params& p, int tid) {
        if (tid == 0 && p.aligned) prefetch_tmap(&p.map);
    }
    __device__ static void stage_x(const Params& p, uint8_t* xa, int tid, int nt) {
        uint32_t* xs = reinterpret_cast<uint32_t*>(xa);
        const int ws = x_words_stride(p.D);
        float* xsum = reinterpret_cast<float*>(xs + 2 * ws);
        const int ng = p.D / kGroup;
        for (int i = tid; i < p.D / 8; i += nt) {
            __half hi[8], lo[8];
            for (int j = 0; j < 8; ++j) {
                const int k = i * 8 + j;
                const float xt = __half2float(p.hidden[k]) * __bfloat162float(p.eff_scale[k]);
                hi[j] = __float2half_rn(xt);
                lo[j] = __float2half_rn(xt - __half2float(hi[j]));
            }
            for (int j = 0; j < 4; ++j) {
                __half2 a = __halves2half2(hi[j], hi[j + 4]);
                __half2 b = __halves2half2(lo[j], lo[j + 4]);
                xs[i * 4 + j] = *reinterpret_cast<uint32_t*>(&a);
                xs[ws + i * 4 + j] = *reinterpret_cast<uint32_t*>(&b);
            }
        }
        __syncthreads();
        const int warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
        for (int g = warp; g < ng; g += nw) {
            // x~ = hi + lo: sum both staged halves of the group's 64 values
            const uint32_t a = xs[g * 32 + lane], b = xs[ws + g * 32 + lane];
            const __half2 ha = *reinterpret_cast<const __half2*>(&a);
            const __half2 hb = *reinterpret_cast<const __half2*>(&b);
            float s = (__low2float(ha) + __low2float(hb)) + (__high2float(ha) + __high2float(hb));
            for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
            if (lane == 0) {
                xsum[g] = s;  // bias term rides on column 0 only
                xsum[ng + g] = 0.f;
            }
        }
    }
    __device__ static bool unit(const Params& p, int job, int u, SegDesc* d, int* chunk) {
        const uint32_t* xs = reinterpret_cast<const uint32_t*>(engine_xarea());
        d->WA = d->WB = p.W;
        d->mapA = d->mapB = &p.map;
        d->eA = d->eB = 0;
        d->SA = d->SB = p.S;
        d->BA = d->BB = p.B;
        d->rowA = job * 16;
        d->rowB = job * 16 + 8;
        d->nA = max(0, min(8, p.E - d->rowA));
        d->nB = max(0, min(8, p.E - d->rowB));
        d->K = p.D;
        d->bits = 8;
        d->xs = xs;
        d->xsum = reinterpret_cast<const float*>(xs + 2 * x_words_stride(p.D));
        d->xcorr = nullptr;
        d->xfold = 0;
        d->xws = x_words_stride(p.D);
        d->ntok = 2;
        d->mult = 1.0f;
        *chunk = u;
        return true;
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int g = lane >> 2, t = lane & 3;
        if (t == 0) {
            const int e0 = job * 16 + g, e1 = e0 + 8;
            for (int r = 0; r < max(1, p.replicas); ++r) {
                if (e0 < p.E) p.logits[r * 256 + e0] = f[0] + f[1];
                if (e1 < p.E) p.logits[r * 256 + e1] = f[2] + f[3];
            }
            if (p.out_logits) {
                if (e0 < p.E) p.out_logits[e0] = f[0] + f[1];
                if (e1 < p.E) p.out_logits[e1] = f[2] + f[3];
            }
        }
        if (p.fused) return;
        __threadfence();
        __syncwarp();
        unsigned int tk = 0;
        if (lane == 0) tk = atomicAdd(p.ticket, 1u);
        tk = __shfl_sync(0xffffffffu, tk, 0);
        const unsigned int njobs = (unsigned int)((p.E + 15) / 16);
        if (tk == njobs - 1) {
            __threadfence();
            warp_topk_softmax(p.logits, p.E, p.top_k, p.per_expert_scale, p.out_idx, p.out_w, lane);
            if (lane == 0) *p.ticket = 0u;
        }
    }
};


// ===========================================================================
// Grouped routed experts on the streaming engine (small token counts per
// expert: batched decode).  The device grouping (tf_moe_route_sort) gives,
// per non-empty expert, a contiguous range of sorted pairs; the range is cut
// into passes of at most `nt` tokens and each (group, pass) is one super-job
// whose token rows are staged once (kStagePerSuperjob).  MODE 0: gate/up rows
// of the expert with GELU(g)*u per token -> acts[pair][f] (sorted-pair order);
// MODE 1: down rows -> route_partials[(token*top_k + rank)][d].  Same
// arithmetic as prefill_grouped_routed_moe_batched_phase1/_down
// (prefill.metal:336-440, 598-670): g and u fp32, act and partial rounded to
// fp16.
// ===========================================================================
struct GroupedParams {
    CUtensorMap map[3];  // gate_w, up_w, down_w of all experts: [E][rows][row_bytes]
    const uint8_t* pool;
    unsigned long long stride;
    uint32_t off[9];
    int E, D, F, top_k, nt;  // nt: tokens per pass
    const tf_moe_group* groups;
    const uint32_t* n_groups;
    const tf_token_expert_pair* pairs;
    const __half* hidden;  // MODE 0 input rows, gathered through the pairs
    int hstride;
    __half* acts;      // [pairs][F] sorted order (MODE 0 out, MODE 1 in)
    __half* partials;  // [T*top_k][D] (MODE 1 out)
    int aligned;
    uint32_t* err;
    Sched sched;  // unused: the schedule comes from the device groups
};

struct GroupTab {
    int ng, passes, staged_pass;
    int prefix[257];  // passes before group g
    int start[256], count[256], expert[256];
};
__device__ __forceinline__ GroupTab& group_tab() {
    __shared__ GroupTab t;
    return t;
}

// Work decomposition: pass = (group, up to nt of its tokens); each pass has
// jobs_per row jobs (8 gate+up rows, or 16 down rows) cut into chunks of
// kWarps / U jobs, so a super-job's units fit the engine's one-round
// reduction.  Super-jobs are numbered so that a CTA's consecutive super-jobs
// are consecutive chunks (usually of one pass): the pass's token rows are
// staged once per CTA per pass.
template <typename ST, int MODE>
struct GroupedPolicy {
    using Params = GroupedParams;
    static constexpr bool kWeightsIndependent = false;
    __device__ static bool lazy(const Params&) { return false; }
    static constexpr bool kStagePerSuperjob = true;
    __host__ __device__ static int kdim(const Params& p) { return MODE == 0 ? p.D : p.F; }
    __host__ __device__ static int jobs_per(const Params& p) { return MODE == 0 ? p.F / 8 : (p.D + 15) / 16; }
    __host__ __device__ static int units(const Params& p) { return units_for_K(kdim(p), 4); }
    __host__ __device__ static int chunk_jobs(const Params& p) { return max(1, kWarps / units(p)); }
    __host__ __device__ static int chunks(const Params& p) {
        return (jobs_per(p) + chunk_jobs(p) - 1) / chunk_jobs(p);
    }
    static size_t x_bytes(int K, int ntok) {
        return (size_t)ntok * x_words_stride(K) * 4 + 2 * (size_t)ntok * (K / kGroup) * 4;
    }
    __device__ static void stage_pre(const Params& p, int tid) {
        GroupTab& tb = group_tab();
        if (tid < 32) {
            const int lane = tid;
            const int ng = min((int)__ldcg(p.n_groups), 256);
            int cnt[8], run = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int g = lane * 8 + j;
                int ps = 0;
                if (g < ng) {
                    const tf_moe_group gr = p.groups[g];
                    tb.start[g] = (int)gr.pair_start;
                    tb.count[g] = (int)gr.pair_count;
                    tb.expert[g] = (int)gr.expert;
                    if (gr.expert < (uint32_t)p.E)
                        ps = ((int)gr.pair_count + p.nt - 1) / p.nt;
                    else if (p.err)
                        atomicOr(p.err, kErrBadExpert);
                }
                cnt[j] = ps;
                run += ps;
            }
            int incl = run;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int acc = incl - run;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int g = lane * 8 + j;
                if (g <= ng) tb.prefix[g] = acc;
                acc += cnt[j];
            }
            if (lane == 31) {
                tb.passes = incl;
                if (ng == 256) tb.prefix[256] = incl;
            }
            if (lane == 0) {
                tb.ng = ng;
                tb.staged_pass = -1;
            }
        } else if (p.aligned && tid == 32) {
            prefetch_tmap(&p.map[MODE == 0 ? 0 : 2]);
            if (MODE == 0) prefetch_tmap(&p.map[1]);
        }
    }
    __device__ static void stage_x(const Params&, uint8_t*, int, int) {}  // per pass instead
    __device__ static int per_cta(const Params& p) {
        const int W = group_tab().passes * chunks(p);
        return (W + (int)gridDim.x - 1) / (int)gridDim.x;
    }
    __device__ static int superjobs(const Params& p) { return per_cta(p) * (int)gridDim.x; }
    // engine index sjx (CTA sjx % grid, its (sjx / grid)-th super-job) ->
    // CTA-contiguous work index -> (pass, chunk); jobs are numbered
    // pass * jobs_per + row job.  J = 0 marks an index past the work.
    __device__ static SuperJob superjob(const Params& p, int sjx) {
        SuperJob s;
        s.U = units(p);
        const int G = (int)gridDim.x;
        const int L = (sjx % G) * per_cta(p) + sjx / G;
        const int C = chunks(p), CJ = chunk_jobs(p), JP = jobs_per(p);
        if (L >= group_tab().passes * C) {
            s.j0 = s.j1 = 0;
            s.J = 0;
            return s;
        }
        const int pass = L / C, ch = L - pass * C;
        const int l0 = ch * CJ, l1 = min(JP, l0 + CJ);
        s.j0 = pass * JP + l0;
        s.j1 = pass * JP + l1;
        s.J = l1 - l0;
        return s;
    }
    // pass -> expert, first pair, tokens of the pass
    __device__ static void locate(const Params& p, int pass, int* e, int* pair0, int* ntok) {
        const GroupTab& tb = group_tab();
        int lo = 0, hi = tb.ng - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (tb.prefix[mid] <= pass) lo = mid; else hi = mid - 1;
        }
        const int k = pass - tb.prefix[lo];
        *e = tb.expert[lo];
        *pair0 = tb.start[lo] + k * p.nt;
        *ntok = min(p.nt, tb.count[lo] - k * p.nt);
    }
    __device__ static void stage_x_sj(const Params& p, const SuperJob& sj, uint8_t* xa, int tid, int nt) {
        if (sj.J == 0) return;
        GroupTab& tb = group_tab();
        const int pass = sj.j0 / jobs_per(p);
        if (pass == tb.staged_pass) return;  // uniform: written only after the barrier below
        int e, p0, ntok;
        locate(p, pass, &e, &p0, &ntok);
        const int K = kdim(p), ws = x_words_stride(K);
        uint32_t* xs = reinterpret_cast<uint32_t*>(xa);
        float* xsum = reinterpret_cast<float*>(xs + p.nt * ws);
        float* xcorr = xsum + p.nt * (K / kGroup);
        if (MODE == 0) {
            for (int t = 0; t < ntok; ++t) {
                const uint32_t row = p.pairs[p0 + t].token;
                stage_words(p.hidden + (size_t)row * p.hstride, p.hstride, 1, K, xs + t * ws, true, false, tid, nt);
            }
        } else {
            stage_words(p.acts + (size_t)p0 * p.F, p.F, ntok, K, xs, true, false, tid, nt);
        }
        __syncthreads();
        stage_xsum_smem(xs, ws, ntok, K, xsum, xcorr, false, tid, nt);
        if (tid == 0) tb.staged_pass = pass;
    }
    __device__ static bool unit(const Params& p, int job, int u, SegDesc* d, int* chunk) {
        const int JP = jobs_per(p);
        const int pass = job / JP, local = job - pass * JP;
        int e, p0, ntok;
        locate(p, pass, &e, &p0, &ntok);
        const uint8_t* b = p.pool + (size_t)e * p.stride;
        const int K = kdim(p);
        d->K = K;
        d->bits = 4;
        d->eA = d->eB = e;
        if (MODE == 0) {
            d->rowA = d->rowB = local * 8;
            d->nA = d->nB = 8;
            d->mapA = &p.map[0];
            d->mapB = &p.map[1];
            d->WA = b + p.off[0];
            d->SA = b + p.off[1];
            d->BA = b + p.off[2];
            d->WB = b + p.off[3];
            d->SB = b + p.off[4];
            d->BB = b + p.off[5];
        } else {
            d->rowA = local * 16;
            d->rowB = d->rowA + 8;
            d->nA = max(0, min(8, p.D - d->rowA));
            d->nB = max(0, min(8, p.D - d->rowB));
            d->mapA = d->mapB = &p.map[2];
            d->WA = d->WB = b + p.off[6];
            d->SA = d->SB = b + p.off[7];
            d->BA = d->BB = b + p.off[8];
        }
        const uint32_t* xs = reinterpret_cast<const uint32_t*>(engine_xarea());
        const int ws = x_words_stride(K);
        d->xs = xs;
        d->xsum = reinterpret_cast<const float*>(xs + p.nt * ws);
        d->xcorr = d->xsum + p.nt * (K / kGroup);
        d->xfold = 0;
        d->xws = ws;
        d->ntok = ntok;
        d->mult = 1.0f;
        *chunk = u;
        return true;
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int JP = jobs_per(p);
        const int pass = job / JP, local = job - pass * JP;
        int e, p0, ntok;
        locate(p, pass, &e, &p0, &ntok);
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int tok = 2 * t + j;
            if (tok >= ntok) continue;
            if (MODE == 0) {
                // rows A = gate f0+g, rows B = up f0+g; g and u stay fp32
                p.acts[(size_t)(p0 + tok) * p.F + local * 8 + g] = __float2half_rn(gelu_tanh(f[j]) * f[2 + j]);
            } else {
                const tf_token_expert_pair pr = p.pairs[p0 + tok];
                __half* out = p.partials + ((size_t)pr.token * p.top_k + pr.rank) * p.D;
                const int r0 = local * 16 + g, r1 = r0 + 8;
                if (r0 < p.D) out[r0] = __float2half_rn(f[j]);
                if (r1 < p.D) out[r1] = __float2half_rn(f[2 + j]);
            }
        }
    }
};

}  // namespace tf
