// tf_policies.cuh -- job/segment/epilogue policies for the streaming engine.
// Each policy maps the reference operator's output rows onto 16-row jobs.
#pragma once
#include "tf_engine.cuh"

namespace tf {

// ===========================================================================
// Plain affine GEMV, Y[tok][row] = sum_k W[row][k] * X[tok][k]
// (dequant_int4_gemv_simd / dequant_int8_gemv_simd; a batch of matrices with
// a common activation block of up to 8 tokens).
// ===========================================================================
struct GemvParams {
    const uint8_t* W;
    const void* S;
    const void* B;
    long long w_bstride;   // bytes between matrices
    long long sb_bstride;  // elements between scale blocks
    int M, K, batch, bits;
    const __half* x;
    int x_row_stride;  // elements between tokens
    int ntok;
    __half* y;
    int y_row_stride;     // elements between tokens of y
    long long y_bstride;  // elements between matrices of y
    int aligned, x_aligned, ns;
    uint32_t* err;
};

template <typename ST>
struct GemvPolicy {
    using Params = GemvParams;
    __device__ static int nranges(const Params&) { return 1; }
    __device__ static void range(const Params& p, int, int* nj, int* U) {
        *nj = p.batch * ((p.M + 15) / 16);
        *U = units_for_K(p.K, p.bits);
    }
    __device__ static void stage_x(const Params& p, uint8_t* xa, int tid, int nt) {
        uint32_t* xs = reinterpret_cast<uint32_t*>(xa);
        float* xsum = reinterpret_cast<float*>(xs + kMaxTok * x_words_stride(p.K));
        if (p.x_aligned)
            tf::stage_x(p.x, p.x_row_stride, p.ntok, p.K, xs, xsum, tid, nt);
        else
            stage_x_scalar(p.x, p.x_row_stride, p.ntok, p.K, xs, xsum, tid, nt);
    }
    static size_t x_bytes(int K) {
        return (size_t)kMaxTok * x_words_stride(K) * 4 + (size_t)kMaxTok * (K / kGroup) * 4;
    }
    __device__ static int nseg(const Params&, int) { return 1; }
    __device__ static void seg(const Params& p, int job, int, SegDesc* d) {
        extern __shared__ __align__(128) uint8_t smem[];
        const int tiles = (p.M + 15) / 16;
        const int b = job / tiles, tile = job % tiles;
        const uint8_t* W = p.W + (size_t)b * p.w_bstride;
        const ST* S = reinterpret_cast<const ST*>(p.S) + (size_t)b * p.sb_bstride;
        const ST* B = reinterpret_cast<const ST*>(p.B) + (size_t)b * p.sb_bstride;
        d->WA = d->WB = W;
        d->SA = d->SB = S;
        d->BA = d->BB = B;
        d->rowA = tile * 16;
        d->nA = max(0, min(8, p.M - d->rowA));
        d->rowB = d->rowA + 8;
        d->nB = max(0, min(8, p.M - d->rowB));
        d->K = p.K;
        d->bits = p.bits;
        const uint32_t* xs = reinterpret_cast<const uint32_t*>(
            smem + engine_fixed_smem(p.ns));
        d->xs = xs;
        d->xsum = reinterpret_cast<const float*>(xs + kMaxTok * x_words_stride(p.K));
        d->xws = x_words_stride(p.K);
        d->ntok = p.ntok;
        d->mult = 1.0f;
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int tiles = (p.M + 15) / 16;
        const int b = job / tiles, tile = job % tiles;
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
};

__device__ __forceinline__ const uint8_t* expert_blob(const ExpertSource& es, int slot, uint32_t* err) {
    if (es.ids == nullptr) return es.blobs[slot];
    const uint32_t e = __ldg(es.ids + slot);
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
    ExpertSource src;
    int D, F, top_k;
    const __half* x;
    __half* acts;  // [top_k][F]
    int has_shared, shared_bits, Fs;
    AffineMat sg, su;
    __half* shared_act;  // [Fs]
    int aligned, x_aligned, ns;
    uint32_t* err;
};

template <typename ST>
struct Phase1Policy {
    using Params = Phase1Params;
    __device__ static int nranges(const Params& p) { return p.has_shared ? 2 : 1; }
    __device__ static void range(const Params& p, int r, int* nj, int* U) {
        if (r == 0) {
            *nj = p.top_k * (p.F / 8);
            *U = units_for_K(p.D, 4);
        } else {
            *nj = p.Fs / 8;
            *U = units_for_K(p.D, p.shared_bits);
        }
    }
    static size_t x_bytes(int D) { return (size_t)x_words_stride(D) * 4 + (size_t)(D / kGroup) * 4; }
    __device__ static void stage_x(const Params& p, uint8_t* xa, int tid, int nt) {
        uint32_t* xs = reinterpret_cast<uint32_t*>(xa);
        float* xsum = reinterpret_cast<float*>(xs + x_words_stride(p.D));
        if (p.x_aligned)
            tf::stage_x(p.x, p.D, 1, p.D, xs, xsum, tid, nt);
        else
            stage_x_scalar(p.x, p.D, 1, p.D, xs, xsum, tid, nt);
    }
    __device__ static int nseg(const Params&, int) { return 1; }
    __device__ static void seg(const Params& p, int job, int, SegDesc* d) {
        extern __shared__ __align__(128) uint8_t smem[];
        const uint32_t* xs = reinterpret_cast<const uint32_t*>(smem + engine_fixed_smem(p.ns));
        d->xs = xs;
        d->xsum = reinterpret_cast<const float*>(xs + x_words_stride(p.D));
        d->xws = x_words_stride(p.D);
        d->ntok = 1;
        d->mult = 1.0f;
        d->K = p.D;
        const int rjobs = p.top_k * (p.F / 8);
        if (job < rjobs) {
            const int slot = job / (p.F / 8), f0 = (job % (p.F / 8)) * 8;
            const uint8_t* b = expert_blob(p.src, slot, p.err);
            d->bits = 4;
            d->rowA = d->rowB = f0;
            d->nA = d->nB = b ? 8 : 0;
            if (!b) b = p.src.pool ? p.src.pool : p.src.blobs[0];
            d->WA = b + p.src.off[0];
            d->SA = b + p.src.off[1];
            d->BA = b + p.src.off[2];
            d->WB = b + p.src.off[3];
            d->SB = b + p.src.off[4];
            d->BB = b + p.src.off[5];
        } else {
            const int f0 = (job - rjobs) * 8;
            d->bits = p.shared_bits;
            d->rowA = d->rowB = f0;
            d->nA = d->nB = 8;
            d->WA = p.sg.W;
            d->SA = p.sg.S;
            d->BA = p.sg.B;
            d->WB = p.su.W;
            d->SB = p.su.S;
            d->BB = p.su.B;
        }
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int g = lane >> 2, t = lane & 3;
        if (t != 0) return;  // token 0 lives in column 0: lanes with t == 0
        const int rjobs = p.top_k * (p.F / 8);
        if (job < rjobs) {
            const int slot = job / (p.F / 8), f0 = (job % (p.F / 8)) * 8;
            // routed: g and u stay fp32 (moe.metal:368)
            p.acts[(size_t)slot * p.F + f0 + g] = __float2half_rn(gelu_tanh(f[0]) * f[2]);
        } else {
            const int f0 = (job - rjobs) * 8;
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
// ===========================================================================
struct Phase2Params {
    ExpertSource src;
    int D, F, top_k;
    const __half* acts;       // [top_k][F]
    const __half* routing_w;  // [top_k] fp16
    const __half* residual;   // [D] or nullptr
    __half* y;                // [D]
    int has_shared, shared_bits, Fs;
    AffineMat sd;
    const __half* shared_act;  // [Fs]
    int aligned, ns;
    uint32_t* err;
};

template <typename ST>
struct Phase2Policy {
    using Params = Phase2Params;
    __device__ static int nranges(const Params&) { return 1; }
    __device__ static void range(const Params& p, int, int* nj, int* U) {
        *nj = (p.D + 15) / 16;
        *U = p.top_k * units_for_K(p.F, 4) + (p.has_shared ? units_for_K(p.Fs, p.shared_bits) : 0);
    }
    // x area: top_k routed act slots (F) then the shared act slot (Fs).
    // Each slot (staged activation + per-group sums) is rounded up to 16 bytes
    // so the next slot's staged words stay 16-byte aligned for vector loads.
    __host__ __device__ static size_t slot_bytes(int K) {
        return ((size_t)x_words_stride(K) * 4 + (size_t)(K / kGroup) * 4 + 15) / 16 * 16;
    }
    static size_t x_bytes(int top_k, int F, int Fs) {
        return (size_t)top_k * slot_bytes(F) + (size_t)(Fs > 0 ? slot_bytes(Fs) : 0);
    }
    __device__ static void stage_x(const Params& p, uint8_t* xa, int tid, int nt) {
        for (int s = 0; s < p.top_k; ++s) {
            uint32_t* xs = reinterpret_cast<uint32_t*>(xa + s * slot_bytes(p.F));
            float* xsum = reinterpret_cast<float*>(xs + x_words_stride(p.F));
            tf::stage_x(p.acts + (size_t)s * p.F, p.F, 1, p.F, xs, xsum, tid, nt);
        }
        if (p.has_shared) {
            uint32_t* xs = reinterpret_cast<uint32_t*>(xa + p.top_k * slot_bytes(p.F));
            float* xsum = reinterpret_cast<float*>(xs + x_words_stride(p.Fs));
            tf::stage_x(p.shared_act, p.Fs, 1, p.Fs, xs, xsum, tid, nt);
        }
    }
    __device__ static int nseg(const Params& p, int) { return p.top_k + (p.has_shared ? 1 : 0); }
    __device__ static void seg(const Params& p, int job, int s, SegDesc* d) {
        extern __shared__ __align__(128) uint8_t smem[];
        uint8_t* xa = smem + engine_fixed_smem(p.ns);
        const int d0 = job * 16;
        d->rowA = d0;
        d->rowB = d0 + 8;
        d->ntok = 1;
        if (s < p.top_k) {
            const uint8_t* b = expert_blob(p.src, s, p.err);
            const bool ok = b != nullptr;
            if (!b) b = p.src.pool ? p.src.pool : p.src.blobs[0];
            d->nA = ok ? max(0, min(8, p.D - d0)) : 0;
            d->nB = ok ? max(0, min(8, p.D - d0 - 8)) : 0;
            d->WA = d->WB = b + p.src.off[6];
            d->SA = d->SB = b + p.src.off[7];
            d->BA = d->BB = b + p.src.off[8];
            d->K = p.F;
            d->bits = 4;
            const uint32_t* xs = reinterpret_cast<const uint32_t*>(xa + s * slot_bytes(p.F));
            d->xs = xs;
            d->xsum = reinterpret_cast<const float*>(xs + x_words_stride(p.F));
            d->xws = x_words_stride(p.F);
            d->mult = __half2float(p.routing_w[s]);
        } else {
            d->nA = max(0, min(8, p.D - d0));
            d->nB = max(0, min(8, p.D - d0 - 8));
            d->WA = d->WB = p.sd.W;
            d->SA = d->SB = p.sd.S;
            d->BA = d->BB = p.sd.B;
            d->K = p.Fs;
            d->bits = p.shared_bits;
            const uint32_t* xs = reinterpret_cast<const uint32_t*>(xa + p.top_k * slot_bytes(p.F));
            d->xs = xs;
            d->xsum = reinterpret_cast<const float*>(xs + x_words_stride(p.Fs));
            d->xws = x_words_stride(p.Fs);
            d->mult = 1.0f;
        }
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
    const uint8_t* W;
    const void* S;
    const void* B;
    const __half* hidden;
    const __nv_bfloat16* eff_scale;
    const __nv_bfloat16* per_expert_scale;
    int E, D, top_k;
    float* logits;        // [E] workspace
    unsigned int* ticket; // workspace counter, left at 0
    uint32_t* out_idx;
    __half* out_w;
    int aligned, ns;
    uint32_t* err;
};

__device__ __forceinline__ void warp_topk_softmax(const float* logits, int E, int k,
                                                  const __nv_bfloat16* pes, uint32_t* out_idx,
                                                  __half* out_w, int lane) {
    // Selection order = sort by (logit desc, expert id asc): identical to the
    // reference's insertion with strict '>' and ties to the lower id.
    constexpr int kPer = 8;  // E <= 256
    float v[kPer];
    for (int i = 0; i < kPer; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < E ? __ldcg(logits + e) : -INFINITY;
    }
    float sel_v[64 / 32 + 1];
    (void)sel_v;
    float top_val = -INFINITY;
    float my_exp = 0.f;
    int my_e = -1;
    float vmax = 0.f;
    float sum = 0.f;
    for (int r = 0; r < k; ++r) {
        // local best
        float bv = -INFINITY;
        int be = 0x7fffffff;
        for (int i = 0; i < kPer; ++i) {
            const int e = lane + 32 * i;
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
            top_val = bv;
        }
        if (be < E && (be & 31) == lane) v[be >> 5] = -INFINITY;
        if (be >= E) break;
    }
    (void)top_val;
    if (lane < k && my_e >= 0) {
        out_idx[lane] = (uint32_t)my_e;
        out_w[lane] = __float2half_rn(my_exp / sum * __bfloat162float(pes[my_e]));
    }
}

template <typename ST>
struct RouterPolicy {
    using Params = RouterParams;
    __device__ static int nranges(const Params&) { return 1; }
    __device__ static void range(const Params& p, int, int* nj, int* U) {
        *nj = (p.E + 15) / 16;
        *U = units_for_K(p.D, 8);
    }
    static size_t x_bytes(int D) { return (size_t)2 * x_words_stride(D) * 4 + (size_t)2 * (D / kGroup) * 4; }
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
        for (int g = tid; g < ng; g += nt) {
            float s = 0.f;
            for (int k = 0; k < kGroup; ++k) {
                const int i = g * kGroup + k;
                s += __half2float(p.hidden[i]) * __bfloat162float(p.eff_scale[i]);
            }
            xsum[g] = s;       // bias term rides on column 0 only
            xsum[ng + g] = 0.f;
        }
    }
    __device__ static int nseg(const Params&, int) { return 1; }
    __device__ static void seg(const Params& p, int job, int, SegDesc* d) {
        extern __shared__ __align__(128) uint8_t smem[];
        const uint32_t* xs = reinterpret_cast<const uint32_t*>(smem + engine_fixed_smem(p.ns));
        d->WA = d->WB = p.W;
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
        d->xws = x_words_stride(p.D);
        d->ntok = 2;
        d->mult = 1.0f;
    }
    __device__ static void epilogue(const Params& p, int job, const float f[4], int lane) {
        const int g = lane >> 2, t = lane & 3;
        if (t == 0) {
            const int e0 = job * 16 + g, e1 = e0 + 8;
            if (e0 < p.E) p.logits[e0] = f[0] + f[1];
            if (e1 < p.E) p.logits[e1] = f[2] + f[3];
        }
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

}  // namespace tf
