// tf_grouped_stream.cu -- grouped routed experts for batched decode: every hit
// expert's weights are streamed from HBM once per pass of up to TP tokens
// (prefill_grouped_routed_moe_batched_phase1 / _down, Metal/Prefill/prefill.metal:
// 336-440,598-670, encoded by PrefillGroupedRoutedMoE.encodeStreamedBatched,
// Kernels/Prefill/MoE/PrefillGroupedRoutedMoE.swift:446-527).
//
// MODE 0 (gate/up): a job is (expert group, pass of <= TP tokens, tile of 120
// features).  Warp w owns features 8w..8w+7 of the tile: the MMA's A rows
// 0-7 are their gate rows and rows 8-15 their up rows, so a lane ends with
// gate and up of the same feature and token and forms act = half(gelu(g) * u)
// in registers: acts[pair][f] in sorted-pair order.
// MODE 1 (down): a job is (group, pass, 240 rows of down); warp w owns rows
// 16w..16w+15 and writes route_partials[(token * top_k + rank)][row] =
// half(sum) from registers.
//
// Data movement: one loader thread puts the weight stages (3-D TMA, 128-byte
// swizzle, 4 groups x 240 rows = 30 KB per stage) into a ring and prefetches
// each tile's scale/bias rows into L2; the 15 consumer warps read their
// scales from L2 into registers one stage ahead.  A CTA works through a
// contiguous range of jobs (tile innermost), so the pass's token rows are
// staged into shared memory once per (group, pass).
// Arithmetic (the engine's offset-folded path): codes -> fp16 1024 + q and
// 1024 + 16q (dq4_folded), the tokens' fp16 rows staged in octet-pair order
// with the odd pairs divided by 16 as the MMA's N columns (8 tokens per MMA),
// mma.sync m16n8k16 f16 -> f32 per group with the accumulator started at
// -1024 * sum(staged x); per group and token acc += s * dot + b * sum(x) in fp32.
// Every wait is bounded; a timeout raises kErrMbarTimeout and all roles leave.
#include "tf_context.cuh"
#include "tf_gemv_tc.cuh"
#include "tf_umma.cuh"

using namespace tf;

namespace {

// 15 consumer warps + the loader warp = 16 warps: 4 per sub-partition, so a
// thread may hold 128 registers
constexpr int kGsConsumers = 15;
constexpr int kGsRowsW0 = 8;                        // MODE 0: features per warp (8 gate + 8 up rows)
constexpr int kGsTile0 = kGsConsumers * kGsRowsW0;  // 120 features
constexpr int kGsTile1 = kGsConsumers * 16;         // MODE 1: 240 rows
constexpr int kGsBox = kGsTile0 * 128;              // one TMA box: 120 rows x 128 B (4 groups)
constexpr int kGsStage = 2 * kGsBox;                // 4 groups x 240 rows (30 KB, a multiple of 1 KB)
constexpr int kGsMaxR = 7;
constexpr int kGsThreads = 32 * (1 + kGsConsumers);
constexpr int kGsMaxGroups = 256;
constexpr size_t kGsSmemLimit = 232448 - 1024;  // room for the static s_tok array
constexpr uint32_t kGsSpin = 1u << 21;

struct GsParams {
    CUtensorMap map0;  // MODE 0: gate codes [E][F][D/2], box 128 B x 120 rows; MODE 1: down [E][D][F/2], 128 x 240
    CUtensorMap map1;  // MODE 0: up codes
    const uint8_t* pool;
    unsigned long long stride;
    uint32_t os0, ob0, os1, ob1;  // scale/bias offsets in the blob (MODE 0: gate, up; MODE 1: down)
    const tf_moe_group* groups;
    const uint32_t* n_groups;
    const tf_token_expert_pair* pairs;
    const __half* x;  // MODE 0: hidden [T][x_stride]; MODE 1: acts [pairs][F]
    long long x_stride;
    __half* acts;
    __half* partials;
    int mode, E, D, F, K, top_k, TP, R, ntile, T;
    uint32_t* err;
};

struct GsBars {
    uint64_t full[kGsMaxR], empty[kGsMaxR];
    int abort_flag;
    int stop;
    int job_start[kGsMaxGroups + 1];  // prefix of jobs per group
    int passes[kGsMaxGroups];
};

struct GsLayout {
    uint32_t xs, xc, bars, total;
};

// [ring: R stages][token rows: TP x x_words_stride(K) words][per group and
// token pair {-1024 * sum(staged x) of both, sum(x) of both}: K/64 x TP/2
// float4, so the epilogue's two tokens are one packed FMA operand][barriers]
__host__ __device__ inline GsLayout gs_layout(int K, int R, int TP) {
    const int ngK = K / 64;
    GsLayout L;
    L.xs = (uint32_t)R * kGsStage;
    L.xc = L.xs + (uint32_t)TP * x_words_stride(K) * 4;
    L.bars = L.xc + (uint32_t)TP * ngK * 8;
    L.total = ((L.bars + (uint32_t)sizeof(GsBars) + 15) & ~15u) + 1024;
    return L;
}

__device__ __forceinline__ bool gs_wait(uint64_t* bar, uint32_t parity, int& abort_flag, uint32_t* err,
                                        uint32_t site) {
    for (uint32_t i = 0; i < kGsSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *reinterpret_cast<volatile int*>(&abort_flag)) return false;
    }
    abort_flag = 1;
    if (err && atomicOr(err, kErrMbarTimeout) == 0) {
        err[1] = site;
        err[2] = blockIdx.x;
    }
    return false;
}

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kGsConsumers * 32) : "memory"); }

__device__ __forceinline__ void prefetch_l2(const void* ptr, uint32_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(ptr) & ~uintptr_t(15);
    const uint32_t n = (uint32_t)((reinterpret_cast<uintptr_t>(ptr) + bytes - a + 15) & ~uintptr_t(15));
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
}

// job -> (group, pass, tile); tile innermost, so a CTA's contiguous job range
// shares the staged token rows of a (group, pass) across its tiles
struct GsJob {
    int group, pass, tile;
};
__device__ __forceinline__ GsJob gs_decode(const GsBars& b, int ng, int job, int ntile) {
    int lo = 0, hi = ng;  // job_start[lo] <= job < job_start[lo + 1]
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (b.job_start[mid] <= job)
            lo = mid;
        else
            hi = mid;
    }
    const int r = job - b.job_start[lo];
    return GsJob{lo, r / ntile, r - (r / ntile) * ntile};
}

// scale/bias of rows A and B for the 4 groups starting at G, packed as the
// raw 16-bit values (zero past ngK): out[0] = s_A, [1] = b_A, [2] = s_B, [3] = b_B
template <typename ST>
__device__ __forceinline__ void load_scales(const ST* s0, const ST* b0, const ST* s1, const ST* b1, int G, int ngK,
                                            bool vec, uint2 out[4]) {
    if (vec) {  // 4 groups = 8 bytes, 8-byte aligned
        out[0] = __ldg(reinterpret_cast<const uint2*>(s0 + G));
        out[1] = __ldg(reinterpret_cast<const uint2*>(b0 + G));
        out[2] = __ldg(reinterpret_cast<const uint2*>(s1 + G));
        out[3] = __ldg(reinterpret_cast<const uint2*>(b1 + G));
    } else {
        const ST* src[4] = {s0, b0, s1, b1};
#pragma unroll
        for (int a = 0; a < 4; ++a) {
            uint16_t v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                v[j] = G + j < ngK ? __ldg(reinterpret_cast<const uint16_t*>(src[a] + G + j)) : (uint16_t)0;
            out[a] = make_uint2((uint32_t)v[0] | ((uint32_t)v[1] << 16), (uint32_t)v[2] | ((uint32_t)v[3] << 16));
        }
    }
}

template <typename ST>
__device__ __forceinline__ float scale_at(const uint2& packed, int j) {
    const uint32_t w = (j < 2) ? packed.x : packed.y;
    const uint16_t bits = (j & 1) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFFu);
    ST v;
    memcpy(&v, &bits, 2);
    return scale_to_float(v);
}

// The pass's token rows into the octet-pair layout (x_words_stride(K) words
// per row), odd pairs divided by 16 for the offset-folded MMA (exact in fp16
// outside the subnormal range); rows ntok..nrows-1 are zero.  MODE 0 gathers
// hidden rows by the pairs' tokens, MODE 1 reads the pass's act rows.
__device__ __forceinline__ void stage_words_gather(const GsParams& p, uint32_t* xs, int ws, int p0, int ntok,
                                                   int nrows, int ctid, uint32_t* s_tok) {
    const int octets = p.K / 8;
    const int n = nrows * octets;
    const __half2 sixteenth = __float2half2_rn(0.0625f);
    constexpr int U = 12;  // 16 rows x 352 octets / 480 threads: every load of a restage in flight at once
    constexpr int NT = kGsConsumers * 32;
    // the pass's token ids first (one load each), so no row load waits on a pair load
    if (p.mode == 0 && ctid < ntok) s_tok[ctid] = p.pairs[p0 + ctid].token;
    consumer_bar();
    for (int base = ctid; base < n; base += U * NT) {
        uint4 raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * NT;
            raw[u] = make_uint4(0u, 0u, 0u, 0u);
            if (i < n) {
                const int tk = i / octets, o = i - tk * octets;
                if (tk < ntok) {
                    if (p.mode == 0) {
                        const uint32_t tok = s_tok[tk];
                        if (tok < (uint32_t)p.T)
                            raw[u] = __ldcg(reinterpret_cast<const uint4*>(p.x + (long long)tok * p.x_stride) + o);
                        else if (o == 0 && p.err)
                            atomicOr(p.err, kErrBadExpert);
                    } else {
                        raw[u] = __ldcg(reinterpret_cast<const uint4*>(p.x + (long long)(p0 + tk) * p.x_stride) + o);
                    }
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int i = base + u * NT;
            if (i < n) {
                const int tk = i / octets, o = i - tk * octets;
                __half h[8];
                memcpy(h, &raw[u], 16);
                uint32_t* dst = xs + tk * ws + o * 4;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    __half2 pr = __halves2half2(h[j], h[j + 4]);
                    if (j & 1) pr = __hmul2(pr, sixteenth);
                    dst[j] = *reinterpret_cast<uint32_t*>(&pr);
                }
            }
        }
    }
}

// Per (token, group): {-1024 * sum(staged), sum(x)}; the odd pairs were staged
// divided by 16, so sum(x) = sum(staged) + 15 * sum(staged odd pairs).  One
// thread per item (32 staged words = eight 16-byte loads, started at a
// thread-dependent chunk so a quarter-warp reads distinct banks).
__device__ __forceinline__ void stage_xc(const uint32_t* xs, int ws, int ntok, int ngK, int TP, float2* xc, int ctid) {
    for (int i = ctid; i < ntok * ngK; i += kGsConsumers * 32) {
        const int tk = i / ngK, G = i - tk * ngK;
        const uint4* w = reinterpret_cast<const uint4*>(xs + tk * ws + G * 32);
        float ev = 0.f, od = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint4 v = w[(k + i) & 7];
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
            const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
            const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
            ev += (a.x + a.y) + (c.x + c.y);  // words 4q, 4q+2: even pairs
            od += (b.x + b.y) + (d.x + d.y);  // words 4q+1, 4q+3: odd pairs (staged / 16)
        }
        const float s = ev + od;
        // a token pair's four floats: {-1024 * sum_even_tok, -1024 * sum_odd_tok, sum_x even, sum_x odd}
        float* xf = reinterpret_cast<float*>(xc) + (size_t)(G * TP + (tk & ~1)) * 2 + (tk & 1);
        xf[0] = -1024.f * s;
        xf[2] = s + 15.f * od;
    }
}

// d = a * b + c on two fp32 lanes at once (one packed FMA, sm_100)
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

// One ring stage (4 groups of 64 codes) of a consumer warp: rows A and B of
// the warp x NB blocks of 8 tokens.  (A FULL variant without the G < ngK test
// spilled registers and ran slower.)
template <typename ST, int NB>
__device__ __forceinline__ void gs_stage(const uint8_t* sbase, int offA, int offB, const uint32_t* xs, int ws,
                                         const float2* xc, int TP, int st, int ngK, int g, int t, const uint2 scl[4],
                                         float acc[2][4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int G = 4 * st + j;
        if (G >= ngK) break;
        const int o = ((((j * 2 + (t >> 1)) ^ g) & 7) << 4) + (t & 1) * 8;
        const uint2 wa = *reinterpret_cast<const uint2*>(sbase + offA + o);
        const uint2 wb = *reinterpret_cast<const uint2*>(sbase + offB + o);
        uint32_t pa0[4], pa1[4], pb0[4], pb1[4];
        dq4_folded(wa.x, pa0);
        dq4_folded(wa.y, pa1);
        dq4_folded(wb.x, pb0);
        dq4_folded(wb.y, pb1);
        const float sa = scale_at<ST>(scl[0], j), ba = scale_at<ST>(scl[1], j);
        const float sb = scale_at<ST>(scl[2], j), bb = scale_at<ST>(scl[3], j);
        const float2 sa2 = make_float2(sa, sa), ba2 = make_float2(ba, ba);
        const float2 sb2 = make_float2(sb, sb), bb2 = make_float2(bb, bb);
#pragma unroll
        for (int b = 0; b < NB; ++b) {
            const uint4* xp = reinterpret_cast<const uint4*>(xs + (b * 8 + g) * ws + (G * 8 + 2 * t) * 4);
            const uint4 x0 = xp[0], x1 = xp[1];
            const float4 xv = *reinterpret_cast<const float4*>(xc + G * TP + b * 8 + 2 * t);
            // the chain starts at -1024 * sum(staged x) and ends at the group's dot
            float c[4] = {xv.x, xv.y, xv.x, xv.y};
            mma16816(c, pa0[0], pb0[0], pa0[1], pb0[1], x0.x, x0.y);
            mma16816(c, pa0[2], pb0[2], pa0[3], pb0[3], x0.z, x0.w);
            mma16816(c, pa1[0], pb1[0], pa1[1], pb1[1], x1.x, x1.y);
            mma16816(c, pa1[2], pb1[2], pa1[3], pb1[3], x1.z, x1.w);
            const float2 sx = make_float2(xv.z, xv.w);
            float2 a0 = ffma2(ba2, sx, make_float2(acc[b][0], acc[b][1]));
            float2 a1 = ffma2(bb2, sx, make_float2(acc[b][2], acc[b][3]));
            a0 = ffma2(sa2, make_float2(c[0], c[1]), a0);
            a1 = ffma2(sb2, make_float2(c[2], c[3]), a1);
            acc[b][0] = a0.x;
            acc[b][1] = a0.y;
            acc[b][2] = a1.x;
            acc[b][3] = a1.y;
        }
    }
}

template <typename ST>
__global__ void __launch_bounds__(kGsThreads, 1) grouped_stream_kernel(const __grid_constant__ GsParams p) {
    extern __shared__ uint8_t gs_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gs_raw) + 1023) & ~uintptr_t(1023));
    const GsLayout L = gs_layout(p.K, p.R, p.TP);
    uint8_t* ring = sm;
    uint32_t* xs = reinterpret_cast<uint32_t*>(sm + L.xs);
    float2* xc = reinterpret_cast<float2*>(sm + L.xc);
    GsBars& sh = *reinterpret_cast<GsBars*>(sm + L.bars);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ uint32_t s_tok[32];  // the staged pass's token ids
    const int ngK = p.K >> 6, nst = (ngK + 3) >> 2, R = p.R, TP = p.TP;
    const int ws = x_words_stride(p.K);
    const int rows_out = p.mode == 0 ? p.F : p.D;  // output rows per expert
    const int tile_rows = p.mode == 0 ? kGsTile0 : kGsTile1;

    griddep_wait();  // the groups / acts come from the previous launch
    const int ng = min((int)__ldg(p.n_groups), kGsMaxGroups);
    if (tid == 0) {
        for (int s = 0; s < R; ++s) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kGsConsumers);
        }
        sh.abort_flag = 0;
        sh.stop = 0;
        fence_mbar_init();
        prefetch_tmap(&p.map0);
        if (p.mode == 0) prefetch_tmap(&p.map1);
    }
    for (int g = tid; g < ng; g += blockDim.x) {
        const tf_moe_group gr = p.groups[g];
        int np = ((int)gr.pair_count + TP - 1) / TP;
        if (gr.expert >= (uint32_t)p.E) {
            np = 0;
            if (p.err && blockIdx.x == 0) atomicOr(p.err, kErrBadExpert);
        }
        sh.passes[g] = np;
    }
    __syncthreads();
    if (tid == 0) {
        int acc = 0;
        for (int g = 0; g < ng; ++g) {
            sh.job_start[g] = acc;
            acc += sh.passes[g] * p.ntile;
        }
        sh.job_start[ng] = acc;
    }
    __syncthreads();
    const int njobs = sh.job_start[ng];
    // this CTA's contiguous, balanced range of jobs
    const int j0 = (int)((long long)njobs * blockIdx.x / gridDim.x);
    const int j1 = (int)((long long)njobs * (blockIdx.x + 1) / gridDim.x);

    if (warp == 0) {
        // ---------------- loader (one thread) ----------------
        if (lane == 0) {
            int slot = 0;
            uint32_t ph = 0;  // ring position as (slot, wrap parity): no division in the loop
            for (int job = j0; job < j1; ++job) {
                const GsJob J = gs_decode(sh, ng, job, p.ntile);
                const tf_moe_group gr = p.groups[J.group];
                const uint8_t* blob = p.pool + (size_t)gr.expert * p.stride;
                const int r0 = J.tile * tile_rows;
                const int rows = min(tile_rows, rows_out - r0);
                const uint32_t sb = (uint32_t)rows * ngK * 2;
                prefetch_l2(blob + p.os0 + (size_t)r0 * ngK * 2, sb);
                prefetch_l2(blob + p.ob0 + (size_t)r0 * ngK * 2, sb);
                if (p.mode == 0) {
                    prefetch_l2(blob + p.os1 + (size_t)r0 * ngK * 2, sb);
                    prefetch_l2(blob + p.ob1 + (size_t)r0 * ngK * 2, sb);
                }
                bool ok = true;
                for (int st = 0; st < nst; ++st) {
                    if (!(ok = gs_wait(&sh.empty[slot], ph ^ 1u, sh.abort_flag, p.err, __LINE__))) break;
                    uint8_t* dst = ring + slot * kGsStage;
                    mbar_arrive_expect_tx(&sh.full[slot], kGsStage);
                    if (p.mode == 0) {
                        tma_load_3d(dst, &p.map0, st * 128, r0, (int)gr.expert, &sh.full[slot]);
                        tma_load_3d(dst + kGsBox, &p.map1, st * 128, r0, (int)gr.expert, &sh.full[slot]);
                    } else {
                        tma_load_3d(dst, &p.map0, st * 128, r0, (int)gr.expert, &sh.full[slot]);  // 240 rows
                    }
                    if (++slot == R) {
                        slot = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
            }
        }
    } else {
        // ---------------- 15 consumer warps ----------------
        const int w = warp - 1;
        const int g = lane >> 2, t = lane & 3;
        const int ctid = tid - 32;
        // this lane's A rows inside a stage: MODE 0 gate row 8w+g (box 0) and
        // up row 8w+g (box 1); MODE 1 rows 16w+g and 16w+g+8
        const int offA = p.mode == 0 ? (8 * w + g) * 128 : (16 * w + g) * 128;
        const int offB = p.mode == 0 ? kGsBox + (8 * w + g) * 128 : (16 * w + g + 8) * 128;
        int slot = 0;
        uint32_t ph = 0;
        int staged_group = -1, staged_pass = -1;
        for (int job = j0; job < j1; ++job) {
            const GsJob J = gs_decode(sh, ng, job, p.ntile);
            const tf_moe_group gr = p.groups[J.group];
            const int p0 = (int)gr.pair_start + J.pass * TP;
            const int ntok = min(TP, (int)gr.pair_count - J.pass * TP);
            const int nblk = (ntok + 7) >> 3;
            if (J.group != staged_group || J.pass != staged_pass) {
                consumer_bar();  // every consumer is done with the previous token rows
                if (ctid == 0) sh.stop = *reinterpret_cast<volatile int*>(&sh.abort_flag);
                stage_words_gather(p, xs, ws, p0, ntok, nblk * 8, ctid, s_tok);
                consumer_bar();
                stage_xc(xs, ws, nblk * 8, ngK, TP, xc, ctid);
                consumer_bar();
                staged_group = J.group;
                staged_pass = J.pass;
            }
            if (sh.stop) break;  // identical for every consumer: read after the barriers above
            const uint8_t* blob = p.pool + (size_t)gr.expert * p.stride;
            const int r0 = J.tile * tile_rows;
            const int rowA = p.mode == 0 ? r0 + 8 * w + g : r0 + 16 * w + g;
            const int rowB = p.mode == 0 ? rowA : rowA + 8;
            const bool okA = rowA < rows_out, okB = rowB < rows_out;
            const ST* sA = reinterpret_cast<const ST*>(blob + p.os0) + (size_t)(okA ? rowA : 0) * ngK;
            const ST* bA = reinterpret_cast<const ST*>(blob + p.ob0) + (size_t)(okA ? rowA : 0) * ngK;
            const ST* sB = reinterpret_cast<const ST*>(blob + (p.mode == 0 ? p.os1 : p.os0)) + (size_t)(okB ? rowB : 0) * ngK;
            const ST* bB = reinterpret_cast<const ST*>(blob + (p.mode == 0 ? p.ob1 : p.ob0)) + (size_t)(okB ? rowB : 0) * ngK;
            const bool vec = (ngK & 3) == 0 && ((reinterpret_cast<uintptr_t>(sA) | reinterpret_cast<uintptr_t>(bA) |
                                                 reinterpret_cast<uintptr_t>(sB) | reinterpret_cast<uintptr_t>(bB)) & 7u) == 0;
            float acc[2][4];
#pragma unroll
            for (int b = 0; b < 2; ++b)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[b][i] = 0.f;
            uint2 scl[4], nscl[4];
            load_scales<ST>(sA, bA, sB, bB, 0, ngK, vec, scl);
            bool ok = true;
            for (int st = 0; st < nst; ++st) {
                if (st + 1 < nst) load_scales<ST>(sA, bA, sB, bB, 4 * (st + 1), ngK, vec, nscl);
                if (!(ok = gs_wait(&sh.full[slot], ph, sh.abort_flag, p.err, __LINE__))) break;
                const uint8_t* sbase = ring + slot * kGsStage;
                // the block count as a template argument: no per-group test of it
                if (nblk == 2)
                    gs_stage<ST, 2>(sbase, offA, offB, xs, ws, xc, TP, st, ngK, g, t, scl, acc);
                else
                    gs_stage<ST, 1>(sbase, offA, offB, xs, ws, xc, TP, st, ngK, g, t, scl, acc);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.empty[slot]);
                if (++slot == R) {
                    slot = 0;
                    ph ^= 1u;
                }
#pragma unroll
                for (int a = 0; a < 4; ++a) scl[a] = nscl[a];
            }
            if (!ok) continue;  // the abort is seen at the next restage, or the range ends
            // epilogue from registers: the lane holds rows (A, B) x tokens (2t, 2t+1) of each block
#pragma unroll
            for (int b = 0; b < 2; ++b) {
                if (b >= nblk) break;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int tk = b * 8 + 2 * t + h;
                    if (tk >= ntok) continue;
                    if (p.mode == 0) {
                        if (okA)
                            p.acts[(long long)(p0 + tk) * p.F + rowA] =
                                __float2half_rn(gelu_tanh(acc[b][h]) * acc[b][2 + h]);
                    } else {
                        const tf_token_expert_pair pr = p.pairs[p0 + tk];
                        __half* dst = p.partials + ((long long)pr.token * p.top_k + pr.rank) * p.D;
                        if (okA) dst[rowA] = __float2half_rn(acc[b][h]);
                        if (okB) dst[rowB] = __float2half_rn(acc[b][2 + h]);
                    }
                }
            }
        }
    }
    __syncthreads();
}

bool gs_map(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint64_t depth,
            uint64_t depth_stride, uint32_t box_rows) {
    memset(m, 0, sizeof(*m));
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(base) & 15u) || row_bytes % 16 || rows == 0 || depth == 0) return false;
    const uint64_t ds = depth > 1 ? depth_stride : row_bytes * rows;
    if (ds % 16 || ds >= (1ull << 40)) return false;
    cuuint64_t dims[3] = {row_bytes, rows, depth};
    cuuint64_t strides[2] = {row_bytes, ds};
    cuuint32_t box[3] = {128, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename ST>
tf_status launch_gs(tf_context* ctx, GsParams p, cudaStream_t s, const char* name) {
    // tokens per pass: 16 when the ring keeps at least 3 stages, else 8
    p.R = 0;
    const char* tpe = getenv("TFCUDA_GS_TP");  // 8 or 16 forces the pass width (read per call)
    const int tp_force = tpe ? atoi(tpe) : 0;
    for (int tp : {16, 8}) {
        if (tp_force && tp != tp_force) continue;
        const GsLayout L0 = gs_layout(p.K, 0, tp);
        const long long left = (long long)kGsSmemLimit - (long long)L0.total;
        const int R = (int)std::min<long long>(kGsMaxR, left / kGsStage);
        if (R >= 3 || (tp == 8 && R >= 2)) {
            p.TP = tp;
            p.R = R;
            break;
        }
    }
    if (p.R < 2) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: K too large for the grouped stream kernel", name);
    const GsLayout L = gs_layout(p.K, p.R, p.TP);
    const void* fn = reinterpret_cast<const void*>(&grouped_stream_kernel<ST>);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return cuda_check(ctx, e, name);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ctx->num_sms);
    cfg.blockDim = dim3(kGsThreads);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_check(ctx, cudaLaunchKernelEx(&cfg, grouped_stream_kernel<ST>, p), name);
}

}  // namespace

namespace tf {

tf_status grouped_stream(tf_context* ctx, const uint8_t* pool, uint64_t stride, uint32_t num_experts,
                         const tf_expert_offsets* off, const tf_token_expert_pair* pairs, const tf_moe_group* groups,
                         const uint32_t* n_groups, const __half* hidden, uint32_t hidden_stride, __half* acts,
                         __half* partials, uint32_t T, uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st,
                         cudaStream_t s, const char* name) {
    if (num_experts > (uint32_t)kGsMaxGroups || d % 64 || f % 64 || hidden_stride % 8 ||
        (reinterpret_cast<uintptr_t>(hidden) & 15u) || (reinterpret_cast<uintptr_t>(acts) & 15u))
        return TF_ERR_UNSUPPORTED_SHAPE;
    GsParams p;
    memset(&p, 0, sizeof(p));
    p.pool = pool;
    p.stride = stride;
    p.groups = groups;
    p.n_groups = n_groups;
    p.pairs = pairs;
    p.acts = acts;
    p.partials = partials;
    p.E = (int)num_experts;
    p.D = (int)d;
    p.F = (int)f;
    p.top_k = (int)top_k;
    p.T = (int)T;
    p.err = ctx->d_err;
    // phase 1: gate/up over K = d, 120 features per job
    p.mode = 0;
    p.K = (int)d;
    p.x = hidden;
    p.x_stride = hidden_stride;
    p.os0 = off->gate_s;
    p.ob0 = off->gate_b;
    p.os1 = off->up_s;
    p.ob1 = off->up_b;
    p.ntile = (int)((f + kGsTile0 - 1) / kGsTile0);
    if (!gs_map(&p.map0, pool + off->gate_w, d / 2, f, num_experts, stride, kGsTile0) ||
        !gs_map(&p.map1, pool + off->up_w, d / 2, f, num_experts, stride, kGsTile0))
        return TF_ERR_UNSUPPORTED_SHAPE;
    tf_status rc = st == TF_SCALE_BF16 ? launch_gs<__nv_bfloat16>(ctx, p, s, name) : launch_gs<__half>(ctx, p, s, name);
    if (rc != TF_OK) return rc;
    // phase 2: down over K = f on the acts, 240 rows per job
    p.mode = 1;
    p.K = (int)f;
    p.x = acts;
    p.x_stride = f;
    p.os0 = off->down_s;
    p.ob0 = off->down_b;
    p.os1 = p.ob1 = 0;
    p.ntile = (int)((d + kGsTile1 - 1) / kGsTile1);
    if (!gs_map(&p.map0, pool + off->down_w, f / 2, d, num_experts, stride, kGsTile1)) return TF_ERR_UNSUPPORTED_SHAPE;
    memset(&p.map1, 0, sizeof(p.map1));
    return st == TF_SCALE_BF16 ? launch_gs<__nv_bfloat16>(ctx, p, s, name) : launch_gs<__half>(ctx, p, s, name);
}

}  // namespace tf
