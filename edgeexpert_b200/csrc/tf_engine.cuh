// tf_engine.cuh -- the streaming tile engine behind every quantized GEMV-like
// kernel of this library (plain int4/int8 GEMV, router logits, routed and
// shared expert gate/up, down + combine).
//
// Work decomposition
//   job   : 16 output rows of one "policy" (e.g. 8 gate + 8 up rows of one
//           expert, or 16 down rows summed over all selected experts).
//   seg   : one 16-row weight tile feeding the job (rows 0-7 and 8-15 may come
//           from two matrices), with its own activation vector and multiplier.
//   unit  : one K-chunk of one seg (11 groups int4 = 352 B/row, 6 groups
//           int8 = 384 B/row).  A unit is what one warp streams and reduces.
//   super-job: J consecutive jobs whose J*U units exactly cover the 8 warps
//           of a CTA when U divides 8, else one job whose units are spread
//           over the warps.  Partial sums are reduced in shared memory in a
//           fixed warp order, so results are deterministic.
//
// Each warp keeps a private ring of NS shared-memory stages.  Lane 0 arms the
// stage's mbarrier with the byte count, lanes 0..15 each issue one
// cp.async.bulk for one weight row, and the warp computes on the stage once
// the mbarrier phase flips (bounded wait; a timeout sets an error bit and the
// unit is skipped).  Loads run NS units ahead across job boundaries, so HBM
// stays busy through the per-super-job barrier.
#pragma once
#include "tf_device.cuh"

namespace tf {

#ifdef TF_TRACE
// Debug-only phase timestamps (%globaltimer, ns) of thread 0 of each CTA.
__device__ unsigned long long g_tf_trace[1024][8];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#define TF_T(i) do { if (threadIdx.x == 0 && blockIdx.x < 1024) g_tf_trace[blockIdx.x][i] = gtimer(); } while (0)
#else
#define TF_T(i) do {} while (0)
#endif

struct SegDesc {
    const uint8_t* WA;
    const void* SA;
    const void* BA;
    int rowA, nA;  // stage rows 0..7  <- rows rowA .. rowA+nA-1 of A
    const uint8_t* WB;
    const void* SB;
    const void* BB;
    int rowB, nB;  // stage rows 8..15 <- rows rowB .. rowB+nB-1 of B
    int K, bits;
    const uint32_t* xs;  // staged activation (octet-pair layout), token 0
    const float* xsum;   // per-group sums, token 0
    int xws;             // words between tokens in xs
    int ntok;            // tokens (MMA columns) carried by xs
    float mult;          // multiplier applied to this seg's contribution
};

__host__ __device__ inline int chunk_groups(int bits) { return bits == 4 ? kChunkGroups4 : kChunkGroups8; }
__host__ __device__ inline int group_bytes(int bits) { return bits == 4 ? 32 : 64; }
__host__ __device__ inline int row_bytes(int K, int bits) { return bits == 4 ? K / 2 : K; }
__host__ __device__ inline int units_for_K(int K, int bits) {
    const int ng = K / kGroup, cg = chunk_groups(bits);
    return (ng + cg - 1) / cg;
}
__host__ __device__ inline int stage_stride(int bits) { return bits == 4 ? kStageStride4 : kStageStride8; }
__host__ __device__ inline int superjob_J(int U) { return (U <= kWarps && kWarps % U == 0) ? kWarps / U : 1; }

// Global address of the unit's first scale (a=0) or bias (a=1) of stage row r.
__device__ __forceinline__ const uint8_t* scale_src(const SegDesc& sd, int r, int a, int G0) {
    const int ngK = sd.K / kGroup;
    const void* base = r < 8 ? (a ? sd.BA : sd.SA) : (a ? sd.BB : sd.SB);
    const int row = r < 8 ? sd.rowA + r : sd.rowB + r - 8;
    return static_cast<const uint8_t*>(base) + ((size_t)row * ngK + G0) * 2;
}

// ---------------------------------------------------------------------------
// Unit compute: fresh accumulator over the unit's groups.
//   c[0] row g   token 2t      c[1] row g   token 2t+1
//   c[2] row g+8 token 2t      c[3] row g+8 token 2t+1
// ---------------------------------------------------------------------------
template <typename ST, int BITS>
__device__ __forceinline__ void compute_unit(const uint8_t* __restrict__ stage, const SegDesc& sd, int chunk,
                                             float out[4], int lane, uint32_t* err) {
    (void)err;
    const int g = lane >> 2, t = lane & 3;
    const int ngK = sd.K / kGroup;
    const int cg = chunk_groups(BITS);
    const int G0 = chunk * cg;
    const int G1 = min(ngK, G0 + cg);
    const int stride = stage_stride(BITS);
    const bool va = g < sd.nA, vb = g < sd.nB;
    // scale/bias slots of rows g and g+8 (byte offset = the copy's misalignment)
    auto slot = [&](int r, int a) {
        const uint8_t* src = scale_src(sd, r, a, G0);
        return reinterpret_cast<const ST*>(stage + kScaleOff + (r * 2 + a) * kScaleSlot +
                                           (reinterpret_cast<uintptr_t>(src) & 3u));
    };
    const ST* sA = slot(g, 0);
    const ST* bA = slot(g, 1);
    const ST* sB = slot(g + 8, 0);
    const ST* bB = slot(g + 8, 1);
    const bool tokv = g < sd.ntok;
    const bool xv0 = 2 * t < sd.ntok, xv1 = 2 * t + 1 < sd.ntok;
    const uint32_t* xrow = sd.xs + g * sd.xws;
    const float* xs0 = sd.xsum + (2 * t) * ngK;
    const float* xs1 = sd.xsum + (2 * t + 1) * ngK;
    const uint8_t* rowa = stage + g * stride;
    const uint8_t* rowb = stage + (g + 8) * stride;

    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    constexpr int kCG = BITS == 4 ? kChunkGroups4 : kChunkGroups8;
    // Fully unrolled over the unit's groups so the scale/bias loads of every
    // group are issued before the first MMA instead of one group at a time.
#pragma unroll
    for (int gl = 0; gl < kCG; ++gl) {
        const int G = G0 + gl;
        if (G >= G1) break;
        uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
        if (tokv) {
            const uint4* xp = reinterpret_cast<const uint4*>(xrow + (G * 8 + 2 * t) * 4);
            if (TF_ALIGNED(xp, 16, err, 1)) {
                x0 = xp[0];
                x1 = xp[1];
            }
        }
        uint32_t pa0[4], pa1[4], pb0[4], pb1[4];
        if (BITS == 4) {
            if (!TF_ALIGNED(rowa + gl * 32 + t * 8, 8, err, 2) || !TF_ALIGNED(rowb + gl * 32 + t * 8, 8, err, 3))
                continue;
            const uint2 wa = *reinterpret_cast<const uint2*>(rowa + gl * 32 + t * 8);
            const uint2 wb = *reinterpret_cast<const uint2*>(rowb + gl * 32 + t * 8);
            dq4(wa.x, pa0);
            dq4(wa.y, pa1);
            dq4(wb.x, pb0);
            dq4(wb.y, pb1);
        } else {
            if (!TF_ALIGNED(rowa + gl * 64 + t * 16, 16, err, 4) || !TF_ALIGNED(rowb + gl * 64 + t * 16, 16, err, 5))
                continue;
            const uint4 wa = *reinterpret_cast<const uint4*>(rowa + gl * 64 + t * 16);
            const uint4 wb = *reinterpret_cast<const uint4*>(rowb + gl * 64 + t * 16);
            dq8(wa.x, wa.y, pa0);
            dq8(wa.z, wa.w, pa1);
            dq8(wb.x, wb.y, pb0);
            dq8(wb.z, wb.w, pb1);
        }
        float c[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(c, pa0[0], pb0[0], pa0[1], pb0[1], x0.x, x0.y);
        mma16816(c, pa0[2], pb0[2], pa0[3], pb0[3], x0.z, x0.w);
        mma16816(c, pa1[0], pb1[0], pa1[1], pb1[1], x1.x, x1.y);
        mma16816(c, pa1[2], pb1[2], pa1[3], pb1[3], x1.z, x1.w);
        const float sa = va ? scale_to_float(sA[gl]) : 0.f;
        const float ba = va ? scale_to_float(bA[gl]) : 0.f;
        const float sb = vb ? scale_to_float(sB[gl]) : 0.f;
        const float bb = vb ? scale_to_float(bB[gl]) : 0.f;
        const float s0 = xv0 ? xs0[G] : 0.f;
        const float s1 = xv1 ? xs1[G] : 0.f;
        acc[0] = fmaf(sa, c[0], acc[0]);
        acc[0] = fmaf(ba, s0, acc[0]);
        acc[1] = fmaf(sa, c[1], acc[1]);
        acc[1] = fmaf(ba, s1, acc[1]);
        acc[2] = fmaf(sb, c[2], acc[2]);
        acc[2] = fmaf(bb, s0, acc[2]);
        acc[3] = fmaf(sb, c[3], acc[3]);
        acc[3] = fmaf(bb, s1, acc[3]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = acc[i];
}

// Bytes one lane copies for one row of a unit, and the row's source address.
__device__ __forceinline__ void unit_row(const SegDesc& sd, int chunk, int r, const uint8_t** src, int* bytes,
                                         bool* valid) {
    const int ngK = sd.K / kGroup;
    const int cg = chunk_groups(sd.bits);
    const int G0 = chunk * cg;
    const int G1 = min(ngK, G0 + cg);
    const int gb = group_bytes(sd.bits);
    const int rb = row_bytes(sd.K, sd.bits);
    *bytes = (G1 - G0) * gb;
    if (r < 8) {
        *valid = r < sd.nA;
        *src = sd.WA + (size_t)(sd.rowA + r) * rb + (size_t)G0 * gb;
    } else {
        *valid = (r - 8) < sd.nB;
        *src = sd.WB + (size_t)(sd.rowB + r - 8) * rb + (size_t)G0 * gb;
    }
}

// Synchronous fallback for weight bases that are only 2-byte aligned (the
// reference accepts those, DequantInt4GEMV.swift:97-102): 16-bit loads.
__device__ __forceinline__ void unit_copy_sync(uint8_t* stage, const SegDesc& sd, int chunk, int lane) {
    const int stride = stage_stride(sd.bits);
    for (int r = 0; r < 16; ++r) {
        const uint8_t* src;
        int bytes;
        bool valid;
        unit_row(sd, chunk, r, &src, &bytes, &valid);
        if (!valid) continue;
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
        uint16_t* d16 = reinterpret_cast<uint16_t*>(stage + r * stride);
        for (int i = lane; i < bytes / 2; i += 32) d16[i] = s16[i];
    }
    const int ngK = sd.K / kGroup;
    const int G0 = chunk * chunk_groups(sd.bits);
    const int n = min(ngK, G0 + chunk_groups(sd.bits)) - G0;
    const int r = lane >> 1, a = lane & 1;
    if (r < 8 ? r < sd.nA : (r - 8) < sd.nB) {
        const uint8_t* src = scale_src(sd, r, a, G0);
        uint8_t* dst = stage + kScaleOff + lane * kScaleSlot + (reinterpret_cast<uintptr_t>(src) & 3u);
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
        uint16_t* d16 = reinterpret_cast<uint16_t*>(dst);
        for (int i = 0; i < n; ++i) d16[i] = s16[i];
    }
}

__device__ __forceinline__ void unit_issue(uint8_t* stage, uint64_t* bar, const SegDesc& sd, int chunk,
                                           int lane, uint32_t* err) {
    (void)err;
    const int stride = stage_stride(sd.bits);
    const int ngK = sd.K / kGroup;
    const int cg = chunk_groups(sd.bits);
    const int G0 = chunk * cg;
    const int gb = group_bytes(sd.bits);
    const int bytes = (min(ngK, G0 + cg) - G0) * gb;
    if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(bytes * (sd.nA + sd.nB)));
    __syncwarp();
    if (lane < 16) {
        const int rb = row_bytes(sd.K, sd.bits);
        const bool lo = lane < 8;
        const int r = lo ? lane : lane - 8;
        const bool valid = r < (lo ? sd.nA : sd.nB);
        const uint8_t* src = (lo ? sd.WA + (size_t)(sd.rowA + r) * rb : sd.WB + (size_t)(sd.rowB + r) * rb) +
                             (size_t)G0 * gb;
        if (valid && TF_ALIGNED(src, 16, err, 6) && TF_ALIGNED(stage + lane * stride, 16, err, 7) &&
            TF_ALIGNED((const void*)(uintptr_t)bytes, 16, err, 8))
            bulk_g2s(stage + lane * stride, src, (uint32_t)bytes, bar);
    }
    {   // scales/biases: lane = 2*row + {0: scale, 1: bias}, 4-byte async copies
        const int r = lane >> 1, a = lane & 1;
        const bool valid = r < 8 ? r < sd.nA : (r - 8) < sd.nB;
        if (valid) {
            const uint8_t* src = scale_src(sd, r, a, G0);
            const uint8_t* al = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(src) & ~uintptr_t(3));
            const int nbytes = (min(ngK, G0 + cg) - G0) * 2 + (int)(src - al);
            uint8_t* dst = stage + kScaleOff + lane * kScaleSlot;
            for (int i = 0; i < (nbytes + 3) / 4; ++i) cp_async4(dst + 4 * i, al + 4 * i);
        }
        cp_async_mbar_arrive(bar);
    }
}

// Host-computed schedule: up to two job ranges (e.g. routed and shared
// experts) with U units per job, J jobs per super-job and S super-jobs each.
struct Sched {
    int nj[2], U[2], J[2], S[2];
    int S_total;
};

inline Sched make_sched(int nj0, int U0, int nj1 = 0, int U1 = 1) {
    Sched s;
    s.nj[0] = nj0;
    s.U[0] = U0;
    s.J[0] = superjob_J(U0);
    s.S[0] = nj0 > 0 ? (nj0 + s.J[0] - 1) / s.J[0] : 0;
    s.nj[1] = nj1;
    s.U[1] = U1;
    s.J[1] = superjob_J(U1);
    s.S[1] = nj1 > 0 ? (nj1 + s.J[1] - 1) / s.J[1] : 0;
    s.S_total = s.S[0] + s.S[1];
    return s;
}

struct SuperJob {
    int j0, j1, J, U;  // jobs [j0, j1), U units per job, J jobs per super-job
};

__device__ __forceinline__ SuperJob decode_superjob(const Sched& sc, int sj) {
    const int r = sj >= sc.S[0] ? 1 : 0;
    const int local = sj - (r ? sc.S[0] : 0);
    const int base = r ? sc.nj[0] : 0;
    SuperJob s;
    s.J = sc.J[r];
    s.U = sc.U[r];
    s.j0 = base + local * s.J;
    s.j1 = base + min(sc.nj[r], (local + 1) * s.J);
    return s;
}

// Unit index v (0..J*U-1) handled by warp w at step i, or -1.
__device__ __forceinline__ int warp_unit(const SuperJob& s, int w, int i) {
    const int v = w + kWarps * i;
    if (v >= s.J * s.U) return -1;
    if (s.j0 + v / s.U >= s.j1) return -1;
    return v;
}

// Shared-memory layout of the engine (bytes):
//   [stages: kWarps * ns * kStageBytes][red: 2 * kWarps * 32 * 4 floats]
//   [bars: kWarps * ns u64][x area: Pol::x_bytes(p)]
__host__ __device__ inline size_t engine_fixed_smem(int ns) {
    return (size_t)kWarps * ns * kStageBytes + 2 * kWarps * 32 * 4 * sizeof(float) + kWarps * ns * 8;
}

template <class Pol, typename ST>
__global__ void __launch_bounds__(kWarps * 32, 1) engine_kernel(const typename Pol::Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int ns = p.ns;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint8_t* stages = smem;
    float* red = reinterpret_cast<float*>(smem + (size_t)kWarps * ns * kStageBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + 2 * kWarps * 32 * 4);
    uint8_t* xarea = reinterpret_cast<uint8_t*>(bars + kWarps * ns);
    uint8_t* my_stages = stages + (size_t)warp * ns * kStageBytes;
    uint64_t* my_bars = bars + warp * ns;

    TF_T(0);
    if (lane == 0)
        for (int s = 0; s < ns; ++s) mbar_init(&my_bars[s], kStageArrivals);
    fence_mbar_init();
    Pol::stage_pre(p, threadIdx.x);
    __syncthreads();
    TF_T(1);

    const int S = p.sched.S_total;

    // Load cursor: same unit sequence as the compute loop below.
    int l_sj = blockIdx.x, l_i = 0;
    auto load_next = [&](int slot) -> void {
        while (l_sj < S) {
            const SuperJob sj = decode_superjob(p.sched, l_sj);
            const int v = warp_unit(sj, warp, l_i);
            if (v < 0) {
                l_sj += gridDim.x;
                l_i = 0;
                continue;
            }
            ++l_i;
            SegDesc sd;
            int chunk;
            if (Pol::unit(p, sj.j0 + v / sj.U, v % sj.U, &sd, &chunk)) {
                unit_issue(my_stages + (size_t)slot * kStageBytes, &my_bars[slot], sd, chunk, lane, p.err);
            } else {  // keep the phase sequence intact
                if (lane == 0) mbar_arrive_expect_tx(&my_bars[slot], 0);
                cp_async_mbar_arrive(&my_bars[slot]);
            }
            return;
        }
    };

    // Weight tiles do not depend on the activations: put the first NS units of
    // every warp in flight before staging the activations.
    if (p.aligned)
        for (int s = 0; s < ns; ++s) load_next(s);
    TF_T(2);
    Pol::stage_x(p, xarea, threadIdx.x, kWarps * 32);
    __syncthreads();
    TF_T(3);

    int seq = 0;
    int parity_buf = 0;
    bool dead = false;
    for (int sjx = blockIdx.x; sjx < S; sjx += gridDim.x) {
        const SuperJob sj = decode_superjob(p.sched, sjx);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0;; ++i) {
            const int v = warp_unit(sj, warp, i);
            if (v < 0) break;
            const int slot = seq % ns;
            const uint32_t ph = (uint32_t)(seq / ns) & 1u;
            uint8_t* st = my_stages + (size_t)slot * kStageBytes;
            SegDesc sd;
            int chunk;
            const bool found = Pol::unit(p, sj.j0 + v / sj.U, v % sj.U, &sd, &chunk);
            bool ready = true;
            if (p.aligned) {
                // once a wait has given up, later waits of this warp are skipped
                ready = !dead && mbar_wait_bounded(&my_bars[slot], ph, p.err);
                dead = dead || !ready;
                if (seq == 0) TF_T(4);
            } else if (found) {
                unit_copy_sync(st, sd, chunk, lane);
                __syncwarp();
            }
            if (found && ready) {
                float u[4];
                if (sd.bits == 4)
                    compute_unit<ST, 4>(st, sd, chunk, u, lane, p.err);
                else
                    compute_unit<ST, 8>(st, sd, chunk, u, lane, p.err);
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[k] = fmaf(sd.mult, u[k], acc[k]);
            }
            __syncwarp();
            if (p.aligned) load_next(slot);
            ++seq;
        }
        float* rb = red + (size_t)parity_buf * kWarps * 32 * 4;
        *reinterpret_cast<float4*>(rb + (warp * 32 + lane) * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncthreads();
        // Leaders: for J > 1 warp jj*U reduces job jj over warps jj*U..jj*U+U-1;
        // for J == 1 warp 0 reduces warps 0..min(U,8)-1.
        const int njobs = sj.j1 - sj.j0;
        const int lead_stride = sj.J > 1 ? sj.U : kWarps;
        if (warp % lead_stride == 0 && warp / lead_stride < njobs) {
            const int jj = warp / lead_stride;
            const int w0 = sj.J > 1 ? jj * sj.U : 0;
            const int wn = sj.J > 1 ? sj.U : min(sj.U, kWarps);
            float f[4] = {0.f, 0.f, 0.f, 0.f};
            for (int w = w0; w < w0 + wn; ++w) {
                const float4 q = *reinterpret_cast<const float4*>(rb + (w * 32 + lane) * 4);
                f[0] += q.x;
                f[1] += q.y;
                f[2] += q.z;
                f[3] += q.w;
            }
            Pol::epilogue(p, sj.j0 + jj, f, lane);
        }
        parity_buf ^= 1;
        TF_T(5);
    }
    TF_T(6);
}

}  // namespace tf
