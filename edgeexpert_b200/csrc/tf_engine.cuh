// tf_engine.cuh -- the streaming tile engine behind every quantized GEMV-like
// kernel of this library (plain int4/int8 GEMV, router logits, routed and
// shared expert gate/up, down + combine).
//
// Work decomposition
//   job   : 16 output rows of one "policy" (e.g. 8 gate + 8 up rows of one
//           expert, or 16 down rows summed over all selected experts).
//   seg   : one 16-row weight tile feeding the job (rows 0-7 and 8-15 may come
//           from two matrices), with its own activation vector and multiplier.
//   unit  : up to kMaxBoxes x 128 bytes of every row of one seg.  A unit is
//           what one warp streams into one shared-memory stage and reduces.
//   super-job: J consecutive jobs whose J*U units exactly cover the warps of a
//           CTA when U divides kWarps, else one job whose units are spread
//           over the warps.  Partial sums are reduced in shared memory in a
//           fixed warp order, so results are deterministic.
//
// Each warp owns one stage.  Lane 0 arms the stage's mbarrier with the byte
// count; lanes 0..5 / 8..13 each issue one 2-D TMA box (8 rows x 128 B,
// 128-byte swizzle) for the two half-tiles; lanes 16..19 bulk-copy the rows'
// scales and biases (whole rows, 8 rows at a time).  The warp computes once
// the phase flips (bounded wait; a timeout sets an error bit and the unit is
// skipped) and immediately re-arms the stage with its next unit, so every
// warp keeps one unit in flight across job boundaries.
#pragma once
#include <cuda.h>

#include <type_traits>

#include "tf_device.cuh"

namespace tf {

#ifdef TF_TRACE
// Debug-only phase timestamps (%globaltimer, ns) of thread 0 of each CTA.
__device__ unsigned long long g_tf_trace[1024][16];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#define TF_TW(i)                                                                            \
    do {                                                                                    \
        if ((threadIdx.x & 31) == 0 && blockIdx.x < 1024 && (threadIdx.x >> 5) == 0)       \
            g_tf_trace[blockIdx.x][i] = gtimer();                                           \
    } while (0)
#define TF_T(i)                                                                          \
    do {                                                                                 \
        if (threadIdx.x == 0 && blockIdx.x < 1024) g_tf_trace[blockIdx.x][i] = gtimer(); \
    } while (0)
#else
#define TF_TW(i) \
    do {         \
    } while (0)
#define TF_T(i) \
    do {        \
    } while (0)
#endif

struct SegDesc {
    const CUtensorMap* mapA;  // rows 0..7 of the tile: rows rowA.. of depth eA
    const CUtensorMap* mapB;  // rows 8..15: rows rowB.. of depth eB
    int eA, eB;
    int rowA, nA, rowB, nB;   // valid rows per half (0..8)
    const uint8_t* WA;        // row 0 of the A / B matrix (fallback copy path)
    const uint8_t* WB;
    const void* SA;           // scales / biases, row 0 of each matrix
    const void* BA;
    const void* SB;
    const void* BB;
    int K, bits;
    const uint32_t* xs;  // staged activation (octet-pair layout), token 0
    const float* xsum;   // per-group sums, token 0
    const float* xcorr;  // folded staging: 1024 * sum of staged values per group
    int xfold;           // 1: xs staged with odd pairs divided by 16 (stage_words fold);
                         // 2: integer layout (stage_x_int), xcorr holds the per-group x scale
    int xws;             // words between tokens in xs
    int ntok;            // tokens (MMA columns) carried by xs
    float mult;          // multiplier applied to this seg's contribution
};

__host__ __device__ inline int group_bytes(int bits) { return bits == 4 ? 32 : 64; }
__host__ __device__ inline int row_bytes(int K, int bits) { return bits == 4 ? K / 2 : K; }
__host__ __device__ inline int boxes_for_K(int K, int bits) { return (row_bytes(K, bits) + kBox - 1) / kBox; }
__host__ __device__ inline int units_for_K(int K, int bits) {
    return (boxes_for_K(K, bits) + kMaxBoxes - 1) / kMaxBoxes;
}
__host__ __device__ inline int superjob_J(int U) { return (U <= kWarps && kWarps % U == 0) ? kWarps / U : 1; }

// Byte offset inside a half-tile of byte `b` of tile row `r` (box-swizzled).
__device__ __forceinline__ int swz(int r, int b) {
    const int o = b & (kBox - 1);
    return (b >> 7) * kBoxBytes + r * kBox + ((((o >> 4) ^ r) & 7) << 4) + (o & 15);
}

// ---------------------------------------------------------------------------
// Unit compute: fresh accumulator over the unit's groups.
//   c[0] row g   token 2t      c[1] row g   token 2t+1
//   c[2] row g+8 token 2t      c[3] row g+8 token 2t+1
// ---------------------------------------------------------------------------
template <typename ST, int BITS>
__device__ __forceinline__ void compute_unit(const uint8_t* __restrict__ stage, const SegDesc& sd, int chunk,
                                             float out[4], int lane) {
    const int g = lane >> 2, t = lane & 3;
    const int ngK = sd.K / kGroup;
    constexpr int kGB = BITS == 4 ? 32 : 64;      // bytes per group per row
    constexpr int kGPU = kMaxBoxes * kBox / kGB;  // groups per unit (24 int4, 12 int8)
    const int G0 = chunk * kGPU;
    const int G1 = min(ngK, G0 + kGPU);
    const bool va = g < sd.nA, vb = g < sd.nB;
    // Scales: whole rows when they fit (ngK <= kMaxScaleGroups), else only
    // the unit's groups (row stride kGPU, index G - G0).
    const bool full = ngK <= kMaxScaleGroups;
    const int sstride = full ? ngK : kGPU;
    const int sbase = full ? 0 : G0;
    const ST* scl = reinterpret_cast<const ST*>(stage + 2 * kHalfBytes) - sbase;
    const ST* sA = scl + g * sstride;
    const ST* bA = scl + kScaleArr / 2 + g * sstride;
    const ST* sB = scl + 2 * (kScaleArr / 2) + g * sstride;
    const ST* bB = scl + 3 * (kScaleArr / 2) + g * sstride;
    const bool tokv = g < sd.ntok;
    const bool xv0 = 2 * t < sd.ntok, xv1 = 2 * t + 1 < sd.ntok;
    const uint32_t* xrow = sd.xs + g * sd.xws;
    const float* xs0 = sd.xsum + (2 * t) * ngK;
    const float* xs1 = sd.xsum + (2 * t + 1) * ngK;
    const uint8_t* halfA = stage;
    const uint8_t* halfB = stage + kHalfBytes;

    constexpr uint32_t k16x2 = 0x4C004C00u;  // fp16 16.0 in both halves
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
    for (int G = G0; G < G1; ++G) {
        const int gl = G - G0;
        uint4 x0 = make_uint4(0, 0, 0, 0), x1 = make_uint4(0, 0, 0, 0);
        if (tokv) {
            const uint4* xp = reinterpret_cast<const uint4*>(xrow + (G * 8 + 2 * t) * 4);
            x0 = xp[0];
            x1 = xp[1];
            if (sd.xfold) {  // undo the 1/16 of the odd pairs (exact)
                x0.y = hmul2_u(x0.y, k16x2);
                x0.w = hmul2_u(x0.w, k16x2);
                x1.y = hmul2_u(x1.y, k16x2);
                x1.w = hmul2_u(x1.w, k16x2);
            }
        }
        uint32_t pa0[4], pa1[4], pb0[4], pb1[4];
        if (BITS == 4) {
            const int o = swz(g, gl * 32 + t * 8);
            const uint2 wa = *reinterpret_cast<const uint2*>(halfA + o);
            const uint2 wb = *reinterpret_cast<const uint2*>(halfB + o);
            dq4(wa.x, pa0);
            dq4(wa.y, pa1);
            dq4(wb.x, pb0);
            dq4(wb.y, pb1);
        } else {
            const int o = swz(g, gl * 64 + t * 16);
            const uint4 wa = *reinterpret_cast<const uint4*>(halfA + o);
            const uint4 wb = *reinterpret_cast<const uint4*>(halfB + o);
            dq8(wa.x, wa.y, pa0);
            dq8(wa.z, wa.w, pa1);
            dq8(wb.x, wb.y, pb0);
            dq8(wb.z, wb.w, pb1);
        }
        float c[4] = {0.f, 0.f, 0.f, 0.f}, cb[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(c, pa0[0], pb0[0], pa0[1], pb0[1], x0.x, x0.y);
        mma16816(cb, pa0[2], pb0[2], pa0[3], pb0[3], x0.z, x0.w);
        mma16816(c, pa1[0], pb1[0], pa1[1], pb1[1], x1.x, x1.y);
        mma16816(cb, pa1[2], pb1[2], pa1[3], pb1[3], x1.z, x1.w);
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] += cb[i];
        const float sa = va ? scale_to_float(sA[G]) : 0.f;
        const float ba = va ? scale_to_float(bA[G]) : 0.f;
        const float sb = vb ? scale_to_float(sB[G]) : 0.f;
        const float bb = vb ? scale_to_float(bB[G]) : 0.f;
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

// ---------------------------------------------------------------------------
// Batch-1 int4 unit with offset folding and groups in the MMA's N dimension.
// Group j of each block of 8 feeds only column j of C (lanes whose column is
// not j supply zeros), so after 8 groups C[row][j] holds that group's dot
// sum_k (q + 1024 or 16q + 1024) * x_staged; the scale/bias epilogue then runs
// once per 8 groups: acc += s * (C - xcorr) + b * xsum.
// Returns the two row sums in out[0] (row g) and out[2] (row g+8) of every lane.
// ---------------------------------------------------------------------------
template <typename ST>
__device__ __forceinline__ void compute_unit_b1(const uint8_t* __restrict__ stage, const SegDesc& sd, int chunk,
                                                float out[4], int lane, const uint4* zeros) {
    const int g = lane >> 2, t = lane & 3;
    const int ngK = sd.K / kGroup;
    constexpr int kGPU = kMaxBoxes * kBox / 32;  // 24 groups per unit
    const int G0 = chunk * kGPU;
    const int G1 = min(ngK, G0 + kGPU);
    const bool va = g < sd.nA, vb = g < sd.nB;
    const bool full = ngK <= kMaxScaleGroups;
    const int sstride = full ? ngK : kGPU;
    const int sbase = full ? 0 : G0;
    const ST* scl = reinterpret_cast<const ST*>(stage + 2 * kHalfBytes) - sbase;
    const ST* sA = scl + g * sstride;
    const ST* bA = scl + kScaleArr / 2 + g * sstride;
    const ST* sB = scl + 2 * (kScaleArr / 2) + g * sstride;
    const ST* bB = scl + 3 * (kScaleArr / 2) + g * sstride;
    const uint8_t* halfA = stage;
    const uint8_t* halfB = stage + kHalfBytes;
    float accA = 0.f, accB = 0.f;
    // One block of 8 groups.  FULL: all 8 groups valid (no per-group branch,
    // so the loads of later groups can be issued ahead of earlier MMAs).
    auto block = [&](const int Gb, const bool full_block) {
        // four independent MMA chains (one per k-step), summed after the block
        float c[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
        float c2[4] = {0.f, 0.f, 0.f, 0.f}, c3[4] = {0.f, 0.f, 0.f, 0.f};
        // this lane's row within the swizzled boxes of the block (2 boxes of 4 groups)
        const int bbase = ((Gb - G0) >> 2) * kBoxBytes + g * kBox;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int G = Gb + j;
            if (full_block || G < G1) {
                const uint4* xp = (g == j) ? reinterpret_cast<const uint4*>(sd.xs + (G * 8 + 2 * t) * 4) : zeros;
                const uint4 x0 = xp[0], x1 = xp[1];
                // swz(g, (G - G0) * 32 + t * 8) with the block's part folded into bbase
                const int o = bbase + (j >> 2) * kBoxBytes + (((((j & 3) * 2 + (t >> 1)) ^ g) & 7) << 4) + (t & 1) * 8;
                const uint2 wa = *reinterpret_cast<const uint2*>(halfA + o);
                const uint2 wb = *reinterpret_cast<const uint2*>(halfB + o);
                uint32_t pa0[4], pa1[4], pb0[4], pb1[4];
                dq4_folded(wa.x, pa0);
                dq4_folded(wa.y, pa1);
                dq4_folded(wb.x, pb0);
                dq4_folded(wb.y, pb1);
                mma16816(c, pa0[0], pb0[0], pa0[1], pb0[1], x0.x, x0.y);
                mma16816(c1, pa0[2], pb0[2], pa0[3], pb0[3], x0.z, x0.w);
                mma16816(c2, pa1[0], pb1[0], pa1[1], pb1[1], x1.x, x1.y);
                mma16816(c3, pa1[2], pb1[2], pa1[3], pb1[3], x1.z, x1.w);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = (c[i] + c1[i]) + (c2[i] + c3[i]);
        // this lane's columns: groups Gb + 2t (c0, c2) and Gb + 2t + 1 (c1, c3)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int G = Gb + 2 * t + h;
            if (full_block || G < G1) {
                const float corr = sd.xcorr[G], xsm = sd.xsum[G];
                if (va) accA += scale_to_float(sA[G]) * (c[h] - corr) + scale_to_float(bA[G]) * xsm;
                if (vb) accB += scale_to_float(sB[G]) * (c[2 + h] - corr) + scale_to_float(bB[G]) * xsm;
            }
        }
    };
    int Gb = G0;
    for (; Gb + 8 <= G1; Gb += 8) block(Gb, true);
    if (Gb < G1) block(Gb, false);
    accA += __shfl_xor_sync(0xffffffffu, accA, 1);
    accA += __shfl_xor_sync(0xffffffffu, accA, 2);
    accB += __shfl_xor_sync(0xffffffffu, accB, 1);
    accB += __shfl_xor_sync(0xffffffffu, accB, 2);
    out[0] = accA;
    out[1] = 0.f;
    out[2] = accB;
    out[3] = 0.f;
}

// Batch-1 int4 path on the integer tensor path: weight codes unpacked to
// bytes (w & 0x0F0F0F0F, (w >> 4) & 0x0F0F0F0F) times the 15-bit activation
// split in two int8 halves (X = 128 hi + lo), exact int32 sums per group.
// The 8 MMA columns hold 4 groups x {hi, lo}: column 2j + h carries half h of
// group j of a 4-group block and is zero for the other groups' k-steps, so one
// m16n8k32 per 32 codes serves both halves.  Lane t then holds group t of the
// block: c[0] = hi, c[1] = lo of row g; c[2], c[3] of row g + 8.
// y = sum_g s_g * xsc_g * (128 hi + lo) + b_g * xsum_g.
// `part` 0/1 of `nparts` 2 covers the first / second half of the unit's groups
// (split at a multiple of 4) when two warps share the stage; nparts 1 = all.
template <typename ST>
__device__ __forceinline__ void compute_unit_b1_int(const uint8_t* __restrict__ stage, const SegDesc& sd, int chunk,
                                                    float out[4], int lane, const uint4* zeros, int part = 0,
                                                    int nparts = 1) {
    const int g = lane >> 2, t = lane & 3;
    const int ngK = sd.K / kGroup;
    constexpr int kGPU = kMaxBoxes * kBox / 32;  // 24 groups per unit
    const int U0 = chunk * kGPU;                 // the unit's groups: [U0, U1)
    const int U1 = min(ngK, U0 + kGPU);
    const int mid = nparts == 1 ? U1 : min(U1, U0 + ((U1 - U0 + 7) >> 3) * 4);
    const int G0 = part == 0 ? U0 : mid;         // this call's groups: [G0, G1)
    const int G1 = part == 0 ? mid : U1;
    const bool va = g < sd.nA, vb = g < sd.nB;
    const bool full = ngK <= kMaxScaleGroups;
    const int sstride = full ? ngK : kGPU;
    const int sbase = full ? 0 : U0;
    const ST* scl = reinterpret_cast<const ST*>(stage + 2 * kHalfBytes) - sbase;
    const ST* sA = scl + g * sstride;
    const ST* bA = scl + kScaleArr / 2 + g * sstride;
    const ST* sB = scl + 2 * (kScaleArr / 2) + g * sstride;
    const ST* bB = scl + 3 * (kScaleArr / 2) + g * sstride;
    const uint8_t* halfA = stage;
    const uint8_t* halfB = stage + kHalfBytes;
    const uint8_t* xb = reinterpret_cast<const uint8_t*>(sd.xs);
    constexpr uint32_t kLo = 0x0F0F0F0Fu;
    float accA = 0.f, accB = 0.f;
    // NB blocks of 4 groups (one 128-byte box column of the stage each), their
    // MMA chains interleaved
    auto blocks = [&](const int Gb, const bool full_block, auto nb_tag) {
        constexpr int NB = decltype(nb_tag)::value;
        int c[NB][2][4];
#pragma unroll
        for (int k = 0; k < NB; ++k)
#pragma unroll
            for (int i = 0; i < 4; ++i) c[k][0][i] = c[k][1][i] = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int k = 0; k < NB; ++k) {
                const int G = Gb + 4 * k + j;
                if (full_block || G < G1) {
                    const int bbase = ((Gb + 4 * k - U0) >> 2) * kBoxBytes + g * kBox;
                    // this lane's column 2j + h: half h = g & 1 of group j
                    const uint4* xp = ((g >> 1) == j)
                                          ? reinterpret_cast<const uint4*>(xb + (G * 4 + t) * 32) + (g & 1)
                                          : zeros;
                    const uint4 xv = xp[0];
                    const int o = bbase + ((((j * 2 + (t >> 1)) ^ g) & 7) << 4) + (t & 1) * 8;
                    const uint2 wa = *reinterpret_cast<const uint2*>(halfA + o);
                    const uint2 wb = *reinterpret_cast<const uint2*>(halfB + o);
                    const uint32_t a0 = wa.x & kLo, a1 = (wa.x >> 4) & kLo, a2 = wa.y & kLo, a3 = (wa.y >> 4) & kLo;
                    const uint32_t b0 = wb.x & kLo, b1 = (wb.x >> 4) & kLo, b2 = wb.y & kLo, b3 = (wb.y >> 4) & kLo;
                    imma16832(c[k][0], a0, b0, a1, b1, xv.x, xv.y);
                    imma16832(c[k][1], a2, b2, a3, b3, xv.z, xv.w);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < NB; ++k) {
            const int G = Gb + 4 * k + t;
            if (full_block || G < G1) {
                const float xsc = sd.xcorr[G], xsm = sd.xsum[G];
                const int dA = 128 * (c[k][0][0] + c[k][1][0]) + (c[k][0][1] + c[k][1][1]);
                const int dB = 128 * (c[k][0][2] + c[k][1][2]) + (c[k][0][3] + c[k][1][3]);
                if (va) accA += scale_to_float(sA[G]) * ((float)dA * xsc) + scale_to_float(bA[G]) * xsm;
                if (vb) accB += scale_to_float(sB[G]) * ((float)dB * xsc) + scale_to_float(bB[G]) * xsm;
            }
        }
    };
    int Gb = G0;
    for (; Gb + 8 <= G1; Gb += 8) blocks(Gb, true, std::integral_constant<int, 2>{});
    for (; Gb < G1; Gb += 4) blocks(Gb, Gb + 4 <= G1, std::integral_constant<int, 1>{});
    accA += __shfl_xor_sync(0xffffffffu, accA, 1);
    accA += __shfl_xor_sync(0xffffffffu, accA, 2);
    accB += __shfl_xor_sync(0xffffffffu, accB, 1);
    accB += __shfl_xor_sync(0xffffffffu, accB, 2);
    out[0] = accA;
    out[1] = 0.f;
    out[2] = accB;
    out[3] = 0.f;
}

// Scale/bias array `a` (0 sA, 1 bA, 2 sB, 3 bB) of a unit: source and bytes
// of the whole-row block (used when K/64 <= kMaxScaleGroups).
__device__ __forceinline__ void scale_block(const SegDesc& sd, int a, const uint8_t** src, int* bytes) {
    const int ngK = sd.K / kGroup;
    if (ngK > kMaxScaleGroups) {  // chunked scales: always the synchronous path
        *src = nullptr;
        *bytes = 1;
        return;
    }
    const void* base = a == 0 ? sd.SA : a == 1 ? sd.BA : a == 2 ? sd.SB : sd.BB;
    const int row = a < 2 ? sd.rowA : sd.rowB;
    const int n = a < 2 ? sd.nA : sd.nB;
    *src = static_cast<const uint8_t*>(base) + (size_t)row * ngK * 2;
    *bytes = n * ngK * 2;
}

__device__ __forceinline__ bool bulk_ok(const void* src, int bytes) {
    return ((reinterpret_cast<uintptr_t>(src) | (uintptr_t)bytes) & 15u) == 0;
}

// Fallback copy (weights only 2-byte aligned, DequantInt4GEMV.swift:97-102,
// or scale rows that are not 16-byte multiples): 16-bit loads by the warp,
// written in the same swizzled layout the TMA produces.
__device__ __forceinline__ void unit_copy_sync(uint8_t* stage, const SegDesc& sd, int chunk, bool weights,
                                               int lane) {
    const int rb = row_bytes(sd.K, sd.bits);
    const int b0 = chunk * kMaxBoxes * kBox;
    const int nbytes = min(rb - b0, kMaxBoxes * kBox);
    if (weights) {
        for (int h = 0; h < 2; ++h) {
            const int nr = h ? sd.nB : sd.nA;
            const uint8_t* W = (h ? sd.WB : sd.WA) + (size_t)(h ? sd.rowB : sd.rowA) * rb + b0;
            uint8_t* dst = stage + h * kHalfBytes;
            for (int i = lane; i < nr * nbytes / 2; i += 32) {
                const int r = (2 * i) / nbytes, b = (2 * i) % nbytes;
                *reinterpret_cast<uint16_t*>(dst + swz(r, b)) =
                    *reinterpret_cast<const uint16_t*>(W + (size_t)r * rb + b);
            }
        }
    }
    const int ngK = sd.K / kGroup;
    if (ngK > kMaxScaleGroups) {
        // chunk-relative scales: row r, groups [G0, G1) at r * gpu + (G - G0)
        const int gpu = kMaxBoxes * kBox / group_bytes(sd.bits);
        const int G0 = chunk * gpu, n = min(ngK, G0 + gpu) - G0;
        for (int a = 0; a < 4; ++a) {
            const void* base = a == 0 ? sd.SA : a == 1 ? sd.BA : a == 2 ? sd.SB : sd.BB;
            const int row0 = a < 2 ? sd.rowA : sd.rowB, nr = a < 2 ? sd.nA : sd.nB;
            const uint16_t* s16 = static_cast<const uint16_t*>(base);
            uint16_t* d16 = reinterpret_cast<uint16_t*>(stage + 2 * kHalfBytes + a * kScaleArr);
            for (int i = lane; i < nr * n; i += 32) {
                const int r = i / n, j = i - r * n;
                d16[r * gpu + j] = s16[(size_t)(row0 + r) * ngK + G0 + j];
            }
        }
        return;
    }
    for (int a = 0; a < 4; ++a) {
        const uint8_t* src;
        int bytes;
        scale_block(sd, a, &src, &bytes);
        if (!weights && bulk_ok(src, bytes)) continue;  // already bulk-copied
        uint16_t* d16 = reinterpret_cast<uint16_t*>(stage + 2 * kHalfBytes + a * kScaleArr);
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
        for (int i = lane; i < bytes / 2; i += 32) d16[i] = s16[i];
    }
}

// Arm the stage's mbarrier and issue the unit's copies.  Scale rows that are
// not bulk-copyable are copied synchronously by the warp.
__device__ __forceinline__ void unit_issue(uint8_t* stage, uint64_t* bar, const SegDesc& sd, int chunk, int lane) {
    const int nbx = min(boxes_for_K(sd.K, sd.bits) - chunk * kMaxBoxes, kMaxBoxes);
    uint32_t total = (uint32_t)((sd.nA > 0) + (sd.nB > 0)) * nbx * kBoxBytes;
    bool sync_scales = false;
    for (int a = 0; a < 4; ++a) {
        const uint8_t* src;
        int bytes;
        scale_block(sd, a, &src, &bytes);
        if (bulk_ok(src, bytes))
            total += bytes;
        else
            sync_scales = true;
    }
    if (lane == 0) mbar_arrive_expect_tx(bar, total);
    __syncwarp();
    const int x0 = chunk * kMaxBoxes * kBox;
    if (lane < nbx && sd.nA > 0)
        tma_load_3d(stage + lane * kBoxBytes, sd.mapA, x0 + lane * kBox, sd.rowA, sd.eA, bar);
    if (lane >= 8 && lane < 8 + nbx && sd.nB > 0)
        tma_load_3d(stage + kHalfBytes + (lane - 8) * kBoxBytes, sd.mapB, x0 + (lane - 8) * kBox, sd.rowB, sd.eB,
                    bar);
    if (lane >= 16 && lane < 20) {
        const int a = lane - 16;
        const uint8_t* src;
        int bytes;
        scale_block(sd, a, &src, &bytes);
        if (bytes > 0 && bulk_ok(src, bytes)) bulk_g2s(stage + 2 * kHalfBytes + a * kScaleArr, src, bytes, bar);
    }
    if (sync_scales) unit_copy_sync(stage, sd, chunk, false, lane);
}

// Host-computed schedule: up to two job ranges (e.g. routed and shared
// experts) with U units per job, J jobs per super-job and S super-jobs each.
struct Sched {
    int nj[2], U[2], J[2], S[2];
    int S_total;
};

// J (jobs per super-job) is the smallest value that still gives every CTA of
// the grid (`ctas`, normally one per SM) work, capped at kWarps / U: spreading
// the bytes over all SMs matters more than filling every warp.
inline int pick_J(int nj, int U, int ctas) {
    const int jmax = superjob_J(U);
    if (jmax <= 1 || ctas <= 0) return jmax;
    const int want = (nj + ctas - 1) / ctas;
    return want < 1 ? 1 : (want > jmax ? jmax : want);
}

// j0 > 0 forces the first class's jobs per super-job.
inline Sched make_sched(int nj0, int U0, int nj1 = 0, int U1 = 1, int ctas = 148, int j0 = 0) {
    Sched s;
    s.nj[0] = nj0;
    s.U[0] = U0;
    s.J[0] = j0 > 0 ? j0 : pick_J(nj0, U0, ctas);
    s.S[0] = nj0 > 0 ? (nj0 + s.J[0] - 1) / s.J[0] : 0;
    s.nj[1] = nj1;
    s.U[1] = U1;
    s.J[1] = pick_J(nj1, U1, ctas);
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

// Shared-memory layout of the engine (bytes), H = helper warps per stage (0/1):
//   [stages: kWarps * kStageBytes (1 KB aligned)][red: 2 * (1 + H) * kWarps * 32 * (H ? 2 : 4) floats]
//   [bars: kWarps u64][32 zero bytes][x area: Pol::x_bytes(p)]
// (with helper warps only the batch-1 integer path runs, whose lanes hold two
// non-zero partial sums, so a slot is a float2)
__host__ __device__ inline size_t engine_red_floats(int H) { return (size_t)2 * (1 + H) * kWarps * 32 * (H ? 2 : 4); }
__host__ __device__ inline size_t engine_fixed_smem(int H = 0) {
    return (size_t)kWarps * kStageBytes + engine_red_floats(H) * sizeof(float) + kWarps * 8 + 32;
}

// Dynamic shared memory rounded up to a 1 KB boundary (the 128-byte TMA
// swizzle needs 1 KB aligned boxes); launches request 1 KB of slack.
__device__ __forceinline__ uint8_t* engine_smem_base() {
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t a = smem_u32(smem);
    return smem + ((1024u - (a & 1023u)) & 1023u);
}

// Per-CTA engine state that persists across the phases of a fused kernel.
struct EngineState {
    uint8_t* smem;      // 1 KB aligned base
    uint8_t* xarea;     // staged activations
    uint64_t* bar;      // this warp's stage mbarrier (a helper warp: its owner's)
    int seq;            // units consumed by this warp (mbarrier phase)
    int parity_buf;     // reduction buffer in use
    bool dead;          // a bounded wait gave up: skip further waits
};

__device__ __forceinline__ void engine_init(EngineState& es, int H = 0) {
    es.smem = engine_smem_base();
    es.xarea = es.smem + engine_fixed_smem(H);
    float* red = reinterpret_cast<float*>(es.smem + (size_t)kWarps * kStageBytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + engine_red_floats(H));
    es.bar = bars + (threadIdx.x >> 5) % kWarps;
    es.seq = 0;
    es.parity_buf = 0;
    es.dead = false;
    if ((threadIdx.x & 31) == 0 && (threadIdx.x >> 5) < kWarps) mbar_init(es.bar, 1);
    if (threadIdx.x < 8) reinterpret_cast<uint32_t*>(bars + kWarps)[threadIdx.x] = 0u;  // zero x fragment
    fence_mbar_init();
}

__device__ __forceinline__ uint8_t* engine_xarea_of(const EngineState& es) { return es.xarea; }

// Two warps that share a stage meet at named barrier 1 + stage index.
__device__ __forceinline__ void stage_pair_sync(int stage_idx) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + stage_idx) : "memory");
}

// One phase: all jobs of policy `Pol`, distributed over the grid's CTAs.
// Every thread of the CTA must call it (it contains CTA barriers).
// H = 1: kWarps helper warps, helper w + kWarps computes the second half of
// the groups of every unit of stage w (batch-1 int4 integer path only; the
// host launches H = 1 only for such phases, with TMA-aligned weights).
template <class Pol, typename ST, int H = 0>
__device__ __forceinline__ void run_phase(const typename Pol::Params& p, EngineState& es) {
    constexpr int kW = kWarps * (1 + H);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int owner = warp % kWarps;
    const bool helper = H && warp >= kWarps;
    uint8_t* smem = es.smem;
    float* red = reinterpret_cast<float*>(smem + (size_t)kWarps * kStageBytes);
    uint8_t* xarea = engine_xarea_of(es);
    uint8_t* stage = smem + (size_t)owner * kStageBytes;
    uint64_t* bar = es.bar;

    // Weights that depend on no earlier kernel (router, plain GEMV) are put in
    // flight before waiting for the preceding kernel; expert ids and
    // activations are read only after the wait.
    if (!Pol::kWeightsIndependent) {
        if (!Pol::lazy(p)) griddep_wait();
        griddep_launch_dependents();
    }
    Pol::stage_pre(p, threadIdx.x);
    __syncthreads();

    const int S = Pol::superjobs(p);

    // Load cursor: same unit sequence as the compute loop below.
    int l_sj = blockIdx.x, l_i = 0;
    auto load_next = [&]() -> void {
        while (l_sj < S) {
            const SuperJob sj = Pol::superjob(p, l_sj);
            const int v = warp_unit(sj, owner, l_i);
            if (v < 0) {
                l_sj += gridDim.x;
                l_i = 0;
                continue;
            }
            ++l_i;
            SegDesc sd;
            int chunk;
            Pol::unit(p, sj.j0 + v / sj.U, v % sj.U, &sd, &chunk);
            unit_issue(stage, bar, sd, chunk, lane);
            return;
        }
    };

    // Weight tiles do not depend on the activations: put the first unit of
    // every warp in flight before staging the activations.
    TF_TW(8);
    if (p.aligned && !es.dead && !helper) load_next();
    TF_TW(9);
    if (Pol::kWeightsIndependent) {
        griddep_wait();
        griddep_launch_dependents();
    }
    Pol::stage_x(p, xarea, threadIdx.x, kW * 32);
    __syncthreads();

    for (int sjx = blockIdx.x; sjx < S; sjx += gridDim.x) {
        const SuperJob sj = Pol::superjob(p, sjx);
        if (Pol::kStagePerSuperjob) {  // activations differ per super-job (grouped experts)
            Pol::stage_x_sj(p, sj, xarea, threadIdx.x, kW * 32);
            __syncthreads();
        }
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int i = 0;; ++i) {
            const int v = warp_unit(sj, owner, i);
            if (v < 0) break;
            SegDesc sd;
            int chunk;
            Pol::unit(p, sj.j0 + v / sj.U, v % sj.U, &sd, &chunk);
            bool ready = true;
            if (p.aligned) {
                // once a wait has given up, later waits of this warp are skipped
                ready = !es.dead && mbar_wait_bounded(bar, (uint32_t)es.seq & 1u, p.err);
                es.dead = es.dead || !ready;
                if (i == 0) TF_TW(10);
            } else {
                unit_copy_sync(stage, sd, chunk, true, lane);
                __syncwarp();
            }
            if (ready) {
                float u[4];
                if constexpr (H != 0)
                    compute_unit_b1_int<ST>(stage, sd, chunk, u, lane, reinterpret_cast<const uint4*>(xarea) - 2,
                                            helper ? 1 : 0, 2);
                else if (sd.bits == 4 && sd.ntok == 1 && sd.xfold == 2)
                    compute_unit_b1_int<ST>(stage, sd, chunk, u, lane,
                                            reinterpret_cast<const uint4*>(xarea) - 2);  // 32 zero bytes before x
                else if (sd.bits == 4 && sd.ntok == 1 && sd.xfold)
                    compute_unit_b1<ST>(stage, sd, chunk, u, lane,
                                        reinterpret_cast<const uint4*>(xarea) - 2);  // 32 zero bytes before x
                else if (sd.bits == 4)
                    compute_unit<ST, 4>(stage, sd, chunk, u, lane);
                else
                    compute_unit<ST, 8>(stage, sd, chunk, u, lane);
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[k] = fmaf(sd.mult, u[k], acc[k]);
                if (i == 0) TF_TW(11);
            }
            __syncwarp();
            if constexpr (H != 0) stage_pair_sync(owner);  // both halves read before the stage is refilled
            if (p.aligned) ++es.seq;
            if (p.aligned && !es.dead && !helper) load_next();
        }
        constexpr int kSlot = H ? 2 : 4;  // floats per lane slot
        float* rb = red + (size_t)es.parity_buf * kW * 32 * kSlot;
        if constexpr (H != 0)
            *reinterpret_cast<float2*>(rb + (warp * 32 + lane) * 2) = make_float2(acc[0], acc[2]);
        else
            *reinterpret_cast<float4*>(rb + (warp * 32 + lane) * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        __syncthreads();
        // Leaders: for J > 1 warp jj*U reduces job jj over warps jj*U..jj*U+U-1;
        // for J == 1 warp 0 reduces warps 0..min(U,kWarps)-1.
        const int njobs = sj.j1 - sj.j0;
        const int lead_stride = sj.J > 1 ? sj.U : kWarps;
        if (!helper && warp % lead_stride == 0 && warp / lead_stride < njobs) {
            const int jj = warp / lead_stride;
            const int w0 = sj.J > 1 ? jj * sj.U : 0;
            const int wn = sj.J > 1 ? sj.U : min(sj.U, kWarps);
            float f[4] = {0.f, 0.f, 0.f, 0.f};
            for (int w = w0; w < w0 + wn; ++w) {
#pragma unroll
                for (int h = 0; h <= H; ++h) {
                    if constexpr (H != 0) {
                        const float2 q = *reinterpret_cast<const float2*>(rb + ((w + h * kWarps) * 32 + lane) * 2);
                        f[0] += q.x;
                        f[2] += q.y;
                    } else {
                        const float4 q = *reinterpret_cast<const float4*>(rb + (w * 32 + lane) * 4);
                        f[0] += q.x;
                        f[1] += q.y;
                        f[2] += q.z;
                        f[3] += q.w;
                    }
                }
            }
            Pol::epilogue(p, sj.j0 + jj, f, lane);
        }
        es.parity_buf ^= 1;
    }
}

template <class Pol, typename ST, int H = 0>
__global__ void __launch_bounds__(kWarps * 32 * (1 + H), 1)
    engine_kernel(const __grid_constant__ typename Pol::Params p) {
    EngineState es;
    TF_T(0);
    engine_init(es, H);
    run_phase<Pol, ST, H>(p, es);
    TF_T(6);
}

}  // namespace tf
