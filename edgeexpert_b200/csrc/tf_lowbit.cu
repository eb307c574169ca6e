// tf_lowbit.cu -- 2-bit and 3-bit affine g64 GEMVs and the 2/3-bit routed
// decode phases.
//
// Reference kernels replaced:
//   moe_int2_gemv_row_simd_dev_vec / moe_int3_gemv_row_simd_dev_vec and their
//   gate/up twins (Sources/TurboFieldfare/Metal/MoE/moe.metal:644-949),
//   moe_phase1_gate_up_act_b2/_b3 (moe.metal:950-1107),
//   moe_phase2_down_reduce_b2/_b3 (moe.metal:1108-1180),
//   dequant_int4_gemv_simd_body_b3 / dequant_int4_gemv_tgx_b3
//   (Sources/TurboFieldfare/Metal/Quant/dequant_int4.metal:512-717).
// Same factoring as the reference: per row and group of 64,
//     y += s * sum(q * x) + b * sum(x),   fp32.
//
// Packing (LSB-first, as Quantization.packCode): 3-bit rows are n*3/8 bytes,
// a group is 24 bytes = six 32-bit words with code c at bits 3c..3c+2; 2-bit
// rows are n/4 bytes, a group is 16 bytes = four words, code c at bits 2c.
//
// Tensor-core mapping (mma.sync m16n8k16, f16 x f16 -> f32).  A warp owns a
// tile of 16 rows (A rows g and g+8 of lane (g, t), g = lane/4, t = lane%4)
// and walks the K axis in boxes of 4 groups; in every box lane t takes group
// 4*box + t whole (24 or 16 bytes of each of its two rows, one 8-byte-aligned
// load per 8 bytes).  Because each MMA then mixes codes of four groups, the
// activation operand B is block-diagonal: column 2j + u holds token u's
// activation on the k slots of lane j and zero elsewhere, so accumulator
// columns 2t, 2t+1 of lane t end the box holding group t's dots for two
// tokens (more tokens: more MMAs on the same A registers).
//
// Code -> fp16 without conversion instructions.  One funnel shift brings a
// 32-bit window of the packed group into a register and one lop3 ANDs two
// codes into the two halves' mantissas and ORs in 0x6400 (fp16 1024):
//   3-bit: window at bit 24u-4 with mask 0x00070070 gives (1024 + 16 q[8u],
//          1024 + q[8u+4]); mask 0x00380380 gives (1024 + 128 q[8u+1],
//          1024 + 8 q[8u+5]); the window at 24u+2 gives the same for codes
//          8u+2, 8u+6, 8u+3, 8u+7.
//   2-bit: word v and word v >> 8 with masks 0x00030003 << 2j give
//          (1024 + 4^j q, 1024 + 4^j q') for codes 16v + 4h + j, + 8.
// The activation is staged divided by the same power of two (exact in fp16
// for normal values), so each product is 1024 x/scale + q x; the 1024 part
// is the per-group constant 1024 * sum(staged x), computed once from the
// staged halves and subtracted in the epilogue.  Codes, activations and
// products are exact; only the fp32 accumulation order differs from the
// reference.
#include <type_traits>

#include "tf_context.cuh"
#include "tf_lowbit.cuh"

using namespace tf;

namespace {

constexpr int kLbWarps = 8;
constexpr int kLbThreads = 32 * kLbWarps;
constexpr int kLbPairStride = 34;  // u32 words per staged (vector, group): 32 pairs + 2 pad (bank spread)
constexpr uint32_t kMagic = 0x64006400u;

// Staged activation of one (vector, group): pair P holds (x[lo]/s_lo, x[hi]/s_hi).
template <int BITS>
__device__ __forceinline__ void lb_pair_codes(int P, int& lo, int& hi, float& inv_lo, float& inv_hi) {
    if constexpr (BITS == 3) {
        const int u = P >> 2, j = P & 3;
        lo = 8 * u + j;
        hi = lo + 4;
        inv_lo = (j & 1) ? (1.0f / 128.0f) : (1.0f / 16.0f);
        inv_hi = (j & 1) ? (1.0f / 8.0f) : 1.0f;
    } else {
        const int v = P >> 3, h = (P >> 2) & 1, j = P & 3;
        lo = 16 * v + 4 * h + j;
        hi = lo + 8;
        inv_lo = inv_hi = 1.0f / (float)(1 << (2 * j));
    }
}

// Stage nvec activation vectors x[v * x_stride + k] (fp16, K = 64 * ngK):
// xs[(v * ngK + G) * kLbPairStride + P] = pair words, xc[v * ngK + G] =
// {1024 * sum(staged halves), sum(x)}.  One thread per (vector, group): the
// group's 64 halves in registers (eight 16-byte loads when aligned), its 32
// pair words and both sums without cross-lane reductions.
template <int BITS>
__device__ void lb_stage(const __half* __restrict__ x, int x_stride, int nvec, int ngK, uint32_t* xs, float2* xc,
                         int tid, int nthreads) {
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) && (nvec == 1 || (x_stride & 7) == 0);
    for (int vg = tid; vg < nvec * ngK; vg += nthreads) {
        const int v = vg / ngK, G = vg - v * ngK;
        const __half* xg = x + (size_t)v * x_stride + 64 * G;
        __half xv[64];
        if (vec) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const uint4 r = __ldg(reinterpret_cast<const uint4*>(xg) + q);
                memcpy(&xv[8 * q], &r, 16);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 64; ++k) xv[k] = xg[k];
        }
        uint32_t* w = xs + vg * kLbPairStride;
        float cs = 0.f, sx = 0.f;
#pragma unroll
        for (int P = 0; P < 32; ++P) {
            int lo, hi;
            float il, ih;
            lb_pair_codes<BITS>(P, lo, hi, il, ih);
            const __half a = __hmul(xv[lo], __float2half_rn(il));
            const __half b = __hmul(xv[hi], __float2half_rn(ih));
            w[P] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
            cs += __half2float(a) + __half2float(b);
            sx += __half2float(xv[lo]) + __half2float(xv[hi]);
        }
        xc[vg] = make_float2(1024.0f * cs, sx);
    }
    __syncthreads();
}

// The packed group of one row: 6 (3-bit) or 4 (2-bit) words.
template <int BITS>
struct LbWords {
    uint32_t w[2 * BITS];
};

// Per-warp cp.async ring: a stage holds, per lane, the packed group of its two
// rows (words [0, 2*BITS) row g, [2*BITS, 4*BITS) row g + 8; lane stride
// padded so 8- / 16-byte reads are bank-conflict free) and the four aligned
// 32-bit words holding its scale/bias values.
constexpr int kLbStages = 3;
template <int BITS>
struct LbRing {
    static constexpr int kLaneWords = BITS == 3 ? 14 : 12;
    static constexpr int kStageWords = 32 * kLaneWords + 4 * 32;
    static constexpr int kWarpBytes = kLbStages * kStageWords * 4;
};

__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The aligned 32-bit word holding a 2-byte scale (an aligned word never
// crosses a page, so reading its other half is harmless).
template <typename ST>
__device__ __forceinline__ const void* lb_word_of(const ST* p) {
    return reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
}
template <typename ST>
__device__ __forceinline__ float lb_half_of(uint32_t w, const ST* p) {
    const uint16_t h = (reinterpret_cast<uintptr_t>(p) & 2) ? (uint16_t)(w >> 16) : (uint16_t)(w & 0xFFFFu);
    if constexpr (std::is_same<ST, __half>::value)
        return __half2float(__ushort_as_half(h));
    else
        return bf16_bits_to_float(h);
}

template <int BITS, typename ST>
__device__ __forceinline__ void lb_issue(uint32_t* stage, int lane, const uint8_t* rowA, const uint8_t* rowB,
                                         const ST* sA, const ST* bA, const ST* sB, const ST* bB, int G) {
    uint32_t* w = stage + lane * LbRing<BITS>::kLaneWords;
    uint32_t* sc = stage + 32 * LbRing<BITS>::kLaneWords + lane;
    if (rowA) {
        if constexpr (BITS == 3) {
#pragma unroll
            for (int k = 0; k < 3; ++k) cp_async8(w + 2 * k, rowA + 24 * G + 8 * k);
        } else {
            cp_async16(w, rowA + 16 * G);
        }
        cp_async4(sc, lb_word_of(sA + G));
        cp_async4(sc + 32, lb_word_of(bA + G));
    }
    if (rowB) {
        if constexpr (BITS == 3) {
#pragma unroll
            for (int k = 0; k < 3; ++k) cp_async8(w + 6 + 2 * k, rowB + 24 * G + 8 * k);
        } else {
            cp_async16(w + 4, rowB + 16 * G);
        }
        cp_async4(sc + 64, lb_word_of(sB + G));
        cp_async4(sc + 96, lb_word_of(bB + G));
    }
}

template <int BITS>
__device__ __forceinline__ LbWords<BITS> lb_read_words(const uint32_t* stage, int lane, int which, bool live) {
    LbWords<BITS> r;
    if (!live) {
#pragma unroll
        for (int i = 0; i < 2 * BITS; ++i) r.w[i] = 0u;
        return r;
    }
    const uint32_t* w = stage + lane * LbRing<BITS>::kLaneWords + which * 2 * BITS;
    if constexpr (BITS == 3) {
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const uint2 v = *reinterpret_cast<const uint2*>(w + 2 * k);
            r.w[2 * k] = v.x;
            r.w[2 * k + 1] = v.y;
        }
    } else {
        const uint4 v = *reinterpret_cast<const uint4*>(w);
        r.w[0] = v.x;
        r.w[1] = v.y;
        r.w[2] = v.z;
        r.w[3] = v.w;
    }
    return r;
}

// Pair register P of a group (the order lb_pair_codes stages).
template <int BITS>
__device__ __forceinline__ uint32_t lb_pair(const LbWords<BITS>& W, int P) {
    if constexpr (BITS == 3) {
        const int u = P >> 2, j = P & 3;
        const int S = 24 * u + ((j & 2) ? 2 : -4);  // window start bit
        const int i = (S + 32) / 32 - 1;           // floor(S / 32), S >= -4
        const int sh = S - 32 * i;
        const uint32_t lo = i < 0 ? 0u : W.w[i];
        const uint32_t hi = (i + 1) < 6 ? W.w[i + 1] : 0u;
        const uint32_t win = sh == 0 ? lo : __funnelshift_r(lo, hi, sh);
        return lop3_and_or(win, (j & 1) ? 0x00380380u : 0x00070070u, kMagic);
    } else {
        const int v = P >> 3, h = (P >> 2) & 1, j = P & 3;
        const uint32_t win = h ? (W.w[v] >> 8) : W.w[v];
        return lop3_and_or(win, 0x00030003u << (2 * j), kMagic);
    }
}

// One box (4 groups) of a warp tile.  acc[r][tok]: rows g (r = 0) and g + 8
// (r = 1) for tokens 0 .. 2*NP-1 of the vectors v0 ...; lane t's share only
// (summed over the quad at the end of the tile).
template <int BITS, int NP>
__device__ __forceinline__ void lb_box(const LbWords<BITS>& WA, const LbWords<BITS>& WB, const uint32_t* xs,
                                       const float2* xc, int ngK, int G, bool valid, int v0, int nvec, float sa,
                                       float ba, float sb, float bb, float (&acc)[2][2 * NP], int g, int t) {
    float c[NP][2][4];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int e = 0; e < 4; ++e) c[p][q][e] = 0.f;
    // B fragment source: column g is token v0 + 2p + (g & 1) of group 4*box + (g >> 1)
    const bool mine = ((g >> 1) == t) && valid;
    const uint32_t* xrow[NP];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
        const int v = v0 + 2 * p + (g & 1);
        xrow[p] = (mine && v < nvec) ? xs + (v * ngK + G) * kLbPairStride : nullptr;
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) {
        const uint32_t a0 = lb_pair<BITS>(WA, 2 * m), a2 = lb_pair<BITS>(WA, 2 * m + 1);
        const uint32_t a1 = lb_pair<BITS>(WB, 2 * m), a3 = lb_pair<BITS>(WB, 2 * m + 1);
#pragma unroll
        for (int p = 0; p < NP; ++p) {
            uint2 b = make_uint2(0u, 0u);
            if (xrow[p]) b = *reinterpret_cast<const uint2*>(xrow[p] + 2 * m);
            mma16816(c[p][m & 1], a0, a1, a2, a3, b.x, b.y);
        }
    }
    if (!valid) return;
#pragma unroll
    for (int p = 0; p < NP; ++p) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int v = v0 + 2 * p + u;
            if (v < nvec) {
                const float2 k = xc[v * ngK + G];
                const float dA = (c[p][0][u] + c[p][1][u]) - k.x;
                const float dB = (c[p][0][2 + u] + c[p][1][2 + u]) - k.x;
                acc[0][2 * p + u] += sa * dA + ba * k.y;
                acc[1][2 * p + u] += sb * dB + bb * k.y;
            }
        }
    }
}

// A warp tile: rows rowA (A row g) and rowB (A row g + 8) of lane (g, t),
// boxes box0, box0 + step, ... streamed through the warp's cp.async ring
// (kLbStages - 1 boxes in flight while one is computed); returns the
// quad-summed accumulators.
template <int BITS, int NP, typename ST>
__device__ __forceinline__ void lb_tile(const uint8_t* rowA, const uint8_t* rowB, const ST* sA, const ST* bA,
                                        const ST* sB, const ST* bB, const uint32_t* xs, const float2* xc, int ngK,
                                        int v0, int nvec, int box0, int step, float (&acc)[2][2 * NP], int lane,
                                        uint32_t* ring) {
    using Ring = LbRing<BITS>;
    const int g = lane >> 2, t = lane & 3;
    const int nbox = (ngK + 3) >> 2;
    const int nj = box0 < nbox ? (nbox - box0 + step - 1) / step : 0;
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 2 * NP; ++k) acc[r][k] = 0.f;
    auto issue = [&](int j) {
        if (j < nj) {
            const int G = 4 * (box0 + j * step) + t;
            if (G < ngK)
                lb_issue<BITS, ST>(ring + (j % kLbStages) * Ring::kStageWords, lane, rowA, rowB, sA, bA, sB, bB, G);
        }
        cp_async_commit();
    };
#pragma unroll
    for (int j = 0; j < kLbStages - 1; ++j) issue(j);
    for (int j = 0; j < nj; ++j) {
        cp_async_wait<kLbStages - 2>();
        const uint32_t* stage = ring + (j % kLbStages) * Ring::kStageWords;
        const int G = 4 * (box0 + j * step) + t;
        const bool valid = G < ngK;
        const LbWords<BITS> wa = lb_read_words<BITS>(stage, lane, 0, valid && rowA);
        const LbWords<BITS> wb = lb_read_words<BITS>(stage, lane, 1, valid && rowB);
        const uint32_t* sc = stage + 32 * Ring::kLaneWords + lane;
        float sa = 0.f, ba = 0.f, sb = 0.f, bb = 0.f;
        if (valid && rowA) {
            sa = lb_half_of(sc[0], sA + G);
            ba = lb_half_of(sc[32], bA + G);
        }
        if (valid && rowB) {
            sb = lb_half_of(sc[64], sB + G);
            bb = lb_half_of(sc[96], bB + G);
        }
        issue(j + kLbStages - 1);
        lb_box<BITS, NP>(wa, wb, xs, xc, ngK, G, valid, v0, nvec, sa, ba, sb, bb, acc, g, t);
    }
    cp_async_wait<0>();
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 2 * NP; ++k) {
            acc[r][k] += __shfl_xor_sync(0xffffffffu, acc[r][k], 1);
            acc[r][k] += __shfl_xor_sync(0xffffffffu, acc[r][k], 2);
        }
}

// [per-warp rings][xs: nvec*ngK*kLbPairStride words][xc: nvec*ngK float2][red: 8 warps x 16 rows x 8 floats]
__host__ __device__ inline size_t lb_ring_bytes(int bits) {
    return (size_t)kLbWarps * (bits == 3 ? LbRing<3>::kWarpBytes : LbRing<2>::kWarpBytes);
}
__host__ __device__ inline size_t lb_smem_bytes(int bits, int nvec, int ngK) {
    return lb_ring_bytes(bits) + (size_t)nvec * ngK * (kLbPairStride * 4 + 8) + (size_t)kLbWarps * 16 * 8 * sizeof(float);
}

struct LbGemvParams {
    const uint8_t* W;
    const uint8_t* S;
    const uint8_t* B;
    long long w_bstride;   // bytes between matrices
    long long sb_bstride;  // elements between matrices' scale (bias) arrays
    int batch, M, K, ntok, x_stride, y_rstride, ks;
    long long y_bstride;
    const __half* x;
    __half* y;
    float* y32;
};

// Batched GEMV: tile = (matrix, 16 rows); the CTA's 8 warps are 8/ks tiles x
// ks K-slices, combined through shared memory in slice order.
template <int BITS, int NP, typename ST>
__global__ void __launch_bounds__(kLbThreads, 2) lb_gemv_kernel(const __grid_constant__ LbGemvParams p) {
    extern __shared__ __align__(16) uint8_t lb_smem[];
    const int ngK = p.K >> 6;
    uint32_t* ring = reinterpret_cast<uint32_t*>(lb_smem) + (threadIdx.x >> 5) * (LbRing<BITS>::kWarpBytes / 4);
    uint32_t* xs = reinterpret_cast<uint32_t*>(lb_smem + lb_ring_bytes(BITS));
    float2* xc = reinterpret_cast<float2*>(xs + (size_t)p.ntok * ngK * kLbPairStride);
    float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xc) + (size_t)p.ntok * ngK * 8);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    lb_stage<BITS>(p.x, p.x_stride, p.ntok, ngK, xs, xc, tid, kLbThreads);

    const int tilesM = (p.M + 15) >> 4, per = kLbWarps / p.ks;
    const int tile = blockIdx.x * per + warp / p.ks, kp = warp % p.ks;
    const bool live = tile < p.batch * tilesM;
    const int b = live ? tile / tilesM : 0;
    const int r0 = (tile - b * tilesM) * 16, g = lane >> 2;
    const int rA = r0 + g, rB = r0 + g + 8;
    const size_t rb = (size_t)(p.K / 64) * 8 * BITS;
    const uint8_t* W = p.W + (long long)b * p.w_bstride;
    const ST* S = reinterpret_cast<const ST*>(p.S) + (long long)b * p.sb_bstride;
    const ST* Bz = reinterpret_cast<const ST*>(p.B) + (long long)b * p.sb_bstride;
    float acc[2][2 * NP];
    if (live) {
        lb_tile<BITS, NP, ST>(rA < p.M ? W + rA * rb : nullptr, rB < p.M ? W + rB * rb : nullptr,
                              S + (size_t)rA * ngK, Bz + (size_t)rA * ngK, S + (size_t)rB * ngK, Bz + (size_t)rB * ngK,
                              xs, xc, ngK, 0, p.ntok, kp, p.ks, acc, lane, ring);
    }
    if (p.ks > 1) {
        if (live && (lane & 3) == 0)
#pragma unroll
            for (int k = 0; k < 2 * NP; ++k) {
                red[(warp * 16 + g) * 8 + k] = acc[0][k];
                red[(warp * 16 + g + 8) * 8 + k] = acc[1][k];
            }
        __syncthreads();
        if (!live || kp != 0) return;
        for (int s = 1; s < p.ks; ++s)
#pragma unroll
            for (int k = 0; k < 2 * NP; ++k) {
                acc[0][k] += red[((warp + s) * 16 + g) * 8 + k];
                acc[1][k] += red[((warp + s) * 16 + g + 8) * 8 + k];
            }
    }
    if (!live) return;
    const int t = lane & 3;
#pragma unroll
    for (int k = 0; k < 2 * NP; ++k) {
        if (k >= p.ntok || (k & 3) != t) continue;  // lane t writes tokens t, t + 4
        const long long ob = (long long)b * p.y_bstride + (long long)k * p.y_rstride;
        if (p.y32) {
            if (rA < p.M) p.y32[ob + rA] = acc[0][k];
            if (rB < p.M) p.y32[ob + rB] = acc[1][k];
        } else {
            if (rA < p.M) p.y[ob + rA] = __float2half_rn(acc[0][k]);
            if (rB < p.M) p.y[ob + rB] = __float2half_rn(acc[1][k]);
        }
    }
}

struct LbPhaseParams {
    const uint8_t* pool;
    unsigned long long stride;
    const uint32_t* ids;  // device [top_k]; nullptr => blobs
    const uint8_t* blobs[8];
    uint32_t off[9];
    int num_experts, D, F, top_k, ks;
    const __half* x;     // phase 1: token [D]; phase 2: acts [top_k][F]
    __half* acts;        // phase 1 output
    const __half* rw;    // phase 2: routing weights [top_k]
    const __half* residual;
    __half* y;
    uint32_t* err;
};

__device__ __forceinline__ const uint8_t* lb_blob(const LbPhaseParams& p, int slot) {
    if (!p.ids) return p.blobs[slot];
    const uint32_t e = __ldg(p.ids + slot);
    if (e >= (uint32_t)p.num_experts) {
        if (p.err) atomicOr(p.err, kErrBadExpert);
        return nullptr;
    }
    return p.pool + (size_t)e * p.stride;
}

// Phase 1: tile = (slot, 8 rows f): A rows 0-7 are gate rows, 8-15 the same up
// rows, so lane t == 0 of quad g holds gate and up of row f0 + g and writes
// acts = half(gelu_tanh(gate) * up).
template <int BITS, typename ST>
__global__ void __launch_bounds__(kLbThreads, 2) lb_phase1_kernel(const __grid_constant__ LbPhaseParams p) {
    extern __shared__ __align__(16) uint8_t lb_smem[];
    const int ngK = p.D >> 6;
    uint32_t* ring = reinterpret_cast<uint32_t*>(lb_smem) + (threadIdx.x >> 5) * (LbRing<BITS>::kWarpBytes / 4);
    uint32_t* xs = reinterpret_cast<uint32_t*>(lb_smem + lb_ring_bytes(BITS));
    float2* xc = reinterpret_cast<float2*>(xs + (size_t)ngK * kLbPairStride);
    float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xc) + (size_t)ngK * 8);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    lb_stage<BITS>(p.x, 0, 1, ngK, xs, xc, tid, kLbThreads);

    const int tilesF = (p.F + 7) >> 3, per = kLbWarps / p.ks;
    const int tile = blockIdx.x * per + warp / p.ks, kp = warp % p.ks;
    const int slot = tile / tilesF, g = lane >> 2;
    const int f = (tile - slot * tilesF) * 8 + g;
    const uint8_t* blob = tile < p.top_k * tilesF ? lb_blob(p, slot) : nullptr;
    const bool live = blob != nullptr;
    const size_t rb = (size_t)ngK * 8 * BITS;
    float acc[2][2];
    if (live) {
        const bool rv = f < p.F;
        const ST* gs = reinterpret_cast<const ST*>(blob + p.off[1]) + (size_t)f * ngK;
        const ST* gb = reinterpret_cast<const ST*>(blob + p.off[2]) + (size_t)f * ngK;
        const ST* us = reinterpret_cast<const ST*>(blob + p.off[4]) + (size_t)f * ngK;
        const ST* ub = reinterpret_cast<const ST*>(blob + p.off[5]) + (size_t)f * ngK;
        lb_tile<BITS, 1, ST>(rv ? blob + p.off[0] + f * rb : nullptr, rv ? blob + p.off[3] + f * rb : nullptr, gs, gb,
                             us, ub, xs, xc, ngK, 0, 1, kp, p.ks, acc, lane, ring);
    }
    if (p.ks > 1) {
        if (live && (lane & 3) == 0) {
            red[(warp * 16 + g) * 8] = acc[0][0];
            red[(warp * 16 + g + 8) * 8] = acc[1][0];
        }
        __syncthreads();
        if (!live || kp != 0) return;
        for (int s = 1; s < p.ks; ++s) {
            acc[0][0] += red[((warp + s) * 16 + g) * 8];
            acc[1][0] += red[((warp + s) * 16 + g + 8) * 8];
        }
    }
    if (live && (lane & 3) == 0 && f < p.F)
        p.acts[(size_t)slot * p.F + f] = __float2half_rn(gelu_tanh(acc[0][0]) * acc[1][0]);
}

// Phase 2: CTA = 16 rows d, warp w = slot w (the reference's threadgroup per
// row with a simdgroup per slot); partial = float(w_slot) * value, then
// y = half(residual + partial[0] + partial[1] + ...).
template <int BITS, typename ST>
__global__ void __launch_bounds__(kLbThreads, 2) lb_phase2_kernel(const __grid_constant__ LbPhaseParams p) {
    extern __shared__ __align__(16) uint8_t lb_smem[];
    const int ngK = p.F >> 6;
    uint32_t* ring = reinterpret_cast<uint32_t*>(lb_smem) + (threadIdx.x >> 5) * (LbRing<BITS>::kWarpBytes / 4);
    uint32_t* xs = reinterpret_cast<uint32_t*>(lb_smem + lb_ring_bytes(BITS));
    float2* xc = reinterpret_cast<float2*>(xs + (size_t)p.top_k * ngK * kLbPairStride);
    float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xc) + (size_t)p.top_k * ngK * 8);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    lb_stage<BITS>(p.x, p.F, p.top_k, ngK, xs, xc, tid, kLbThreads);

    const int d0 = blockIdx.x * 16, g = lane >> 2;
    const int dA = d0 + g, dB = d0 + g + 8;
    const size_t rb = (size_t)ngK * 8 * BITS;
    if (warp < p.top_k) {
        const uint8_t* blob = lb_blob(p, warp);
        float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
        if (blob) {
            const ST* ds = reinterpret_cast<const ST*>(blob + p.off[7]);
            const ST* db = reinterpret_cast<const ST*>(blob + p.off[8]);
            const uint8_t* dw = blob + p.off[6];
            lb_tile<BITS, 1, ST>(dA < p.D ? dw + dA * rb : nullptr, dB < p.D ? dw + dB * rb : nullptr,
                                 ds + (size_t)dA * ngK, db + (size_t)dA * ngK, ds + (size_t)dB * ngK,
                                 db + (size_t)dB * ngK, xs, xc, ngK, warp, warp + 1, 0, 1, acc, lane, ring);
        }
        if ((lane & 3) == 0) {
            const float w = __half2float(p.rw[warp]);
            part[warp * 16 + g] = w * acc[0][0];
            part[warp * 16 + g + 8] = w * acc[1][0];
        }
    }
    __syncthreads();
    if (tid < 16 && d0 + tid < p.D) {
        const int d = d0 + tid;
        float a = p.residual ? __half2float(p.residual[d]) : 0.f;
        for (int s = 0; s < p.top_k; ++s) a += part[s * 16 + tid];
        p.y[d] = __float2half_rn(a);
    }
}

template <class K>
tf_status lb_launch(tf_context* ctx, K kernel, int grid, size_t smem, cudaStream_t stream, const void* params,
                    const char* name) {
    const void* fn = reinterpret_cast<const void*>(kernel);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_check(ctx, e, name);
    }
    void* args[] = {const_cast<void*>(params)};
    return cuda_check(ctx, cudaLaunchKernel(fn, dim3(grid), dim3(kLbThreads), args, smem, stream), name);
}

// K-slices per tile so that the grid covers about two CTAs per SM.
int lb_split(tf_context* ctx, long long tiles, int nbox) {
    int ks = 1;
    while (ks < kLbWarps && ks * 2 <= nbox && (tiles * ks + kLbWarps - 1) / kLbWarps < 2ll * ctx->num_sms) ks *= 2;
    return ks;
}

constexpr size_t kLbSmemMax = 200 * 1024;

}  // namespace

namespace tf {

tf_status lowbit_gemv(tf_context* ctx, uint32_t bits, const void* W, const void* S, const void* B, uint64_t wbs,
                      uint64_t sbs, uint32_t batch, const void* x, uint32_t ntok, uint32_t xrs, void* y, float* y32,
                      uint32_t yrs, uint64_t ybs, uint32_t m, uint32_t n, tf_scale_type st, cudaStream_t stream,
                      const char* name) {
    const unsigned wal = bits == 2 ? 16u : 8u;
    if ((reinterpret_cast<uintptr_t>(W) & (wal - 1)) || (batch > 1 && wbs % wal))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: %u-bit weights must be %u-byte aligned", name, bits, wal);
    const int ngK = (int)(n / 64);
    const size_t smem = lb_smem_bytes((int)bits, (int)ntok, ngK);
    if (smem > kLbSmemMax)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: ntok * n too large for the %u-bit GEMV", name, bits);
    LbGemvParams p;
    memset(&p, 0, sizeof(p));
    p.W = static_cast<const uint8_t*>(W);
    p.S = static_cast<const uint8_t*>(S);
    p.B = static_cast<const uint8_t*>(B);
    p.w_bstride = (long long)wbs;
    p.sb_bstride = (long long)sbs;
    p.batch = (int)batch;
    p.M = (int)m;
    p.K = (int)n;
    p.ntok = (int)ntok;
    p.x_stride = (int)xrs;
    p.y_rstride = (int)yrs;
    p.y_bstride = (long long)ybs;
    p.x = static_cast<const __half*>(x);
    p.y = static_cast<__half*>(y);
    p.y32 = y32;
    const long long tiles = (long long)batch * ((m + 15) / 16);
    if (tiles > (1ll << 30)) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: too many rows", name);
    p.ks = lb_split(ctx, tiles, (ngK + 3) / 4);
    const int grid = (int)((tiles * p.ks + kLbWarps - 1) / kLbWarps);
    const int np = (ntok + 1) / 2;
    auto go = [&](auto kern) { return lb_launch(ctx, kern, grid, smem, stream, &p, name); };
#define TF_LB_CASE(BITS_, NP_)                                                                               \
    if (bits == BITS_ && np <= NP_)                                                                          \
        return st == TF_SCALE_BF16 ? go(lb_gemv_kernel<BITS_, NP_, __nv_bfloat16>) : go(lb_gemv_kernel<BITS_, NP_, __half>);
    TF_LB_CASE(2, 1)
    TF_LB_CASE(2, 2)
    TF_LB_CASE(2, 4)
    TF_LB_CASE(3, 1)
    TF_LB_CASE(3, 2)
    TF_LB_CASE(3, 4)
#undef TF_LB_CASE
    return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: bits must be 2 or 3", name);
}

static tf_status lb_phase_params(tf_context* ctx, uint32_t bits, const void* pool, uint64_t stride, uint32_t E,
                                 const void* ids, const void* const* blobs, const tf_expert_offsets* off,
                                 uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st, LbPhaseParams* p,
                                 const char* name) {
    if (bits != 2 && bits != 3) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: bits must be 2, 3 or 4", name);
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return fail(ctx, TF_ERR_INVALID_ARG, "%s: unknown scale type", name);
    if (!off) return fail(ctx, TF_ERR_INVALID_ARG, "%s: offsets is NULL", name);
    if (top_k == 0 || top_k > 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: top_k must be in 1..8, got %u", name, top_k);
    if (d == 0 || f == 0 || d % 64 || f % 64)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d and f must be positive multiples of 64", name);
    const uint32_t o[9] = {off->gate_w, off->gate_s, off->gate_b, off->up_w, off->up_s, off->up_b,
                           off->down_w, off->down_s, off->down_b};
    const unsigned wal = bits == 2 ? 16u : 8u;
    for (int i = 0; i < 9; ++i) {
        const unsigned a = (i % 3 == 0) ? wal : 2u;
        if (o[i] % a) return fail(ctx, TF_ERR_MISALIGNED, "%s: sub-tensor offset %d must be %u-byte aligned", name, i, a);
    }
    memset(p, 0, sizeof(*p));
    if (ids) {
        if (!pool || E == 0) return fail(ctx, TF_ERR_INVALID_ARG, "%s: expert pool / num_experts missing", name);
        if ((reinterpret_cast<uintptr_t>(pool) % wal) || stride % wal)
            return fail(ctx, TF_ERR_MISALIGNED, "%s: pool and stride must be %u-byte aligned", name, wal);
        p->pool = static_cast<const uint8_t*>(pool);
        p->stride = stride;
        p->ids = static_cast<const uint32_t*>(ids);
        p->num_experts = (int)E;
    } else {
        if (!blobs) return fail(ctx, TF_ERR_INVALID_ARG, "%s: need expert_ids or blobs", name);
        for (uint32_t i = 0; i < top_k; ++i) {
            if (!blobs[i]) return fail(ctx, TF_ERR_INVALID_ARG, "%s: blob %u is NULL", name, i);
            if (reinterpret_cast<uintptr_t>(blobs[i]) % wal)
                return fail(ctx, TF_ERR_MISALIGNED, "%s: blob %u must be %u-byte aligned", name, i, wal);
            p->blobs[i] = static_cast<const uint8_t*>(blobs[i]);
        }
    }
    memcpy(p->off, o, sizeof(o));
    p->D = (int)d;
    p->F = (int)f;
    p->top_k = (int)top_k;
    p->err = ctx->d_err;
    return TF_OK;
}

tf_status lowbit_phase1(tf_context* ctx, uint32_t bits, const void* pool, uint64_t stride, uint32_t E, const void* ids,
                        const void* const* blobs, const tf_expert_offsets* off, const void* x, void* acts, uint32_t d,
                        uint32_t f, uint32_t top_k, tf_scale_type st, cudaStream_t stream, const char* name) {
    LbPhaseParams p;
    tf_status s = lb_phase_params(ctx, bits, pool, stride, E, ids, blobs, off, d, f, top_k, st, &p, name);
    if (s) return s;
    if (!x || !acts) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned2(x) || !aligned2(acts)) return fail(ctx, TF_ERR_MISALIGNED, "%s: buffers must be 2-byte aligned", name);
    const int ngK = (int)(d / 64);
    const size_t smem = lb_smem_bytes((int)bits, 1, ngK);
    if (smem > kLbSmemMax) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d too large", name);
    p.x = static_cast<const __half*>(x);
    p.acts = static_cast<__half*>(acts);
    const long long tiles = (long long)top_k * ((f + 7) / 8);
    p.ks = lb_split(ctx, tiles, (ngK + 3) / 4);
    const int grid = (int)((tiles * p.ks + kLbWarps - 1) / kLbWarps);
    auto go = [&](auto kern) { return lb_launch(ctx, kern, grid, smem, stream, &p, name); };
    if (bits == 2)
        return st == TF_SCALE_BF16 ? go(lb_phase1_kernel<2, __nv_bfloat16>) : go(lb_phase1_kernel<2, __half>);
    return st == TF_SCALE_BF16 ? go(lb_phase1_kernel<3, __nv_bfloat16>) : go(lb_phase1_kernel<3, __half>);
}

tf_status lowbit_phase2(tf_context* ctx, uint32_t bits, const void* pool, uint64_t stride, uint32_t E, const void* ids,
                        const void* const* blobs, const tf_expert_offsets* off, const void* acts, const void* rw,
                        const void* residual, void* y, uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st,
                        cudaStream_t stream, const char* name) {
    LbPhaseParams p;
    tf_status s = lb_phase_params(ctx, bits, pool, stride, E, ids, blobs, off, d, f, top_k, st, &p, name);
    if (s) return s;
    if (!acts || !rw || !y) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned2(acts) || !aligned2(rw) || !aligned2(y) || !aligned2(residual))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: buffers must be 2-byte aligned", name);
    const int ngK = (int)(f / 64);
    const size_t smem = lb_smem_bytes((int)bits, (int)top_k, ngK);
    if (smem > kLbSmemMax) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: top_k * f too large", name);
    p.x = static_cast<const __half*>(acts);
    p.rw = static_cast<const __half*>(rw);
    p.residual = static_cast<const __half*>(residual);
    p.y = static_cast<__half*>(y);
    const int grid = (int)((d + 15) / 16);
    auto go = [&](auto kern) { return lb_launch(ctx, kern, grid, smem, stream, &p, name); };
    if (bits == 2)
        return st == TF_SCALE_BF16 ? go(lb_phase2_kernel<2, __nv_bfloat16>) : go(lb_phase2_kernel<2, __half>);
    return st == TF_SCALE_BF16 ? go(lb_phase2_kernel<3, __nv_bfloat16>) : go(lb_phase2_kernel<3, __half>);
}

}  // namespace tf

extern "C" {

tf_status tf_moe_phase1_bits(tf_context* ctx, uint32_t bits, const void* pool, uint64_t stride, uint32_t E,
                             const void* ids, const void* const* blobs, const tf_expert_offsets* off, const void* x,
                             void* acts, uint32_t d, uint32_t f, uint32_t top_k, tf_scale_type st, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (bits == 4) return tf_moe_phase1(ctx, pool, stride, E, ids, blobs, off, x, acts, d, f, top_k, st, stream);
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    return lowbit_phase1(ctx, bits, pool, stride, E, ids, blobs, off, x, acts, d, f, top_k, st,
                         static_cast<cudaStream_t>(stream), "tf_moe_phase1_bits");
}

tf_status tf_moe_phase2_bits(tf_context* ctx, uint32_t bits, const void* pool, uint64_t stride, uint32_t E,
                             const void* ids, const void* const* blobs, const tf_expert_offsets* off, const void* acts,
                             const void* rw, const void* residual, void* y, uint32_t d, uint32_t f, uint32_t top_k,
                             tf_scale_type st, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (bits == 4)
        return tf_moe_phase2(ctx, pool, stride, E, ids, blobs, off, acts, rw, residual, y, d, f, top_k, st, stream);
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    return lowbit_phase2(ctx, bits, pool, stride, E, ids, blobs, off, acts, rw, residual, y, d, f, top_k, st,
                         static_cast<cudaStream_t>(stream), "tf_moe_phase2_bits");
}

}  // extern "C"
