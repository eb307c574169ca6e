// tf_gemv_tc.cu -- one-token int4 g64 GEMV streamed through the 5th-generation
// tensor cores (tcgen05.mma kind::i8, A operand in TMEM).
//
// Reference kernel replaced: dequant_int4_gemv
// (Sources/TurboFieldfare/Metal/Quant/dequant_int4.metal:126-173, encoded by
// DequantInt4GEMV.encode, Kernels/Quant/DequantInt4GEMV.swift:84-180), here for
// one or many matrices that share the activation vector (tf_affine_gemv_batched
// with one token).  Same factoring as the reference:
//     y[r] = sum_g s[r][g] * (sum_{k in g} q[r][k] x[k]) + b[r][g] * (sum_{k in g} x[k])
//
// Why tensor cores for a GEMV: the bound is HBM, but the legacy mma.sync path
// needs four 16x8x16 MMAs per 16 rows x 64 codes and saturates its pipe below
// the HBM rate.  One tcgen05.mma covers 128 rows x 32 codes, so the MMA cost
// vanishes and what is left per code is a shift and two ANDs.
//
// Arithmetic.  The activation is quantised per group of 64 exactly as the
// engine's integer path (stage_x_int): X = rn(x * 16383 / max|x_g|), split
// X = 128 hi + lo with hi in [-128, 127], lo in [0, 127].  The codes q (u8)
// times hi and lo (s8) give exact int32 group dots; the epilogue forms
// s * xsc_g * (128 hi + lo) + b * xsum_g in fp32.
//
// Operands.  A = codes, one row per TMEM lane: a raw word w (8 nibbles) becomes
// the two u8 words w & 0x0F0F0F0F (elements 0,2,4,6) and (w >> 4) & 0x0F0F0F0F
// (elements 1,3,5,7), so the K order inside each 8 is 0,2,4,6,1,3,5,7; the
// activation operand B is staged in that order.  B is block-diagonal: for a
// stage of 8 groups it has N = 16 columns (group j: hi in column 2j, lo in
// 2j+1) that are zero outside their group, so one accumulator of 16 columns
// holds the 8 group dots of the stage for all 128 rows.
//
// Roles (384 threads, one CTA per SM, persistent over jobs = (matrix, 128-row tile)):
//   warp 0      one thread: scale/bias block of a job (1-D bulk copy, exact
//               bytes) and the raw weight stages (two 3-D TMA boxes of 128 rows
//               x 128 B, 128-byte swizzle, 8 groups per stage) into a ring
//   warp 1      TMEM allocation; one thread issues the MMAs (16 per stage)
//   warps 4-7   unpack: raw nibbles -> u8 words -> tcgen05.st into A (3 buffers)
//   warps 8-11  epilogue: tcgen05.ld of the stage's 16 accumulator columns
//               (4 buffers), scale/bias, fp16 store at the job's end
// Every wait is bounded; on a timeout the CTA records kErrMbarTimeout and all
// roles leave their loops.
#include "tf_context.cuh"
#include "tf_gemv_tc.cuh"
#include "tf_umma.cuh"

using namespace tf;

namespace {

constexpr int kGtThreads = 384;
constexpr int kGtRows = 128;                 // rows per job (MMA M, TMEM lanes)
constexpr int kGtBox = kGtRows * 128;        // one TMA box: 128 rows x 128 B (4 groups)
constexpr int kGtStage = 2 * kGtBox;         // 8 groups per stage
constexpr int kGtBStage = 16 * 512;          // activation operand of one stage: 16 x 512 B
constexpr int kGtMaxR = 6;                   // raw stages in the ring
constexpr uint32_t kGtTmemCols = 512;
constexpr int kGtNA = 3;                     // A operand buffers (128 columns each)
constexpr int kGtND = 4;                     // accumulators (16 columns each)
constexpr uint32_t kGtA0 = 0;                // A buffers: columns [0, 384)
constexpr uint32_t kGtD0 = 128 * kGtNA;      // accumulators: [384, 448)
constexpr int kGtUnpackWarp0 = 4;
constexpr int kGtEpiWarp0 = 8;
constexpr size_t kGtSmemLimit = 232448;
constexpr uint32_t kGtSpin = 1u << 20;

struct GtParams {
    CUtensorMap wmap;  // uint8 [batch][M][K/2], box 128 B x 128 rows x 1, 128-byte swizzle
    const uint8_t* S;  // scales [batch][M][K/64] (bytes)
    const uint8_t* B;  // biases
    long long sb_bstride;  // bytes between matrices' scale (and bias) arrays
    const __half* x;
    __half* y;
    float* y32;           // fp32 output instead of y (NULL = fp16 y)
    long long y_bstride;  // elements between matrices' outputs
    int M, K, batch, tiles, jobs, R;
    uint32_t* err;
};

struct GtShared {
    uint64_t full[kGtMaxR], empty[kGtMaxR];
    uint64_t afull[kGtNA], aempty[kGtNA], dfull[kGtND], dempty[kGtND];
    uint64_t sfull[2], sempty[2];
    uint64_t done;
    uint32_t tmem_base;
    int abort_flag;
};

struct GtLayout {
    uint32_t bop, scl, sslot, xsc, xsum, sh, total;
};

// Shared-memory layout (offsets from a 1024-aligned base): raw ring, the
// activation operand (1024-aligned swizzle atoms), two job slots of scales and
// biases, the per-group activation scale and sum, the barriers.
__host__ __device__ inline GtLayout gt_layout(int K, int R) {
    const int ngK = K / 64, nst = (ngK + 7) / 8;
    GtLayout L;
    L.bop = (uint32_t)R * kGtStage;
    L.sslot = (uint32_t)((kGtRows * ngK * 2 + 15) & ~15);
    L.scl = L.bop + (uint32_t)nst * kGtBStage;
    L.xsc = L.scl + 4 * L.sslot;
    L.xsum = L.xsc + (uint32_t)ngK * 4;
    L.sh = (L.xsum + (uint32_t)ngK * 4 + 15) & ~15u;
    L.total = L.sh + (uint32_t)sizeof(GtShared) + 1024;
    return L;
}

// Byte of the activation operand holding half h (0 = hi, 1 = lo) of element e
// (0..63) of group G: stage G/8, swizzle atom (G%8)/2 of 128 K-bytes x 16 rows
// (row n = 2*(G%8) + h at n*128, rows 8-15 one KB on), 16-byte chunks XOR-ed
// with n % 8, and inside each 8 elements the unpacked order 0,2,4,6,1,3,5,7.
__device__ __forceinline__ int gt_bpos(int G, int e, int h) {
    const int k = e & 7;
    const int pos = (e & ~7) | ((k & 1) ? 4 + (k >> 1) : (k >> 1));
    const int gl = G & 7, n = 2 * gl + h;
    const int kb = 64 * (gl & 1) + pos;
    return (G >> 3) * kGtBStage + (gl >> 1) * 2048 + (n >> 3) * 1024 + (n & 7) * 128 +
           ((((kb >> 4) ^ n) & 7) << 4) + (kb & 15);
}

// Bounded wait; the first wait of the launch to give up records its source
// line and (CTA << 20 | job << 10 | stage & 1023) in the status words 1-2.
__device__ __forceinline__ bool gwait(uint64_t* bar, uint32_t parity, int& abort_flag, uint32_t* err, uint32_t site = 0,
                                      uint32_t info = 0) {
    for (uint32_t i = 0; i < kGtSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *reinterpret_cast<volatile int*>(&abort_flag)) return false;
    }
    abort_flag = 1;
    if (err && atomicOr(err, kErrMbarTimeout) == 0) {
        err[1] = site;
        err[2] = info;
    }
    return false;
}
__device__ __forceinline__ uint32_t gt_info(int jl, uint32_t q) {
    return (blockIdx.x << 20) | ((uint32_t)(jl & 1023) << 10) | (q & 1023u);
}
__device__ __forceinline__ bool gwait(uint64_t* bar, uint32_t parity, GtShared& sh, uint32_t* err) {
    return gwait(bar, parity, sh.abort_flag, err);
}

// The loader role of both GEMV kernels (one thread): per job (matrix b, rows
// row0..row0+127) the scale and bias block -- one contiguous run of
// rows * K/64 elements each, bulk-copied in 16-byte multiples, the < 16 ragged
// bytes of a short last tile by plain loads -- into job slot jl % 2, then the
// job's stages of 8 groups (two TMA boxes of 128 rows x 128 B; the second is
// skipped when it starts past the row) into the ring.
struct GtRing {
    uint8_t* ring;
    uint8_t* scl;
    uint32_t sslot;
    uint64_t* full;
    uint64_t* empty;
    uint64_t* sfull;
    uint64_t* sempty;
    int* abort_flag;
};

__device__ __forceinline__ void gt_load_jobs(const GtParams& p, const GtRing& r) {
    const int ngK = p.K >> 6, nst = (ngK + 7) >> 3, R = p.R;
    uint32_t q = 0;
    int jl = 0;
    for (int job = blockIdx.x; job < p.jobs; job += gridDim.x, ++jl) {
        const int b = job / p.tiles, row0 = (job - b * p.tiles) * kGtRows;
        const int rows = min(kGtRows, p.M - row0);
        const int js = jl & 1;
        if (!gwait(&r.sempty[js], ((jl >> 1) & 1) ^ 1, *r.abort_flag, p.err, __LINE__, gt_info(jl, q))) return;
        const uint32_t nbytes = (uint32_t)rows * ngK * 2, bulk = nbytes & ~15u;
        const size_t off = (size_t)b * p.sb_bstride + (size_t)row0 * ngK * 2;
        uint8_t* ds = r.scl + (2 * js) * r.sslot;
        uint8_t* db = ds + r.sslot;
        for (uint32_t i = bulk; i < nbytes; i += 2) {
            *reinterpret_cast<uint16_t*>(ds + i) = __ldg(reinterpret_cast<const uint16_t*>(p.S + off + i));
            *reinterpret_cast<uint16_t*>(db + i) = __ldg(reinterpret_cast<const uint16_t*>(p.B + off + i));
        }
        mbar_arrive_expect_tx(&r.sfull[js], 2 * bulk);
        if (bulk) {
            bulk_g2s(ds, p.S + off, bulk, &r.sfull[js]);
            bulk_g2s(db, p.B + off, bulk, &r.sfull[js]);
        }
        for (int st = 0; st < nst; ++st, ++q) {
            const int slot = (int)(q % (uint32_t)R);
            if (!gwait(&r.empty[slot], ((q / R) & 1) ^ 1, *r.abort_flag, p.err, __LINE__, gt_info(jl, q))) return;
            const int x0 = st * 256;
            const bool two = x0 + 128 < p.K / 2;
            mbar_arrive_expect_tx(&r.full[slot], two ? 2 * kGtBox : kGtBox);
            tma_load_3d(r.ring + slot * kGtStage, &p.wmap, x0, row0, b, &r.full[slot]);
            if (two) tma_load_3d(r.ring + slot * kGtStage + kGtBox, &p.wmap, x0 + 128, row0, b, &r.full[slot]);
        }
    }
}

template <typename ST>
__global__ void __launch_bounds__(kGtThreads, 1) gemv_tc_kernel(const __grid_constant__ GtParams p) {
    extern __shared__ uint8_t gt_smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gt_smem_raw) + 1023) & ~uintptr_t(1023));
    const GtLayout L = gt_layout(p.K, p.R);
    uint8_t* ring = sm;
    uint8_t* bop = sm + L.bop;
    uint8_t* scl = sm + L.scl;
    float* xsc = reinterpret_cast<float*>(sm + L.xsc);
    float* xsum = reinterpret_cast<float*>(sm + L.xsum);
    GtShared& sh = *reinterpret_cast<GtShared*>(sm + L.sh);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ngK = p.K >> 6, nst = (ngK + 7) >> 3, R = p.R;

    if (tid == 0) {
        for (int s = 0; s < R; ++s) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], 4);
        }
        for (int a = 0; a < kGtNA; ++a) {
            mbar_init(&sh.afull[a], 4);
            mbar_init(&sh.aempty[a], 1);
        }
        for (int a = 0; a < kGtND; ++a) {
            mbar_init(&sh.dfull[a], 1);
            mbar_init(&sh.dempty[a], 4);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&sh.sfull[a], 1);
            mbar_init(&sh.sempty[a], 4);
        }
        mbar_init(&sh.done, 1);
        sh.abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&p.wmap);
    }
    {
        uint4* z = reinterpret_cast<uint4*>(bop);
        const int n16 = nst * kGtBStage / 16;
        for (int i = tid; i < n16; i += kGtThreads) z[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    __syncthreads();
    // activation operand: per group, X = rn(x * 16383 / max|x|) = 128 hi + lo
    for (int G = warp; G < ngK; G += kGtThreads / 32) {
        const float a = __half2float(__ldg(p.x + G * 64 + 2 * lane));
        const float b = __half2float(__ldg(p.x + G * 64 + 2 * lane + 1));
        float m = fmaxf(fabsf(a), fabsf(b)), sum = a + b;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
        }
        const float q = m > 0.f ? 16383.0f / m : 0.f;
        const int XA = __float2int_rn(a * q), XB = __float2int_rn(b * q);
        bop[gt_bpos(G, 2 * lane, 0)] = (uint8_t)(XA >> 7);
        bop[gt_bpos(G, 2 * lane, 1)] = (uint8_t)(XA & 127);
        bop[gt_bpos(G, 2 * lane + 1, 0)] = (uint8_t)(XB >> 7);
        bop[gt_bpos(G, 2 * lane + 1, 1)] = (uint8_t)(XB & 127);
        if (lane == 0) {
            xsum[G] = sum;
            xsc[G] = m / 16383.0f;
        }
    }
    if (warp == 1) {
        tmem_alloc(&sh.tmem_base, kGtTmemCols);
        tc_fence_before();
    }
    fence_proxy_async_smem();  // activation operand -> tensor core (async proxy)
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;

    if (warp == 0) {
        // ================= loader =================
        if (lane == 0) {
            const GtRing r{ring, scl, L.sslot, sh.full, sh.empty, sh.sfull, sh.sempty, &sh.abort_flag};
            gt_load_jobs(p, r);
        }
    } else if (warp == 1) {
        // ================= MMA issue =================
        if (lane == 0) {
            const uint32_t idesc = make_idesc_u8s8(kGtRows, 16);
            const uint64_t bdesc0 = make_sw128_desc(bop);
            uint32_t q = 0;
            bool ok = true;
            for (int job = blockIdx.x; ok && job < p.jobs; job += gridDim.x) {
                for (int st = 0; st < nst; ++st, ++q) {
                    const uint32_t a = q % kGtNA, d = q % kGtND;
                    if (!(ok = gwait(&sh.afull[a], (q / kGtNA) & 1u, sh, p.err))) break;
                    if (!(ok = gwait(&sh.dempty[d], ((q / kGtND) & 1u) ^ 1u, sh, p.err))) break;
                    tc_fence_after();
                    const int ksteps = 2 * min(8, ngK - 8 * st);
                    for (int j = 0; j < ksteps; ++j) {
                        const uint32_t boff = (uint32_t)st * kGtBStage + (j >> 2) * 2048 + (j & 3) * 32;
                        umma_i8_ts(tmem + kGtD0 + 16 * d, tmem + kGtA0 + 128 * a + 8 * j, bdesc0 + (boff >> 4),
                                   idesc, j > 0 ? 1u : 0u);
                    }
                    umma_commit(&sh.dfull[d]);
                    umma_commit(&sh.aempty[a]);
                }
            }
            // every issued MMA has retired before TMEM is freed
            umma_commit(&sh.done);
            gwait(&sh.done, 0, sh, p.err);
        }
    } else if (warp >= kGtUnpackWarp0 && warp < kGtEpiWarp0) {
        // ================= unpack: codes -> u8 A operand in TMEM =================
        const int rr = (warp - kGtUnpackWarp0) * 32 + lane;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const int sw = rr & 7;
        constexpr uint32_t kLo = 0x0F0F0F0Fu;
        uint32_t q = 0;
        bool ok = true;
        for (int job = blockIdx.x; ok && job < p.jobs; job += gridDim.x) {
            for (int st = 0; st < nst; ++st, ++q) {
                const int slot = (int)(q % (uint32_t)R);
                const uint32_t a = q % kGtNA;
                if (!(ok = gwait(&sh.full[slot], (q / R) & 1u, sh, p.err))) break;
                if (!(ok = gwait(&sh.aempty[a], ((q / kGtNA) & 1u) ^ 1u, sh, p.err))) break;
                tc_fence_after();
                const int ng = min(8, ngK - 8 * st);
                const uint8_t* rs = ring + slot * kGtStage + rr * 128;
                const uint32_t ta = tmem + lane_off + kGtA0 + 128 * a;
#pragma unroll 2
                for (int gl = 0; gl < ng; ++gl) {
                    const uint8_t* bx = rs + (gl >> 2) * kGtBox;
                    const int c = (gl & 3) * 2;
                    const uint4 w0 = *reinterpret_cast<const uint4*>(bx + ((c ^ sw) << 4));
                    const uint4 w1 = *reinterpret_cast<const uint4*>(bx + (((c + 1) ^ sw) << 4));
                    const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                    uint32_t v[16];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v[2 * i] = w[i] & kLo;
                        v[2 * i + 1] = (w[i] >> 4) & kLo;
                    }
                    tmem_st16(ta + 16 * gl, v);
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&sh.afull[a]);
                    mbar_arrive(&sh.empty[slot]);
                }
            }
        }
    } else if (warp >= kGtEpiWarp0) {
        // ================= epilogue =================
        const int rr = (warp - kGtEpiWarp0) * 32 + lane;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        uint32_t q = 0;
        int jl = 0;
        bool ok = true;
        for (int job = blockIdx.x; ok && job < p.jobs; job += gridDim.x, ++jl) {
            const int b = job / p.tiles, row0 = (job - b * p.tiles) * kGtRows;
            const int js = jl & 1;
            if (!(ok = gwait(&sh.sfull[js], (jl >> 1) & 1, sh, p.err))) break;
            const ST* ss = reinterpret_cast<const ST*>(scl + (2 * js) * L.sslot) + rr * ngK;
            const ST* sb = reinterpret_cast<const ST*>(scl + (2 * js + 1) * L.sslot) + rr * ngK;
            float acc = 0.f;
            for (int st = 0; st < nst; ++st, ++q) {
                const uint32_t a = q % kGtND;
                if (!(ok = gwait(&sh.dfull[a], (q / kGtND) & 1u, sh, p.err))) break;
                tc_fence_after();
                uint32_t d[16];
                tmem_ld16(tmem + lane_off + kGtD0 + 16 * a, d);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.dempty[a]);
                const int G0 = 8 * st, ng = min(8, ngK - G0);
#pragma unroll
                for (int gl = 0; gl < 8; ++gl) {
                    if (gl < ng) {
                        const int G = G0 + gl;
                        const int dv = 128 * (int)d[2 * gl] + (int)d[2 * gl + 1];
                        acc += scale_to_float(ss[G]) * ((float)dv * xsc[G]) + scale_to_float(sb[G]) * xsum[G];
                    }
                }
            }
            if (!ok) break;
            if (row0 + rr < p.M) {
                if (p.y32)
                    p.y32[(long long)b * p.y_bstride + row0 + rr] = acc;
                else
                    p.y[(long long)b * p.y_bstride + row0 + rr] = __float2half_rn(acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.sempty[js]);
        }
    }

    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kGtTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Streaming GEMV on the integer mma.sync path (the default for many 128-row
// tiles).  Same loader and ring as above; 8 consumer warps, warp w owning rows
// 16w..16w+15 of the job, read the raw stage directly: a lane loads 8 code
// bytes of row g and of row g + 8 (the 128-byte swizzle of the TMA box is the
// engine's swizzle of an 8-row box), unpacks them to u8 (w & 0x0F0F0F0F,
// (w >> 4) & 0x0F0F0F0F) and runs m16n8k32 against the activation staged as
// in the engine's integer path (stage_x_int): the 8 MMA columns are 4 groups x
// {hi, lo}, so lane t ends a 4-group block holding group t's two int32 dots.
// The warp keeps its rows' fp32 sums for the whole job in registers.
// ---------------------------------------------------------------------------
// SPLIT = 2: 16 consumers, the warps w and w + 8 of a row tile take the
// stage's first and second TMA box (groups 0-3 / 4-7) and add their row sums
// through shared memory at the job's end.
// Exact int -> float for |v| < 2^22 with integer and FMA-pipe operations
// (1.5 * 2^23 as the magic), keeping the conversion unit out of the loop.
// The group dots it converts are at most 15 * 128 * 64 in magnitude.
__device__ __forceinline__ float i2f_small(int v) { return __int_as_float(v + 0x4B400000) - 12582912.0f; }

template <int SPLIT>
struct GsCfg {
    static constexpr int kConsumers = 8 * SPLIT;
    static constexpr int kThreads = 32 * (1 + kConsumers);
};

struct GsShared {
    uint64_t full[kGtMaxR], empty[kGtMaxR];
    uint64_t sfull[2], sempty[2];
    uint64_t pdone[8];       // SPLIT = 2: row tile w's second-half sums written
    uint64_t pfree[8];       // SPLIT = 2: ... and read by the first-half warp
    float part[kGtRows];     // SPLIT = 2: second-half row sums of the current job
    int abort_flag;
};

struct GsLayout {
    uint32_t scl, sslot, xs, xsum, xsc, sh, total;
};

// [ring: R stages][scale/bias job slots: 4 x sslot][16 zero bytes + pad][xs: K/64 x 128 B]
// [xsum, xsc: K/64 floats each][barriers]
__host__ __device__ inline GsLayout gs_layout(int K, int R) {
    const int ngK = K / 64;
    GsLayout L;
    L.scl = (uint32_t)R * kGtStage;
    L.sslot = (uint32_t)((kGtRows * ngK * 2 + 15) & ~15);
    L.xs = L.scl + 4 * L.sslot + 32;
    L.xsum = L.xs + (uint32_t)ngK * 128;
    L.xsc = L.xsum + (uint32_t)ngK * 4;
    L.sh = (L.xsc + (uint32_t)ngK * 4 + 15) & ~15u;
    L.total = L.sh + (uint32_t)sizeof(GsShared) + 1024;
    return L;
}

template <typename ST, int SPLIT>
__global__ void __launch_bounds__(GsCfg<SPLIT>::kThreads, 1) gemv_stream_kernel(const __grid_constant__ GtParams p) {
    constexpr int kConsumers = GsCfg<SPLIT>::kConsumers;
    constexpr int kThreads = GsCfg<SPLIT>::kThreads;
    extern __shared__ uint8_t gs_smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gs_smem_raw) + 1023) & ~uintptr_t(1023));
    const GsLayout L = gs_layout(p.K, p.R);
    uint8_t* ring = sm;
    uint8_t* scl = sm + L.scl;
    uint8_t* xb = sm + L.xs;
    float* xsum = reinterpret_cast<float*>(sm + L.xsum);
    float* xsc = reinterpret_cast<float*>(sm + L.xsc);
    GsShared& sh = *reinterpret_cast<GsShared*>(sm + L.sh);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ngK = p.K >> 6, nst = (ngK + 7) >> 3, R = p.R;

    if (tid == 0) {
        for (int s = 0; s < R; ++s) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], kConsumers);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&sh.sfull[a], 1);
            mbar_init(&sh.sempty[a], kConsumers);
        }
        for (int a = 0; a < 8; ++a) {
            mbar_init(&sh.pdone[a], 1);
            mbar_init(&sh.pfree[a], 1);
        }
        sh.abort_flag = 0;
        fence_mbar_init();
        prefetch_tmap(&p.wmap);
    }
    if (tid < 8) reinterpret_cast<uint32_t*>(xb - 32)[tid] = 0u;  // zero activation fragment
    stage_x_int(p.x, p.K, reinterpret_cast<uint32_t*>(xb), xsum, xsc, tid, kThreads);
    __syncthreads();

    if (warp == 0) {
        if (lane == 0) {
            const GtRing r{ring, scl, L.sslot, sh.full, sh.empty, sh.sfull, sh.sempty, &sh.abort_flag};
            gt_load_jobs(p, r);
        }
    } else {
        const int w = (warp - 1) & 7, half = (warp - 1) >> 3;  // row tile; box of the stage (SPLIT = 2)
        const int g = lane >> 2, t = lane & 3;
        const uint4* zeros = reinterpret_cast<const uint4*>(xb - 32);
        constexpr uint32_t kLo = 0x0F0F0F0Fu;
        uint32_t q = 0, rph = 0;
        int rslot = 0;
        int jl = 0;
        bool ok = true;
        for (int job = blockIdx.x; ok && job < p.jobs; job += gridDim.x, ++jl) {
            const int b = job / p.tiles, row0 = (job - b * p.tiles) * kGtRows;
            const int js = jl & 1;
            if (!(ok = gwait(&sh.sfull[js], (jl >> 1) & 1, sh.abort_flag, p.err, __LINE__, gt_info(jl, q)))) break;
            const ST* sA = reinterpret_cast<const ST*>(scl + (2 * js) * L.sslot) + (16 * w + g) * ngK;
            const ST* bA = reinterpret_cast<const ST*>(scl + (2 * js + 1) * L.sslot) + (16 * w + g) * ngK;
            const ST* sB = sA + 8 * ngK;
            const ST* bB = bA + 8 * ngK;
            float accA = 0.f, accB = 0.f;
            for (int st = 0; st < nst; ++st, ++q) {
                const int slot = rslot;
                if (!(ok = gwait(&sh.full[slot], rph, sh.abort_flag, p.err, __LINE__, gt_info(jl, q)))) break;
                if (++rslot == R) {  // ring position without a division per stage
                    rslot = 0;
                    rph ^= 1u;
                }
                const uint8_t* rowA = ring + slot * kGtStage + (16 * w + g) * 128;
                const int ng = min(8, ngK - 8 * st);
                // one block of 4 groups = one TMA box (k): two interleaved MMA
                // chains; lane t ends with group t's dots
                auto block = [&](const int k, int c[2][4]) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int gl = 4 * k + j;
                        if (gl < ng) {
                            const int G = 8 * st + gl;
                            const uint4* xp = ((g >> 1) == j)
                                                  ? reinterpret_cast<const uint4*>(xb + (G * 4 + t) * 32) + (g & 1)
                                                  : zeros;
                            const uint4 xv = xp[0];
                            const int o = k * kGtBox + ((((j * 2 + (t >> 1)) ^ g) & 7) << 4) + (t & 1) * 8;
                            const uint2 wa = *reinterpret_cast<const uint2*>(rowA + o);
                            const uint2 wb = *reinterpret_cast<const uint2*>(rowA + 8 * 128 + o);
                            const uint32_t a0 = wa.x & kLo, a1 = (wa.x >> 4) & kLo;
                            const uint32_t a2 = wa.y & kLo, a3 = (wa.y >> 4) & kLo;
                            const uint32_t b0 = wb.x & kLo, b1 = (wb.x >> 4) & kLo;
                            const uint32_t b2 = wb.y & kLo, b3 = (wb.y >> 4) & kLo;
                            imma16832(c[0], a0, b0, a1, b1, xv.x, xv.y);
                            imma16832(c[1], a2, b2, a3, b3, xv.z, xv.w);
                        }
                    }
                };
                auto finish = [&](const int k, const int c[2][4]) {
                    if (4 * k + t < ng) {
                        const int G = 8 * st + 4 * k + t;
                        const float xc = xsc[G], xm = xsum[G];
                        const float dA = fmaf(128.f, i2f_small(c[0][0] + c[1][0]), i2f_small(c[0][1] + c[1][1]));
                        const float dB = fmaf(128.f, i2f_small(c[0][2] + c[1][2]), i2f_small(c[0][3] + c[1][3]));
                        accA += scale_to_float(sA[G]) * (dA * xc) + scale_to_float(bA[G]) * xm;
                        accB += scale_to_float(sB[G]) * (dB * xc) + scale_to_float(bB[G]) * xm;
                    }
                };
                if constexpr (SPLIT == 2) {
                    int c[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
                    block(half, c);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sh.empty[slot]);  // codes are in registers
                    finish(half, c);
                } else {
                    int c0[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}}, c1[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
                    block(0, c0);
                    block(1, c1);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&sh.empty[slot]);
                    finish(0, c0);
                    finish(1, c1);
                }
            }
            if (!ok) break;
            accA += __shfl_xor_sync(0xffffffffu, accA, 1);
            accA += __shfl_xor_sync(0xffffffffu, accA, 2);
            accB += __shfl_xor_sync(0xffffffffu, accB, 1);
            accB += __shfl_xor_sync(0xffffffffu, accB, 2);
            if constexpr (SPLIT == 2) {
                // the second-half warp hands its row sums over (pdone) and
                // writes the next job's only after the first-half warp read
                // them (pfree): with jobs shorter than the ring a warp can run
                // two jobs ahead of its partner, so a one-way barrier's parity
                // would wrap
                float* part = sh.part;
                if (half == 1) {
                    if (!(ok = gwait(&sh.pfree[w], (jl & 1) ^ 1, sh.abort_flag, p.err, __LINE__, gt_info(jl, q))))
                        break;
                    if (t == 0) {
                        part[16 * w + g] = accA;
                        part[16 * w + 8 + g] = accB;
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(&sh.pdone[w]);
                        mbar_arrive(&sh.sempty[js]);
                    }
                    continue;
                }
                if (!(ok = gwait(&sh.pdone[w], jl & 1, sh.abort_flag, p.err, __LINE__, gt_info(jl, q)))) break;
                accA += part[16 * w + g];
                accB += part[16 * w + 8 + g];
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.pfree[w]);
            }
            const int rA = row0 + 16 * w + g;
            if (p.y32) {
                float* yb = p.y32 + (long long)b * p.y_bstride;
                if (t == 0 && rA < p.M) yb[rA] = accA;
                if (t == 1 && rA + 8 < p.M) yb[rA + 8] = accB;
            } else {
                __half* yb = p.y + (long long)b * p.y_bstride;
                if (t == 0 && rA < p.M) yb[rA] = __float2half_rn(accA);
                if (t == 1 && rA + 8 < p.M) yb[rA + 8] = __float2half_rn(accB);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh.sempty[js]);
        }
    }
    __syncthreads();
}

// uint8 [depth][rows][row_bytes] in boxes of 128 B x 128 rows, 128-byte swizzle.
bool make_gt_map(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint64_t depth,
                 uint64_t depth_stride) {
    memset(m, 0, sizeof(*m));
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || !aligned16(base) || row_bytes % 16 || rows == 0 || depth == 0) return false;
    const uint64_t ds = depth > 1 ? depth_stride : row_bytes * rows;
    if (ds % 16 || ds >= (1ull << 40)) return false;
    cuuint64_t dims[3] = {row_bytes, rows, depth};
    cuuint64_t strides[2] = {row_bytes, ds};
    cuuint32_t box[3] = {128, (cuuint32_t)kGtRows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int gt_ring_stages(int K) {
    const GtLayout L0 = gt_layout(K, 0);
    const long long left = (long long)kGtSmemLimit - (long long)L0.total;
    return (int)std::min<long long>(kGtMaxR, left / kGtStage);
}

int gs_ring_stages(int K) {
    const GsLayout L0 = gs_layout(K, 0);
    const long long left = (long long)kGtSmemLimit - (long long)L0.total;
    return (int)std::min<long long>(kGtMaxR, left / kGtStage);
}

template <typename ST, int SPLIT>
tf_status launch_gemv_stream_split(tf_context* ctx, const GtParams& p, cudaStream_t stream, const char* name) {
    const GsLayout L = gs_layout(p.K, p.R);
    const void* fn = reinterpret_cast<const void*>(&gemv_stream_kernel<ST, SPLIT>);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return cuda_check(ctx, e, name);
    const int grid = std::min(ctx->num_sms, p.jobs);
    gemv_stream_kernel<ST, SPLIT><<<grid, GsCfg<SPLIT>::kThreads, L.total, stream>>>(p);
    return cuda_check(ctx, cudaGetLastError(), name);
}

// TFCUDA_GEMV_SPLIT=1 selects 8 consumer warps instead of 16 (read per call).
template <typename ST>
tf_status launch_gemv_stream(tf_context* ctx, const GtParams& p, cudaStream_t stream, const char* name) {
    const char* e = getenv("TFCUDA_GEMV_SPLIT");
    if (e && e[0] == '1') return launch_gemv_stream_split<ST, 1>(ctx, p, stream, name);
    return launch_gemv_stream_split<ST, 2>(ctx, p, stream, name);
}

template <typename ST>
tf_status launch_gemv_tc(tf_context* ctx, const GtParams& p, cudaStream_t stream, const char* name) {
    const GtLayout L = gt_layout(p.K, p.R);
    const void* fn = reinterpret_cast<const void*>(&gemv_tc_kernel<ST>);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) return cuda_check(ctx, e, name);
    const int grid = std::min(ctx->num_sms, p.jobs);
    gemv_tc_kernel<ST><<<grid, kGtThreads, L.total, stream>>>(p);
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // namespace

namespace tf {

tf_status gemv_tc_try(tf_context* ctx, const void* W, const void* S, const void* B, uint64_t wbs, uint64_t sbs,
                      uint32_t batch, const void* x, void* y, uint64_t ybs, uint32_t m, uint32_t n,
                      tf_scale_type st, cudaStream_t stream, int kind, int force, bool* used, const char* name) {
    *used = false;
    if (n % 64 || n / 2 % 16) return TF_OK;
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return TF_OK;
    if (!aligned16(S) || !aligned16(B) || (batch > 1 && (sbs * 2) % 16)) return TF_OK;
    const int tiles = (int)((m + kGtRows - 1) / kGtRows);
    const long long jobs = (long long)tiles * batch;
    if (jobs > (1ll << 30)) return TF_OK;
    if (!force && jobs < ctx->num_sms) return TF_OK;  // too few tiles to fill the GPU: the engine splits K
    const int R = kind == kGemvTensorCore ? gt_ring_stages((int)n) : gs_ring_stages((int)n);
    if (R < 2) return TF_OK;
    GtParams p;
    memset(&p, 0, sizeof(p));
    if (!make_gt_map(&p.wmap, W, n / 2, m, batch, wbs)) return TF_OK;
    p.S = static_cast<const uint8_t*>(S);
    p.B = static_cast<const uint8_t*>(B);
    p.sb_bstride = (long long)sbs * 2;
    p.x = static_cast<const __half*>(x);
    p.y = static_cast<__half*>(y);
    p.y_bstride = (long long)ybs;
    p.M = (int)m;
    p.K = (int)n;
    p.batch = (int)batch;
    p.tiles = tiles;
    p.jobs = (int)jobs;
    p.R = R;
    p.err = ctx->d_err;
    *used = true;
    if (kind == kGemvTensorCore)
        return st == TF_SCALE_BF16 ? launch_gemv_tc<__nv_bfloat16>(ctx, p, stream, name)
                                   : launch_gemv_tc<__half>(ctx, p, stream, name);
    return st == TF_SCALE_BF16 ? launch_gemv_stream<__nv_bfloat16>(ctx, p, stream, name)
                               : launch_gemv_stream<__half>(ctx, p, stream, name);
}

}  // namespace tf

namespace tf {

// One-token int4 GEMV on the ring-streamed kernel with fp32 output (the LM
// head's logits).  Returns TF_ERR_UNSUPPORTED_SHAPE when the shape does not
// suit the kernel (n % 64, fewer row tiles than SMs, misaligned scales).
tf_status gemv_stream_f32(tf_context* ctx, const void* W, const void* S, const void* B, const void* x, float* y32,
                          uint32_t m, uint32_t n, tf_scale_type st, cudaStream_t stream, const char* name) {
    if (n % 64 || n / 2 % 16 || !aligned16(S) || !aligned16(B) || (st != TF_SCALE_BF16 && st != TF_SCALE_F16))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: shape or alignment unsupported by the streaming GEMV", name);
    const int tiles = (int)((m + kGtRows - 1) / kGtRows);
    const int R = gs_ring_stages((int)n);
    if (R < 2) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: K too large for the streaming GEMV", name);
    GtParams p;
    memset(&p, 0, sizeof(p));
    if (!make_gt_map(&p.wmap, W, n / 2, m, 1, 0))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: weights must be 16-byte aligned", name);
    p.S = static_cast<const uint8_t*>(S);
    p.B = static_cast<const uint8_t*>(B);
    p.x = static_cast<const __half*>(x);
    p.y32 = y32;
    p.M = (int)m;
    p.K = (int)n;
    p.batch = 1;
    p.tiles = tiles;
    p.jobs = tiles;
    p.R = R;
    p.err = ctx->d_err;
    return st == TF_SCALE_BF16 ? launch_gemv_stream<__nv_bfloat16>(ctx, p, stream, name)
                               : launch_gemv_stream<__half>(ctx, p, stream, name);
}

}  // namespace tf
