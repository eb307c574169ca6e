// tf_qmm.cu -- prefill GEMMs with int4 affine (MLX group-64) weights on the
// 5th-generation tensor cores (tcgen05 + TMEM).
//
// Reference kernels replaced:
//   prefill_dequant_int4_qmm_f16_block  (Metal/Prefill/prefill.metal:672-709,
//       PrefillInt4QMM.encode, Kernels/Prefill/Primitives/PrefillPrimitives.swift:73-122)
//   mpp_prefill_affine_threadgroup_f16  (Metal/TensorCore/tensorops.metal:8-105,
//       MPPPrefillInt4QMM.encode) -- the same "dequantise a weight tile to fp16
//       in on-chip memory, then run the matrix unit" scheme, here at 128 x 256.
//   prefill_grouped_routed_moe_batched_phase1 / _down (prefill.metal:336-440,
//       598-670; PrefillGroupedRoutedMoE.encodeStreamedBatched,
//       Kernels/Prefill/MoE/PrefillGroupedRoutedMoE.swift:446-527)
//   prefill_moe_reduce_token_major (prefill.metal:575-596; PrefillMoE.swift:11-40)
//
// One persistent kernel, one CTA per SM, warp-specialised:
//   warps 0-3   epilogue: tcgen05.ld of the fp32 accumulator (TMEM lane = weight
//               row), fused GELU(gate)*up, fp16 stores
//   warp 4      loader: one thread issues, per k-block, the TMA loads of the
//               raw int4 weight tile (2 boxes of 64 rows x 32 B, 3-D maps so
//               a pool expert is one coordinate) and of the activation rows
//               (64-row boxes, 128-byte swizzle = the K-major operand layout,
//               only as many boxes as the tile has rows)
//   warps 5-12  dequantiser: raw nibbles from shared memory + bf16/fp16
//               scale/bias -> fp16 w = fma(q, s, b) (one rounding) in the
//               swizzled K-major layout; scales come through a register ring
//   warp 13     TMEM allocation and the single-thread tcgen05.mma issue
// Tile: 128 weight rows (M) x up to 256 tokens (N), k-block 64 (= one
// quantisation group), 4 shared-memory stages of 52 KB, two TMEM accumulators
// of 256 fp32 columns so the epilogue of one tile overlaps the next tile's
// main loop.  Gate/up projections interleave their rows (even = gate, odd = up)
// so a lane pair holds both operands of GELU(g)*u after one shuffle.  Routed
// rows are first gathered into sorted-pair order (gather_rows_kernel) so that
// every expert's tokens are one contiguous TMA range.
#include <type_traits>

#include "tf_context.cuh"
#include "tf_gemv_tc.cuh"
#include "tf_umma.cuh"

using namespace tf;

namespace {

constexpr int kEpiWarps = 4;
constexpr int kLoadWarp = 4;
constexpr int kAWarps = 8;
constexpr int kAWarp0 = 5;
constexpr int kMmaWarp = kAWarp0 + kAWarps;  // 13
constexpr int kScaleWarp = kMmaWarp + 1;       // 14, 15
constexpr int kScaleWarps = 2;
constexpr int kQWarps = kScaleWarp + kScaleWarps;
constexpr int kQThreads = kQWarps * 32;
constexpr int kTM = 128;               // weight rows per CTA (MMA M per CTA)
constexpr int kTN = 256;               // tokens per tile (MMA N, max)
constexpr int kAStage = kTM * 128;     // 16 KB fp16 operand
constexpr int kRawStage = kTM * 32;    // 4 KB packed int4
constexpr int kBBoxRows = 64;          // rows per activation TMA box (8 KB)
constexpr int kAccCols = 256;
constexpr int kTmemCols = 512;
constexpr int kMaxGroups = 256;
constexpr uint32_t kQSpin = 1u << 24;

// Optional per-role timestamps of CTA 0 (SM clock), for pipeline studies:
// built only with -DTF_QMM_TRACE, read back with tf_debug_qmm_trace.
#ifdef TF_QMM_TRACE
__device__ unsigned long long g_qmm_trace[8][512];
#define QTRACE(ev, i)                                                              \
    do {                                                                           \
        if (blockIdx.x == 0 && (i) < 512) g_qmm_trace[ev][i] = (unsigned long long)clock64(); \
    } while (0)
#else
#define QTRACE(ev, i) \
    do {              \
    } while (0)
#endif

// CG = CTAs per MMA (1: one SM, 128 x N tiles; 2: a CTA pair, 256 x N tiles,
// each CTA holding half of the weight rows and half of the token rows).
// TN = tokens per tile: 256, or 64 for few tokens per tile (a smaller
// activation stage buys a deeper load ring and dequantised-operand ring).
template <int CG, int TN = kTN>
struct QCfg {
    static constexpr int kTN = TN;
    static constexpr int kStages = TN == 256 ? (CG == 2 ? 9 : 5) : (CG == 2 ? 14 : 12);  // load ring
    static constexpr int kAStages = TN == 256 ? 2 : 4;  // dequantised operand ring
    static constexpr int kBRows = TN / CG;              // token rows staged per CTA
    static constexpr int kBStage = kBRows * 128;
    static constexpr int kSStage = kTM * 4;          // fp16 scale | bias per weight row
    static constexpr int kScaleAhead = 8;            // scale loads in flight (k-blocks)
};

enum QMode : int { kDensePlain = 0, kDenseGateUp = 1, kGroupedGateUp = 2, kGroupedDown = 3 };

struct QmmParams {
    CUtensorMap xmap;   // activations [rows][K] fp16, 64-row boxes
    CUtensorMap xmap256;  // the same with 256-row boxes (one TMA per k-block for a full tile), if xbig
    CUtensorMap wmap0;  // packed weights (plain / gate), [depth][rows][K/2] uint8
    CUtensorMap wmap1;  // packed weights (up)
    int mode;
    int K;      // reduction length (multiple of 64)
    int nfeat;  // rows of one weight matrix (output features)
    int T;      // dense: tokens
    // scales/biases of matrix 0 (plain / gate) and 1 (up); grouped: offsets
    // from the expert's blob at pool + e*stride
    const uint8_t* sbase;
    uint64_t stride;
    uint64_t os0, ob0, os1, ob1;
    uint32_t num_experts;
    const tf_moe_group* groups;
    const uint32_t* n_groups;
    const tf_token_expert_pair* pairs;
    int top_k;
    __half* y;
    float* y32;  // dense plain mode: fp32 output instead of y (NULL = fp16 y)
    long long ldy;
    int round_gu;  // gate/up rounded to fp16 before GELU (shared expert)
    int small_tiles;  // grouped: 64-token tiles (few tokens per expert expected)
    int xbig;         // xmap256 is valid
    int ksplit;       // dense: K split over this many CTAs (tiles x ksplit jobs), >= 1
    float* part;      // ksplit > 1: fp32 partials [ksplit][T][ldp] (gate/up interleaved per feature)
    long long ldp;
    int wbig;         // plain modes: wmap0 has 128-row boxes (one TMA per k-block)
    uint32_t* err;
};

template <int CG, int TN = kTN>
struct QShared {
    static constexpr int S = QCfg<CG, TN>::kStages;
    static constexpr int SA = QCfg<CG, TN>::kAStages;
    static constexpr int kCG = CG;
    static constexpr int kTileN = TN;
    uint64_t rawfull[S];  // this CTA's raw weight bytes landed
    uint64_t bfull[S];    // (leader) activation bytes of the pair landed
    uint64_t empty[S];    // MMAs reading the stage's token rows retired (both CTAs)
    uint64_t sfull[S];    // scales of the stage written
    uint64_t sempty[S];   // scales of the stage read by every dequantiser warp
    uint64_t afull[SA];   // (leader) dequantised operand of the pair written
    uint64_t aempty[SA];  // MMAs reading the operand retired (both CTAs)
    uint64_t tfull[2];
    uint64_t tempty[2];   // (leader) epilogues of the pair released the accumulator
    uint64_t done;
    uint32_t tmem_base;
    int abort_flag;
    int ng;
    int total;
    int prefix[kMaxGroups + 1];
    int gstart[kMaxGroups];
    int gcount[kMaxGroups];
    int gexpert[kMaxGroups];
};

template <int CG, int TN = kTN>
constexpr size_t qsmem_bytes() {
    using C = QCfg<CG, TN>;
    return 1024 + (size_t)C::kAStages * kAStage +
           (size_t)C::kStages * (C::kBStage + kRawStage + C::kSStage) + sizeof(QShared<CG, TN>);
}
static_assert(qsmem_bytes<1>() <= 232448 && qsmem_bytes<2>() <= 232448, "shared memory");
static_assert(qsmem_bytes<1, 64>() <= 232448, "shared memory");
static_assert(QCfg<1, 64>::kBRows % kBBoxRows == 0, "a token stage holds whole activation boxes");

struct QTile {
    int feat0;
    int row0;  // dense: first token row; grouped: first sorted pair
    int cnt;   // tokens / pairs in the tile
    int expert;
    int split;  // dense split-K: which K slice
    int kb0;    // first k-block of the slice
};

__device__ __forceinline__ bool gate_up(int mode) { return mode == kDenseGateUp || mode == kGroupedGateUp; }
__device__ __forceinline__ bool grouped(int mode) { return mode == kGroupedGateUp || mode == kGroupedDown; }
// output features covered by one tile
__device__ __forceinline__ int feat_per_tile(int mode, int cg) { return (gate_up(mode) ? kTM / 2 : kTM) * cg; }

template <class SH>
__device__ __forceinline__ bool decode_tile(const QmmParams& p, const SH& sh, int idx, QTile& t) {
    constexpr int CG = SH::kCG, kTN = SH::kTileN;
    if (idx >= sh.total) return false;
    const int fpt = feat_per_tile(p.mode, CG);
    const int nft = (p.nfeat + fpt - 1) / fpt;
    if (!grouped(p.mode)) {
        const int tile = idx / p.ksplit, sp = idx - tile * p.ksplit;
        const int tt = tile / nft, ft = tile - tt * nft;
        t.feat0 = ft * fpt;
        t.row0 = tt * kTN;
        t.cnt = min(kTN, p.T - t.row0);
        t.expert = 0;
        t.split = sp;
        t.kb0 = sp * ((p.K >> 6) / p.ksplit);
        return true;
    }
    // largest g with prefix[g] <= idx
    int lo = 0, hi = sh.ng - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sh.prefix[mid] <= idx) lo = mid; else hi = mid - 1;
    }
    const int g = lo, local = idx - sh.prefix[g], c = sh.gcount[g];
    const int ntt = (c + kTN - 1) / kTN;
    const int q = (c + ntt - 1) / ntt;
    const int tt = local / nft, ft = local - tt * nft;
    t.feat0 = ft * fpt;
    t.row0 = sh.gstart[g] + tt * q;
    t.cnt = min(q, c - tt * q);
    t.expert = sh.gexpert[g];
    t.split = 0;
    t.kb0 = 0;
    return true;
}

// Bounded wait that gives up early once another role of this CTA has given up.
template <class SH>
__device__ __forceinline__ bool qwait(uint64_t* bar, uint32_t parity, SH& sh, uint32_t* err) {
    for (uint32_t i = 0; i < kQSpin; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *reinterpret_cast<volatile int*>(&sh.abort_flag)) return false;
    }
    sh.abort_flag = 1;
    if (err) atomicOr(err, kErrMbarTimeout);
    return false;
}

// arrive on the pair leader's copy of `bar` (this CTA's own when CG == 1)
template <int CG>
__device__ __forceinline__ void arrive_leader(uint64_t* bar) {
    if constexpr (CG == 1)
        mbar_arrive(bar);
    else
        mbar_arrive_cluster(mapa_shared(bar, 0));
}

__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

__device__ __forceinline__ void tma_load_3d_u8(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// fp16 bits of raw bf16 / fp16 scale or bias bits
template <typename ST>
__device__ __forceinline__ uint32_t scale_raw_f16(uint32_t raw) {
    if constexpr (std::is_same<ST, __half>::value)
        return raw;
    else
        return (uint32_t)__half_as_ushort(__float2half_rn(__uint_as_float(raw << 16)));
}


// 8 nibbles (elements 8c..8c+7, low nibble first) -> 4 half2 in k order,
// w_k = fma(q_k, s, b) rounded once to fp16.
__device__ __forceinline__ void dq8_natural(uint32_t w, uint32_t s2, uint32_t b2, uint32_t o[4]) {
    constexpr uint32_t k1024 = 0x64006400u;
    const uint32_t t = w & 0x0F0F0F0Fu;          // e0 e2 e4 e6
    const uint32_t u = (w >> 4) & 0x0F0F0F0Fu;   // e1 e3 e5 e7
    const uint32_t lo = __byte_perm(t, u, 0x5140);  // e0 e1 e2 e3
    const uint32_t hi = __byte_perm(t, u, 0x7362);  // e4 e5 e6 e7
    const uint32_t m = 0x64646464u;
    o[0] = hfma2_u(hsub2_u(__byte_perm(lo, m, 0x4140), k1024), s2, b2);
    o[1] = hfma2_u(hsub2_u(__byte_perm(lo, m, 0x4342), k1024), s2, b2);
    o[2] = hfma2_u(hsub2_u(__byte_perm(hi, m, 0x4140), k1024), s2, b2);
    o[3] = hfma2_u(hsub2_u(__byte_perm(hi, m, 0x4342), k1024), s2, b2);
}

// Iteration cursor over (tile, k-block) of this CTA (pair).
struct QCursor {
    int idx, kb;
    bool valid;
    QTile t;
};

template <class SH>
__device__ __forceinline__ void cursor_start(const QmmParams& p, const SH& sh, QCursor& c) {
    c.idx = blockIdx.x / SH::kCG;
    c.kb = 0;
    c.valid = decode_tile(p, sh, c.idx, c.t);
}

template <class SH>
__device__ __forceinline__ void cursor_next(const QmmParams& p, const SH& sh, QCursor& c, int nkb) {
    if (!c.valid) return;
    if (++c.kb == nkb) {
        c.kb = 0;
        c.idx += gridDim.x / SH::kCG;
        c.valid = decode_tile(p, sh, c.idx, c.t);
    }
}

// first output feature of this CTA's 128 weight rows
template <int CG>
__device__ __forceinline__ int cta_feat0(const QmmParams& p, const QTile& t, int rank) {
    return t.feat0 + rank * (gate_up(p.mode) ? kTM / 2 : kTM);
}

// Scale and bias rows of weight row r (0..127 of this CTA) in the cursor's
// tile; null when the row is past the matrix (it then dequantises to 0).
template <typename ST, int CG>
__device__ __forceinline__ const ST* scale_row(const QmmParams& p, const QTile& t, int r, int rank, bool bias) {
    const bool gu = gate_up(p.mode);
    const int mat = gu ? (r & 1) : 0;
    const int f = cta_feat0<CG>(p, t, rank) + (gu ? (r >> 1) : r);
    if (f >= p.nfeat) return nullptr;
    // dense: os/ob are addresses; grouped: byte offsets inside the expert's blob
    const uint64_t base = grouped(p.mode) ? reinterpret_cast<uint64_t>(p.sbase) + (uint64_t)t.expert * p.stride : 0;
    const uint64_t off = bias ? (mat ? p.ob1 : p.ob0) : (mat ? p.os1 : p.os0);
    return reinterpret_cast<const ST*>(base + off) + (size_t)f * (p.K >> 6);
}

template <typename ST, int CG, int TN>
__global__ void __launch_bounds__(kQThreads, 1) qmm_kernel(const __grid_constant__ QmmParams p) {
    using Cfg = QCfg<CG, TN>;
    constexpr int kTN = TN;
    constexpr int S = Cfg::kStages;
    constexpr int SA = Cfg::kAStages;
    extern __shared__ uint8_t q_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(q_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* As = smem;
    uint8_t* Bs = As + SA * kAStage;
    uint8_t* Ws = Bs + S * Cfg::kBStage;
    uint32_t* Ss = reinterpret_cast<uint32_t*>(Ws + S * kRawStage);
    QShared<CG, TN>& sh = *reinterpret_cast<QShared<CG, TN>*>(reinterpret_cast<uint8_t*>(Ss) + S * Cfg::kSStage);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = CG == 2 ? (int)cluster_ctarank() : 0;
    const bool leader = rank == 0;
    const int nkb = (p.K >> 6) / p.ksplit;  // k-blocks per job
    const int fpt = feat_per_tile(p.mode, CG);
    const int nft = (p.nfeat + fpt - 1) / fpt;

    // ---- setup: barriers, tile table, TMEM ----
    if (tid == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&sh.rawfull[s], 1);
            mbar_init(&sh.bfull[s], CG);
            mbar_init(&sh.empty[s], 1);
            mbar_init(&sh.sfull[s], kScaleWarps);
            mbar_init(&sh.sempty[s], kAWarps / SA);
        }
        for (int a = 0; a < SA; ++a) {
            mbar_init(&sh.afull[a], (kAWarps / SA) * CG);
            mbar_init(&sh.aempty[a], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&sh.tfull[a], 1);
            mbar_init(&sh.tempty[a], kEpiWarps * CG);
        }
        mbar_init(&sh.done, 1);
        sh.abort_flag = 0;
        fence_mbar_init();
    }
    if (!grouped(p.mode)) {
        if (tid == 0) {
            sh.ng = 0;
            sh.total = ((p.T + kTN - 1) / kTN) * nft * p.ksplit;
        }
    } else if (warp == 0) {
        const int ng = min((int)*p.n_groups, kMaxGroups);
        // each lane owns 8 consecutive groups
        int cnt[8];
        int run = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int g = lane * 8 + j;
            int tiles = 0;
            if (g < ng) {
                const tf_moe_group gr = p.groups[g];
                sh.gstart[g] = (int)gr.pair_start;
                sh.gcount[g] = (int)gr.pair_count;
                sh.gexpert[g] = (int)gr.expert;
                if (gr.expert < p.num_experts) {
                    tiles = (((int)gr.pair_count + kTN - 1) / kTN) * nft;
                } else if (p.err && rank == 0) {
                    atomicOr(p.err, kErrBadExpert);
                }
            }
            cnt[j] = tiles;
            run += tiles;
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
            if (g <= ng) sh.prefix[g] = acc;
            acc += cnt[j];
        }
        if (lane == 31) sh.total = incl;
        if (lane == 0) sh.ng = ng;
        if (ng == kMaxGroups && lane == 31) sh.prefix[kMaxGroups] = incl;
    }
    if (warp == kMmaWarp) {
        if constexpr (CG == 2)
            tmem_alloc_pair(&sh.tmem_base, kTmemCols);
        else
            tmem_alloc(&sh.tmem_base, kTmemCols);
        tc_fence_before();
    }
    __syncthreads();
    if constexpr (CG == 2) cluster_sync_all();  // peer barriers initialised, TMEM of both allocated
    tc_fence_after();
    const uint32_t tmem = sh.tmem_base;

    if (warp >= kAWarp0 && warp < kMmaWarp) {
        // ================= dequantiser =================
        // k-blocks of this CTA: nkb per tile, tiles blockIdx/CG, + units, ...
        const int units = gridDim.x / CG, u0 = blockIdx.x / CG;
        const int iters = (sh.total > u0 ? (sh.total - u0 + units - 1) / units : 0) * nkb;
        // SA groups of kAWarps / SA warps: group a dequantises the k-blocks
        // it = a, a + SA, ... (operand buffer a), so SA k-blocks are in
        // flight at once and each group's barrier round trips overlap the
        // others' work; a thread covers kUnits (row, half-row) units.
        constexpr int kGW = kAWarps / SA;          // warps per group
        constexpr int kUnits = 256 / (32 * kGW);   // 16-byte raw units per thread
        const int grp = (warp - kAWarp0) / kGW;
        const int gt = ((warp - kAWarp0) % kGW) * 32 + lane;
        for (int it = grp; it < iters; it += SA) {
            const int s = it % S, a = grp;
            const uint32_t ps = (uint32_t)(it / S) & 1u, pa = (uint32_t)(it / SA) & 1u;
            const bool tr = (warp - kAWarp0) % kGW == 0 && lane == 0;
            if (!qwait(&sh.rawfull[s], ps, sh, p.err)) break;
            if (tr) QTRACE(1, it);
            if (!qwait(&sh.sfull[s], ps, sh, p.err)) break;
            if (tr) QTRACE(2, it);
            if (!qwait(&sh.aempty[a], pa ^ 1u, sh, p.err)) break;
            if (tr) QTRACE(3, it);
            const uint32_t dst = smem_u32(As + a * kAStage);
            uint4 q[kUnits];
            uint32_t sb[kUnits];
#pragma unroll
            for (int u = 0; u < kUnits; ++u) {
                const int at = gt + u * 32 * kGW;  // 0..255
                const int r = at >> 1, h = at & 1;
                // raw rows: plain = r; gate/up = gate rows 0-63, up rows 64-127
                const int rr = gate_up(p.mode) ? ((r & 1) * 64 + (r >> 1)) : r;
                q[u] = lds128(smem_u32(Ws + s * kRawStage + rr * 32 + h * 16));
                sb[u] = Ss[s * kTM + r];
            }
#pragma unroll
            for (int u = 0; u < kUnits; ++u) {
                const int at = gt + u * 32 * kGW;
                const int r = at >> 1, h = at & 1;
                const uint32_t s2 = (sb[u] & 0xFFFFu) * 0x10001u, b2 = (sb[u] >> 16) * 0x10001u;
                const uint32_t wv[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    uint32_t o[4];
                    dq8_natural(wv[i], s2, b2, o);
                    sts128(dst + sw128(r, h * 4 + i), o[0], o[1], o[2], o[3]);
                }
            }
            fence_proxy_async_smem();
            // the leader's warps also wait for the stage's token rows, so a
            // full afull implies a full bfull: the MMA thread (the serial step
            // of the pipeline) then waits on one barrier per k-block
            if (leader && !qwait(&sh.bfull[s], ps, sh, p.err)) break;
            __syncwarp();
            if (lane == 0) {
                if ((warp - kAWarp0) % kGW == 0) QTRACE(4, it);
                arrive_leader<CG>(&sh.afull[a]);
                mbar_arrive(&sh.sempty[s]);
            }
        }
    } else if (warp >= kScaleWarp) {
        // ================= scale / bias loader =================
        // two warps, 2 weight rows per lane; loads run kScaleAhead k-blocks
        // ahead of use; row pointers are set once per tile
        constexpr int D = Cfg::kScaleAhead;
        const int r0 = (warp - kScaleWarp) * 64 + lane;  // rows r0, r0 + 32
        QCursor lc;
        cursor_start(p, sh, lc);
        const int units = gridDim.x / CG, u0 = blockIdx.x / CG;
        const int iters = (sh.total > u0 ? (sh.total - u0 + units - 1) / units : 0) * nkb;
        const ST* ps[2] = {nullptr, nullptr};
        const ST* pb[2] = {nullptr, nullptr};
        // the ring holds the raw 16-bit loads: nothing reads a loaded
        // register until its k-block is consumed D blocks later, so the loads
        // stay in flight (converting at fetch time would wait for each one)
        auto fetch = [&](uint32_t v[4]) {
            if (lc.valid && lc.kb == 0) {
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    ps[i] = scale_row<ST, CG>(p, lc.t, r0 + 32 * i, rank, false);
                    pb[i] = scale_row<ST, CG>(p, lc.t, r0 + 32 * i, rank, true);
                }
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const bool ok = lc.valid && ps[i];
                v[2 * i] = ok ? (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(ps[i] + lc.t.kb0 + lc.kb)) : 0u;
                v[2 * i + 1] = ok ? (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(pb[i] + lc.t.kb0 + lc.kb)) : 0u;
            }
            cursor_next(p, sh, lc, nkb);
        };
        uint32_t ring[D][4];
#pragma unroll
        for (int j = 0; j < D; ++j) fetch(ring[j]);
        bool live = true;
        for (int it0 = 0; it0 < iters && live; it0 += D) {
#pragma unroll
            for (int j = 0; j < D; ++j) {
                const int it = it0 + j;
                if (it >= iters) break;
                const uint32_t c0 = scale_raw_f16<ST>(ring[j][0]) | (scale_raw_f16<ST>(ring[j][1]) << 16);
                const uint32_t c1 = scale_raw_f16<ST>(ring[j][2]) | (scale_raw_f16<ST>(ring[j][3]) << 16);
                fetch(ring[j]);
                const int s = it % S;
                if (!qwait(&sh.sempty[s], (((uint32_t)(it / S)) & 1u) ^ 1u, sh, p.err)) {
                    live = false;
                    break;
                }
                Ss[s * kTM + r0] = c0;
                Ss[s * kTM + r0 + 32] = c1;
                __syncwarp();
                if (lane == 0) mbar_arrive(&sh.sfull[s]);
            }
        }
    } else if (warp == kLoadWarp) {
        // ================= TMA loader (one thread) =================
        if (lane == 0) {
            prefetch_tmap(&p.xmap);
            if (p.xbig) prefetch_tmap(&p.xmap256);
            prefetch_tmap(&p.wmap0);
            if (gate_up(p.mode)) prefetch_tmap(&p.wmap1);
            QCursor cur;
            cursor_start(p, sh, cur);
            int it = 0;
            while (cur.valid) {
                const int s = it % S;
                if (!qwait(&sh.empty[s], ((uint32_t)(it / S) & 1u) ^ 1u, sh, p.err)) break;
                QTRACE(0, it);
                // raw int4 weight rows of this CTA -> local barrier
                mbar_arrive_expect_tx(&sh.rawfull[s], (uint32_t)kRawStage);
                uint8_t* w = Ws + s * kRawStage;
                const int z = cur.t.expert, fb = cta_feat0<CG>(p, cur.t, rank);
                if (gate_up(p.mode)) {
                    tma_load_3d_u8(w, &p.wmap0, (cur.t.kb0 + cur.kb) * 32, fb, z, &sh.rawfull[s]);
                    tma_load_3d_u8(w + kRawStage / 2, &p.wmap1, (cur.t.kb0 + cur.kb) * 32, fb, z, &sh.rawfull[s]);
                } else if (p.wbig) {
                    tma_load_3d_u8(w, &p.wmap0, (cur.t.kb0 + cur.kb) * 32, fb, z, &sh.rawfull[s]);  // 128 rows
                } else {
                    tma_load_3d_u8(w, &p.wmap0, (cur.t.kb0 + cur.kb) * 32, fb, z, &sh.rawfull[s]);
                    tma_load_3d_u8(w + kRawStage / 2, &p.wmap0, (cur.t.kb0 + cur.kb) * 32, fb + 64, z, &sh.rawfull[s]);
                }
                // this CTA's token rows -> the leader's barrier
                const int N = max(16, (cur.t.cnt + 15) & ~15);
                const int brows = CG == 2 ? N / 2 : cur.t.cnt;
                const int brow0 = cur.t.row0 + rank * (N / 2);
                const int nbox = (brows + kBBoxRows - 1) / kBBoxRows;
                uint8_t* dst = Bs + s * Cfg::kBStage;
                if constexpr (CG == 2) {
                    const uint32_t lb = mapa_shared(&sh.bfull[s], 0);
                    mbar_arrive_expect_tx_cluster(lb, (uint32_t)(nbox * kBBoxRows * 128));
                    for (int i = 0; i < nbox; ++i)
                        tma_load_2d_pair(dst + i * kBBoxRows * 128, &p.xmap, (cur.t.kb0 + cur.kb) * 64, brow0 + i * kBBoxRows, lb);
                } else if (Cfg::kBRows >= 256 && p.xbig && nbox > 1) {
                    // one 256-row box: the same swizzled image as four 64-row boxes,
                    // one TMA issue instead of four (the loader thread is the
                    // pipeline's serial step at one k-block per iteration)
                    mbar_arrive_expect_tx(&sh.bfull[s], 256u * 128u);
                    tma_load_2d(dst, &p.xmap256, (cur.t.kb0 + cur.kb) * 64, brow0, &sh.bfull[s]);
                } else {
                    mbar_arrive_expect_tx(&sh.bfull[s], (uint32_t)(nbox * kBBoxRows * 128));
                    for (int i = 0; i < nbox; ++i)
                        tma_load_2d(dst + i * kBBoxRows * 128, &p.xmap, (cur.t.kb0 + cur.kb) * 64, brow0 + i * kBBoxRows,
                                    &sh.bfull[s]);
                }
                ++it;
                cursor_next(p, sh, cur, nkb);
            }
        }
        __syncwarp();
    } else if (warp == kMmaWarp) {
        // ================= MMA issue (one thread of the leader) =================
        if (leader) {
            int it = 0, lt = 0;
            bool live = true;
            for (int idx = blockIdx.x / CG; live; idx += gridDim.x / CG, ++lt) {
                QTile t;
                if (!decode_tile(p, sh, idx, t)) break;
                const int acc = lt & 1;
                if (!qwait(&sh.tempty[acc], (((uint32_t)lt >> 1) & 1u) ^ 1u, sh, p.err)) {
                    live = false;
                    break;
                }
                tc_fence_after();
                const int N = max(16, (t.cnt + 15) & ~15);
                const uint32_t idesc = make_idesc_f16(kTM * CG, N);
                const uint32_t d = tmem + (uint32_t)(acc * kAccCols);
                for (int kb = 0; kb < nkb; ++kb, ++it) {
                    const int s = it % S, a = it % SA;
                    if (!qwait(&sh.afull[a], (uint32_t)(it / SA) & 1u, sh, p.err)) {
                        live = false;
                        break;
                    }
                    if (lane == 0) QTRACE(5, it);
                    tc_fence_after();
                    if (lane == 0) {
                        const uint64_t ad = make_sw128_desc(As + a * kAStage);
                        const uint64_t bd = make_sw128_desc(Bs + s * Cfg::kBStage);
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            if constexpr (CG == 2)
                                umma_f16_pair(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc,
                                              (kb | k) ? 1u : 0u);
                            else
                                umma_f16(d, ad + (uint64_t)(2 * k), bd + (uint64_t)(2 * k), idesc,
                                         (kb | k) ? 1u : 0u);
                        }
                        if constexpr (CG == 2) {
                            umma_commit_pair(&sh.empty[s], 3);
                            umma_commit_pair(&sh.aempty[a], 3);
                        } else {
                            umma_commit(&sh.empty[s]);
                            umma_commit(&sh.aempty[a]);
                        }
                        QTRACE(7, it);
                    }
                    __syncwarp();
                }
                if (!live) break;
                if (lane == 0) {
                    if constexpr (CG == 2)
                        umma_commit_pair(&sh.tfull[acc], 3);
                    else
                        umma_commit(&sh.tfull[acc]);
                }
                __syncwarp();
            }
            // all issued MMAs retire before TMEM is released
            if (lane == 0) {
                if constexpr (CG == 2)
                    umma_commit_pair(&sh.done, 3);
                else
                    umma_commit(&sh.done);
            }
            __syncwarp();
        }
        uint32_t i = 0;
        for (; i < kQSpin; ++i)
            if (mbar_try_wait(&sh.done, 0)) break;
        if (i == kQSpin && p.err) atomicOr(p.err, kErrMbarTimeout);
    } else {
        // ================= epilogue (warps 0-3) =================
        const int ew = warp;  // TMEM lanes 32*ew .. 32*ew+31
        const int row = ew * 32 + lane;
        const bool gu = gate_up(p.mode);
        int lt = 0;
        for (int idx = blockIdx.x / CG;; idx += gridDim.x / CG, ++lt) {
            QTile t;
            if (!decode_tile(p, sh, idx, t)) break;
            const int acc = lt & 1;
            if (!qwait(&sh.tfull[acc], ((uint32_t)lt >> 1) & 1u, sh, p.err)) break;
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(ew * 32) << 16) + (uint32_t)(acc * kAccCols);
            const int f = cta_feat0<CG>(p, t, rank) + (gu ? (row >> 1) : row);
            const bool fok = f < p.nfeat;
            for (int cc = 0; cc * 32 < t.cnt; ++cc) {
                float v[32];
                tmem_ld32(tbase + (uint32_t)(cc * 32), v);
                const int colbase = cc * 32;
                if (p.part) {
                    // split-K slice: raw fp32 sums, gate/up interleaved by row
                    const long long pc = gu ? 2ll * cta_feat0<CG>(p, t, rank) + row : (long long)f;
                    float* pr = p.part + ((long long)t.split * p.T + t.row0 + colbase) * p.ldp + pc;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (fok && colbase + j < t.cnt) pr[(long long)j * p.ldp] = v[j];
                } else if (gu) {
                    const bool even = (lane & 1) == 0;
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) {
                        const float send = even ? v[16 + jj] : v[jj];
                        const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
                        float g = even ? v[jj] : recv;
                        float u = even ? recv : v[16 + jj];
                        const int col = colbase + (even ? jj : 16 + jj);
                        if (p.round_gu) {
                            g = __half2float(__float2half_rn(g));
                            u = __half2float(__float2half_rn(u));
                        }
                        if (fok && col < t.cnt)
                            p.y[(long long)(t.row0 + col) * p.ldy + f] = __float2half_rn(gelu_tanh(g) * u);
                    }
                } else if (p.mode == kGroupedDown) {
                    long long orow = 0;
                    if (colbase + lane < t.cnt) {
                        const tf_token_expert_pair pr = p.pairs[t.row0 + colbase + lane];
                        orow = (long long)pr.token * p.top_k + pr.rank;
                    }
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const long long o = __shfl_sync(0xffffffffu, orow, j);
                        if (fok && colbase + j < t.cnt) p.y[o * p.ldy + f] = __float2half_rn(v[j]);
                    }
                } else {
                    if (p.y32) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (fok && colbase + j < t.cnt) p.y32[(long long)(t.row0 + colbase + j) * p.ldy + f] = v[j];
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (fok && colbase + j < t.cnt)
                                p.y[(long long)(t.row0 + colbase + j) * p.ldy + f] = __float2half_rn(v[j]);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) arrive_leader<CG>(&sh.tempty[acc]);
        }
    }

    __syncthreads();
    // the pair's MMAs have retired (done barrier) and both epilogues are
    // finished before either CTA frees TMEM or leaves its shared memory
    if constexpr (CG == 2) cluster_sync_all();
    if (warp == kMmaWarp) {
        tc_fence_after();
        if constexpr (CG == 2)
            tmem_dealloc_pair(tmem, kTmemCols);
        else
            tmem_dealloc(tmem, kTmemCols);
    }
}

// Xg[p][:] = X[pairs[p].token][:] (16-byte units): the routed rows in
// sorted-pair order, so each expert's tokens are one contiguous TMA range.
// Only the pairs the group table covers are gathered: with empty routing
// slots (UINT32_MAX ids, skipped by the sort) fewer than P entries are valid.
__global__ void gather_rows_kernel(const __half* __restrict__ x, long long ldx,
                                   const tf_token_expert_pair* __restrict__ pairs, __half* __restrict__ xg, int P,
                                   int D, int T, const tf_moe_group* __restrict__ groups,
                                   const uint32_t* __restrict__ n_groups, uint32_t* err) {
    const int d8 = D >> 3;
    const uint32_t ng = __ldg(n_groups);
    if (ng) {
        const tf_moe_group last = groups[ng - 1];
        P = min(P, (int)(last.pair_start + last.pair_count));
    } else {
        P = 0;
    }
    const long long n = (long long)P * d8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int pr = (int)(i / d8), c = (int)(i - (long long)pr * d8);
        const uint32_t tok = __ldg(&pairs[pr].token);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (tok < (uint32_t)T)
            v = __ldg(reinterpret_cast<const uint4*>(x + (long long)tok * ldx) + c);
        else if (c == 0 && err)
            atomicOr(err, kErrBadExpert);
        reinterpret_cast<uint4*>(xg + (long long)pr * D)[c] = v;
    }
}

// h2[t][d] = half(sum_r fma(w[t][r], partial[t*K + r][d])) in rank order
// (prefill.metal:575-596).  8 outputs per thread, 16-byte loads.
__global__ void reduce_token_major_kernel(const __half* __restrict__ partials, const __half* __restrict__ w,
                                          __half* __restrict__ h2, int T, int K, int D) {
    const int d8 = D >> 3;
    const long long n = (long long)T * d8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / d8), dv = (int)(i % d8);
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int r = 0; r < K; ++r) {
            const float wr = __half2float(w[(long long)t * K + r]);
            const uint4 q = __ldcs(reinterpret_cast<const uint4*>(partials + ((long long)t * K + r) * D) + dv);
            const __half2* hp = reinterpret_cast<const __half2*>(&q);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f2 = __half22float2(hp[j]);
                acc[2 * j] = fmaf(wr, f2.x, acc[2 * j]);
                acc[2 * j + 1] = fmaf(wr, f2.y, acc[2 * j + 1]);
            }
        }
        uint4 o;
        __half2* op = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) op[j] = __floats2half2_rn(acc[2 * j], acc[2 * j + 1]);
        reinterpret_cast<uint4*>(h2 + (long long)t * D)[dv] = o;
    }
}

template <typename ST, int CG, int TN>
tf_status launch_qmm_cg(tf_context* ctx, const QmmParams& p, cudaStream_t stream, const char* name) {
    constexpr int kTN = TN;
    const void* fn = reinterpret_cast<const void*>(&qmm_kernel<ST, CG, TN>);
    const int smem = (int)qsmem_bytes<CG, TN>();
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_check(ctx, e, name);
    // persistent: one CTA (pair) per SM (pair); dense problems never need more
    // than their tile count
    long long units = ctx->num_sms / CG;
    if (p.mode == kDensePlain || p.mode == kDenseGateUp) {
        const int fpt = (p.mode == kDenseGateUp ? kTM / 2 : kTM) * CG;
        units = std::min<long long>(units,
                                    (long long)((p.T + kTN - 1) / kTN) * ((p.nfeat + fpt - 1) / fpt) * p.ksplit);
    }
    if (units <= 0) return TF_OK;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(units * CG));
    cfg.blockDim = dim3(kQThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CG;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CG == 2 ? 1 : 0;
    return cuda_check(ctx, cudaLaunchKernelEx(&cfg, qmm_kernel<ST, CG, TN>, p), name);
}

// One SM per tile by default (measured faster on B200: 590 vs 400 TFLOP/s on
// the 4096 x 2112 x 2816 shape); TFCUDA_QMM_PAIR=1 selects CTA pairs with
// 2-SM MMAs (same arithmetic).  Read per call.
// Token tiles of 64 (deeper rings) when one 256-token tile would leave SMs
// idle (dense) or the caller expects few tokens per expert (grouped,
// p.small_tiles); TFCUDA_QMM_TN=64 / 256 forces one (read per call).
bool use_small_tiles(const tf_context* ctx, const QmmParams& p, bool pair) {
    bool small = p.small_tiles != 0;
    if (p.mode == kDensePlain || p.mode == kDenseGateUp) {
        const int fpt = (p.mode == kDenseGateUp ? kTM / 2 : kTM) * (pair ? 2 : 1);
        // one 64-token tile; above that one 256-token tile, whose few feature
        // tiles then split K over the idle SMs (T = 256 shared expert: 64-token
        // tiles took 4 tiles x 44 k-blocks per CTA, 256-token tiles with a
        // 4-way split 11 k-blocks; the batch-256 step 10.24 -> 9.83 ms)
        small = p.T <= 64 && (long long)((p.nfeat + fpt - 1) / fpt) < ctx->num_sms / (pair ? 2 : 1);
    }
    const char* tn = getenv("TFCUDA_QMM_TN");
    if (tn) small = atoi(tn) == 64;
    return small && !pair;  // 64-token tiles only on one SM (see QCfg)
}

bool use_pair() {
    const char* env = getenv("TFCUDA_QMM_PAIR");
    return env && env[0] == '1';
}

tf_status launch_qmm(tf_context* ctx, const QmmParams& p0, tf_scale_type st, cudaStream_t stream, const char* name) {
    QmmParams p = p0;
    if (p.ksplit < 1) p.ksplit = 1;
    const bool pair = use_pair();
    const bool small = use_small_tiles(ctx, p, pair);
#define TF_QMM_GO(ST_)                                                                                    \
    return pair ? launch_qmm_cg<ST_, 2, 256>(ctx, p, stream, name)                                        \
                : (small ? launch_qmm_cg<ST_, 1, 64>(ctx, p, stream, name)                               \
                         : launch_qmm_cg<ST_, 1, 256>(ctx, p, stream, name));
    if (st == TF_SCALE_BF16) TF_QMM_GO(__nv_bfloat16)
    TF_QMM_GO(__half)
#undef TF_QMM_GO
}

// Split-K for a dense problem whose tiles leave most SMs idle (the shared
// expert and the LM head at a few tokens): K slices of >= 3 k-blocks over
// extra CTAs, fp32 partials in the context scratch, then qmm_split_reduce
// adds the slices in slice order. Returns 1 (no split) otherwise;
// TFCUDA_QMM_SPLIT=0 turns it off (read per call).
int choose_ksplit(const tf_context* ctx, const QmmParams& p) {
    const char* env = getenv("TFCUDA_QMM_SPLIT");
    if (env && env[0] == '0') return 1;
    const bool pair = use_pair();
    if (pair) return 1;
    const int tn = use_small_tiles(ctx, p, pair) ? 64 : kTN;
    const int fpt = p.mode == kDenseGateUp ? kTM / 2 : kTM;
    const long long tiles = (long long)((p.T + tn - 1) / tn) * ((p.nfeat + fpt - 1) / fpt);
    const long long ldp = p.mode == kDenseGateUp ? 2ll * p.nfeat : p.nfeat;
    const int nkb = p.K >> 6;
    int best = 1;
    for (int sp = 2; sp <= 16; ++sp) {
        if (nkb % sp || nkb / sp < 3) continue;
        if (tiles * sp > (long long)ctx->num_sms * 3 / 2) break;
        if ((long long)sp * p.T * ldp > (long long)kQmmPartCap) break;
        best = sp;
    }
    return best;
}

__global__ void __launch_bounds__(256) qmm_split_reduce_kernel(const float* __restrict__ part, int S, int T,
                                                               int nfeat, long long ldp, int gu, int round_gu,
                                                               __half* __restrict__ y, float* __restrict__ y32,
                                                               long long ldy) {
    const long long n = (long long)T * nfeat;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / nfeat), f = (int)(i - (long long)t * nfeat);
        if (gu) {
            float g = 0.f, u = 0.f;
            for (int sp = 0; sp < S; ++sp) {
                const float2 gv = *reinterpret_cast<const float2*>(part + ((long long)sp * T + t) * ldp + 2 * f);
                g += gv.x;
                u += gv.y;
            }
            if (round_gu) {
                g = __half2float(__float2half_rn(g));
                u = __half2float(__float2half_rn(u));
            }
            y[(long long)t * ldy + f] = __float2half_rn(gelu_tanh(g) * u);
        } else {
            float v = 0.f;
            for (int sp = 0; sp < S; ++sp) v += part[((long long)sp * T + t) * ldp + f];
            if (y32)
                y32[(long long)t * ldy + f] = v;
            else
                y[(long long)t * ldy + f] = __float2half_rn(v);
        }
    }
}

// One dense launch, split over K when that fills the GPU better.
tf_status launch_dense(tf_context* ctx, QmmParams p, tf_scale_type st, cudaStream_t stream, const char* name) {
    p.ksplit = choose_ksplit(ctx, p);
    if (p.ksplit == 1) return launch_qmm(ctx, p, st, stream, name);
    p.part = ctx->d_qmm_part;
    p.ldp = p.mode == kDenseGateUp ? 2ll * p.nfeat : p.nfeat;
    tf_status rc = launch_qmm(ctx, p, st, stream, name);
    if (rc != TF_OK) return rc;
    const long long n = (long long)p.T * p.nfeat;
    const int grid = (int)std::min<long long>((n + 255) / 256, (long long)ctx->num_sms * 8);
    qmm_split_reduce_kernel<<<grid, 256, 0, stream>>>(p.part, p.ksplit, p.T, p.nfeat, p.ldp,
                                                      p.mode == kDenseGateUp ? 1 : 0, p.round_gu, p.y, p.y32,
                                                      p.ldy);
    return cuda_check(ctx, cudaGetLastError(), name);
}

bool scale_type_ok(tf_scale_type st) { return st == TF_SCALE_BF16 || st == TF_SCALE_F16; }


// Dense weight matrix [n][k] as a one-deep raw map plus scale/bias addresses.
bool dense_weights(QmmParams& p, CUtensorMap* m, const void* w, uint32_t rows, uint32_t k, const void* sc,
                   const void* bi, int which, bool big_box = false) {
    if (!make_raw_map(m, w, k / 2, rows, 1, 0, big_box ? 128u : 64u)) return false;
    if (big_box) p.wbig = 1;
    if (which == 0) {
        p.os0 = reinterpret_cast<uint64_t>(sc);
        p.ob0 = reinterpret_cast<uint64_t>(bi);
    } else {
        p.os1 = reinterpret_cast<uint64_t>(sc);
        p.ob1 = reinterpret_cast<uint64_t>(bi);
    }
    return true;
}

}  // namespace

namespace {

// Grouped routed experts on the streaming engine (few tokens per expert):
// gate/up (MODE 0) then down (MODE 1), one super-job per (expert, token pass).
template <typename ST>
tf_status grouped_gemv(tf_context* ctx, GroupedParams p, cudaStream_t s, const char* name) {
    auto launch = [&](auto pol_tag) -> tf_status {
        using Pol = decltype(pol_tag);
        const int K = Pol::kdim(p);
        const size_t limit = engine_smem_limit<Pol, ST>(ctx);
        int nt = 8;
        while (nt > 1 && engine_fixed_smem() + Pol::x_bytes(K, nt) + 1024 > limit) --nt;
        if (engine_fixed_smem() + Pol::x_bytes(K, nt) + 1024 > limit)
            return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: hidden size too large for the engine", name);
        GroupedParams q = p;
        q.nt = nt;
        return launch_engine<Pol, ST>(ctx, q, Pol::x_bytes(K, nt), ctx->num_sms, s, name);
    };
    tf_status rc = launch(GroupedPolicy<ST, 0>{});
    if (rc != TF_OK) return rc;
    return launch(GroupedPolicy<ST, 1>{});
}

}  // namespace

extern "C" {

static tf_status qmm_dense(tf_context* ctx, const void* weights, const void* scales, const void* biases,
                           const void* x, void* y, float* y32, uint32_t t, uint32_t n, uint32_t k, uint32_t x_stride,
                           uint32_t y_stride, tf_scale_type st, void* stream, const char* name) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (!scale_type_ok(st)) return fail(ctx, TF_ERR_INVALID_ARG, "%s: bad scale type", name);
    if (k == 0 || k % 64 || n == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: k %% 64 == 0, n > 0", name);
    if (x_stride == 0) x_stride = k;
    if (y_stride == 0) y_stride = n;
    if (x_stride < k || y_stride < n || x_stride % 8)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: x_stride >= k (multiple of 8), y_stride >= n", name);
    if (t == 0) return TF_OK;
    void* out = y32 ? static_cast<void*>(y32) : y;
    if (!weights || !scales || !biases || !x || !out) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(weights) || !aligned16(x) || !(y32 ? aligned4(out) : aligned2(out)) || !aligned2(scales) ||
        !aligned2(biases))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: weights/x 16-byte, y/scales/biases 2-byte aligned", name);
    QmmParams p{};
    p.mode = kDensePlain;
    p.K = (int)k;
    p.nfeat = (int)n;
    p.T = (int)t;
    if (!dense_weights(p, &p.wmap0, weights, n, k, scales, biases, 0, n >= 128) ||
        !make_act_map(&p.xmap, x, k, t, x_stride))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: tensor map rejected", name);
    p.xbig = t >= 256 && make_act_map(&p.xmap256, x, k, t, x_stride, 256) ? 1 : 0;
    p.y = static_cast<__half*>(y);
    p.y32 = y32;
    p.ldy = y_stride;
    p.err = ctx->d_err;
    return launch_dense(ctx, p, st, static_cast<cudaStream_t>(stream), name);
}

tf_status tf_int4_qmm(tf_context* ctx, const void* weights, const void* scales, const void* biases, const void* x,
                      void* y, uint32_t t, uint32_t n, uint32_t k, uint32_t x_stride, uint32_t y_stride,
                      tf_scale_type st, void* stream) {
    return qmm_dense(ctx, weights, scales, biases, x, y, nullptr, t, n, k, x_stride, y_stride, st, stream,
                     "tf_int4_qmm");
}

tf_status tf_prefill_shared_expert(tf_context* ctx, const void* x, uint32_t x_stride, const tf_affine_matrix* gate,
                                   const tf_affine_matrix* up, const tf_affine_matrix* down, void* act_scratch,
                                   void* y, uint32_t y_stride, uint32_t t, tf_scale_type st, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_prefill_shared_expert";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (!gate || !up || !down || !scale_type_ok(st)) return fail(ctx, TF_ERR_INVALID_ARG, "%s: bad argument", name);
    if (gate->bits != 4 || up->bits != 4 || down->bits != 4)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: int4 projections only", name);
    const uint32_t d = gate->cols, f = gate->rows;
    if (up->rows != f || up->cols != d || down->rows != d || down->cols != f)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: projection shapes disagree", name);
    if (d % 64 || f % 64 || d == 0 || f == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d, f multiples of 64", name);
    if (x_stride == 0) x_stride = d;
    if (y_stride == 0) y_stride = d;
    if (x_stride < d || x_stride % 8 || y_stride < d)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: strides", name);
    if (t == 0) return TF_OK;
    if (!x || !y || !act_scratch) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    const tf_affine_matrix* ms[3] = {gate, up, down};
    for (const tf_affine_matrix* m : ms)
        if (!m->weights || !m->scales || !m->biases || !aligned16(m->weights) || !aligned2(m->scales) ||
            !aligned2(m->biases))
            return fail(ctx, TF_ERR_MISALIGNED, "%s: projection pointers", name);
    if (!aligned16(x) || !aligned16(act_scratch) || !aligned2(y))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: x/act_scratch 16-byte aligned", name);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    QmmParams p{};
    p.mode = kDenseGateUp;
    p.K = (int)d;
    p.nfeat = (int)f;
    p.T = (int)t;
    if (!dense_weights(p, &p.wmap0, gate->weights, f, d, gate->scales, gate->biases, 0) ||
        !dense_weights(p, &p.wmap1, up->weights, f, d, up->scales, up->biases, 1) ||
        !make_act_map(&p.xmap, x, d, t, x_stride))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: tensor map rejected", name);
    p.xbig = t >= 256 && make_act_map(&p.xmap256, x, d, t, x_stride, 256) ? 1 : 0;
    p.y = static_cast<__half*>(act_scratch);
    p.ldy = f;
    p.round_gu = 1;
    p.err = ctx->d_err;
    tf_status rc = launch_dense(ctx, p, st, s, name);
    if (rc != TF_OK) return rc;
    QmmParams q{};
    q.mode = kDensePlain;
    q.K = (int)f;
    q.nfeat = (int)d;
    q.T = (int)t;
    if (!dense_weights(q, &q.wmap0, down->weights, d, f, down->scales, down->biases, 0, d >= 128) ||
        !make_act_map(&q.xmap, act_scratch, f, t, f))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: tensor map rejected", name);
    q.xbig = t >= 256 && make_act_map(&q.xmap256, act_scratch, f, t, f, 256) ? 1 : 0;
    q.y = static_cast<__half*>(y);
    q.ldy = y_stride;
    q.err = ctx->d_err;
    return launch_dense(ctx, q, st, s, name);
}

tf_status tf_moe_grouped_routed(tf_context* ctx, const void* pool, uint64_t expert_stride, uint32_t num_experts,
                                const tf_expert_offsets* off, const void* sorted_pairs, const void* groups,
                                const void* n_groups, const void* hidden, uint32_t hidden_stride, void* act_scratch,
                                void* route_partials, uint32_t t, uint32_t d, uint32_t f, uint32_t top_k,
                                tf_scale_type st, void* stream) {
    return tf_moe_grouped_routed_expected(ctx, pool, expert_stride, num_experts, off, sorted_pairs, groups, n_groups,
                                          hidden, hidden_stride, act_scratch, route_partials, t, d, f, top_k, 0, st,
                                          stream);
}

tf_status tf_moe_grouped_routed_expected(tf_context* ctx, const void* pool, uint64_t expert_stride,
                                         uint32_t num_experts, const tf_expert_offsets* off, const void* sorted_pairs,
                                         const void* groups, const void* n_groups, const void* hidden,
                                         uint32_t hidden_stride, void* act_scratch, void* route_partials, uint32_t t,
                                         uint32_t d, uint32_t f, uint32_t top_k, uint32_t expected_pairs,
                                         tf_scale_type st, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_moe_grouped_routed";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (!off || !scale_type_ok(st)) return fail(ctx, TF_ERR_INVALID_ARG, "%s: bad argument", name);
    if (d % 64 || f % 64 || d == 0 || f == 0 || top_k == 0 || num_experts == 0 || num_experts > (uint32_t)kMaxGroups)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d, f multiples of 64; 1 <= num_experts <= 256", name);
    if (hidden_stride == 0) hidden_stride = d;
    if (hidden_stride < d || hidden_stride % 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: hidden stride", name);
    if (t == 0) return TF_OK;
    if (!pool || !sorted_pairs || !groups || !n_groups || !hidden || !act_scratch || !route_partials)
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(pool) || expert_stride % 16 || off->gate_w % 16 || off->up_w % 16 || off->down_w % 16 ||
        off->gate_s % 2 || off->gate_b % 2 || off->up_s % 2 || off->up_b % 2 || off->down_s % 2 || off->down_b % 2)
        return fail(ctx, TF_ERR_MISALIGNED, "%s: weight matrices 16-byte aligned", name);
    if (!aligned16(hidden) || !aligned16(act_scratch) || !aligned16(route_partials) || !aligned4(sorted_pairs) ||
        !aligned4(groups) || !aligned4(n_groups))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: activation pointers", name);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint32_t P = t * top_k;
    // the pairs the groups are expected to hold: all t * top_k unless the
    // caller knows better (expert parallelism: most slots are other ranks')
    const uint32_t P_est = expected_pairs ? std::min(expected_pairs, P) : P;
    const uint8_t* pb = static_cast<const uint8_t*>(pool);
    // Few tokens per expert (batched decode): the streaming engine reads each
    // hit expert's weights once with up to 8 tokens per MMA column block; many
    // (prefill): the tcgen05 GEMMs.  TFCUDA_GROUPED=gemv|gemm forces one.
    const char* env = getenv("TFCUDA_GROUPED");
    bool gemv = (uint64_t)P_est <= 24ull * num_experts;  // measured crossover with the tcgen05 GEMMs
    bool engine = false;
    if (env && env[0] == 'g' && env[1] == 'e' && env[2] == 'm') gemv = env[3] == 'v';
    if (env && env[0] == 'e' && env[1] == 'n') gemv = engine = true;
    if (gemv && !engine) {
        // default for few tokens per expert: the grouped ring-streamed kernel
        const tf_status rc = grouped_stream(
            ctx, pb, expert_stride, num_experts, off, static_cast<const tf_token_expert_pair*>(sorted_pairs),
            static_cast<const tf_moe_group*>(groups), static_cast<const uint32_t*>(n_groups),
            static_cast<const __half*>(hidden), hidden_stride, static_cast<__half*>(act_scratch),
            static_cast<__half*>(route_partials), t, d, f, top_k, st, s, name);
        if (rc != TF_ERR_UNSUPPORTED_SHAPE) return rc;
    }
    if (gemv) {
        GroupedParams g{};
        bool ok = make_weight_map(&g.map[0], pb + off->gate_w, d / 2, f, num_experts, expert_stride) &&
                  make_weight_map(&g.map[1], pb + off->up_w, d / 2, f, num_experts, expert_stride) &&
                  make_weight_map(&g.map[2], pb + off->down_w, f / 2, d, num_experts, expert_stride);
        g.aligned = ok ? 1 : 0;
        g.pool = pb;
        g.stride = expert_stride;
        const uint32_t o9[9] = {off->gate_w, off->gate_s, off->gate_b, off->up_w, off->up_s,
                                off->up_b,   off->down_w, off->down_s, off->down_b};
        for (int i = 0; i < 9; ++i) g.off[i] = o9[i];
        g.E = (int)num_experts;
        g.D = (int)d;
        g.F = (int)f;
        g.top_k = (int)top_k;
        g.groups = static_cast<const tf_moe_group*>(groups);
        g.n_groups = static_cast<const uint32_t*>(n_groups);
        g.pairs = static_cast<const tf_token_expert_pair*>(sorted_pairs);
        g.hidden = static_cast<const __half*>(hidden);
        g.hstride = (int)hidden_stride;
        g.acts = static_cast<__half*>(act_scratch);
        g.partials = static_cast<__half*>(route_partials);
        g.err = ctx->d_err;
        return st == TF_SCALE_BF16 ? grouped_gemv<__nv_bfloat16>(ctx, g, s, name) : grouped_gemv<__half>(ctx, g, s, name);
    }
    QmmParams p{};
    p.mode = kGroupedGateUp;
    p.K = (int)d;
    p.nfeat = (int)f;
    p.sbase = pb;
    p.stride = expert_stride;
    p.os0 = off->gate_s;
    p.ob0 = off->gate_b;
    p.os1 = off->up_s;
    p.ob1 = off->up_b;
    p.num_experts = num_experts;
    p.groups = static_cast<const tf_moe_group*>(groups);
    p.n_groups = static_cast<const uint32_t*>(n_groups);
    p.pairs = static_cast<const tf_token_expert_pair*>(sorted_pairs);
    p.top_k = (int)top_k;
    p.y = static_cast<__half*>(act_scratch);
    p.ldy = f;
    p.err = ctx->d_err;
    // the routed rows in sorted-pair order are staged in the partials buffer
    // (same [T*top_k][d] shape; the down projection overwrites it afterwards)
    if (!make_raw_map(&p.wmap0, pb + off->gate_w, d / 2, f, num_experts, expert_stride) ||
        !make_raw_map(&p.wmap1, pb + off->up_w, d / 2, f, num_experts, expert_stride) ||
        !make_act_map(&p.xmap, route_partials, d, P, d))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: tensor map rejected", name);
    p.xbig = P >= 256 && make_act_map(&p.xmap256, route_partials, d, P, d, 256) ? 1 : 0;
    QmmParams q = p;
    q.mode = kGroupedDown;
    q.K = (int)f;
    q.nfeat = (int)d;
    q.os0 = off->down_s;
    q.ob0 = off->down_b;
    q.y = static_cast<__half*>(route_partials);
    q.ldy = d;
    q.wbig = d >= 128 ? 1 : 0;
    if (!make_raw_map(&q.wmap0, pb + off->down_w, f / 2, d, num_experts, expert_stride, q.wbig ? 128u : 64u) ||
        !make_act_map(&q.xmap, act_scratch, f, P, f))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: tensor map rejected", name);
    q.xbig = P >= 256 && make_act_map(&q.xmap256, act_scratch, f, P, f, 256) ? 1 : 0;
    {
        const long long n = (long long)P * (d / 8);
        const int grid = (int)std::min<long long>((n + 255) / 256, (long long)ctx->num_sms * 8);
        gather_rows_kernel<<<grid, 256, 0, s>>>(static_cast<const __half*>(hidden), hidden_stride,
                                                static_cast<const tf_token_expert_pair*>(sorted_pairs),
                                                static_cast<__half*>(route_partials), (int)P, (int)d, (int)t,
                                                static_cast<const tf_moe_group*>(groups),
                                                static_cast<const uint32_t*>(n_groups), ctx->d_err);
        tf_status rc0 = cuda_check(ctx, cudaGetLastError(), name);
        if (rc0 != TF_OK) return rc0;
    }
    tf_status rc = launch_qmm(ctx, p, st, s, name);
    if (rc != TF_OK) return rc;
    return launch_qmm(ctx, q, st, s, name);
}

tf_status tf_moe_reduce_token_major(tf_context* ctx, const void* route_partials, const void* routing_weights,
                                    void* h2, uint32_t t, uint32_t top_k, uint32_t d, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_moe_reduce_token_major";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0, top_k > 0", name);
    if (t == 0) return TF_OK;
    if (!route_partials || !routing_weights || !h2) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(route_partials) || !aligned16(h2) || !aligned2(routing_weights))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: partials/h2 16-byte aligned", name);
    const long long n = (long long)t * (d / 8);
    const int threads = 256;
    const int grid = (int)std::min<long long>((n + threads - 1) / threads, (long long)ctx->num_sms * 8);
    reduce_token_major_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(route_partials), static_cast<const __half*>(routing_weights),
        static_cast<__half*>(h2), (int)t, (int)top_k, (int)d);
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // extern "C"

namespace tf {

// Dense int4 GEMM with fp32 output Y32[t][j] (row stride y_stride floats):
// the LM head's logits for several tokens at once.
tf_status int4_qmm_f32(tf_context* ctx, const void* weights, const void* scales, const void* biases, const void* x,
                       float* y32, uint32_t t, uint32_t n, uint32_t k, uint32_t x_stride, uint32_t y_stride,
                       tf_scale_type st, cudaStream_t stream, const char* name) {
    return qmm_dense(ctx, weights, scales, biases, x, nullptr, y32, t, n, k, x_stride, y_stride, st, stream, name);
}

}  // namespace tf

#ifdef TF_QMM_TRACE
extern "C" TF_API int tf_debug_qmm_trace(unsigned long long* out) {
    return (int)cudaMemcpyFromSymbol(out, g_qmm_trace, sizeof(g_qmm_trace));
}
#endif
