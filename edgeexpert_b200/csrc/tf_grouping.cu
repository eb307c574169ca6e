// tf_grouping.cu -- token -> expert grouping (PrefillMoEGrouping.groupTokenExpertPairs,
// Sources/TurboFieldfare/Kernels/Prefill/MoE/PrefillMoEGrouping.swift:91-192).
//
// Two implementations with the same output contract:
//   tf_group_token_expert_pairs  host restatement (arbitrary pair order, full
//                                validation with the reference's error cases);
//   tf_moe_route_sort            device kernel for the on-GPU pipeline: takes
//                                the router's token-major [T][K] ids/weights,
//                                never leaves the GPU.
// Order: pairs sorted by (expert sort key if given, expert, token, rank);
// per-expert offsets (UINT32_MAX when empty) and counts; groups = non-empty
// experts in sorted order; tiles = runs of <= tile_expert_count groups.
#include <algorithm>
#include <unordered_set>
#include <vector>

#include "tf_context.cuh"

using namespace tf;

namespace {

constexpr int kSortThreads = 1024;
constexpr int kSortMaxExperts = 256;

// Pass 1, one CTA per chunk of the token-major pair list (pair p = token*K + rank):
// per-chunk expert histogram -> cnt[chunk][expert].
__global__ void __launch_bounds__(kSortThreads) route_count_kernel(const uint32_t* __restrict__ ids, int n,
                                                                   int chunk, int E, uint32_t* cnt, uint32_t* err) {
    __shared__ uint32_t c[kSortMaxExperts];
    for (int e = threadIdx.x; e < E; e += blockDim.x) c[e] = 0;
    __syncthreads();
    const int p0 = blockIdx.x * chunk, p1 = min(n, p0 + chunk);
    for (int p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
        const uint32_t e = ids[p];
        if (e < (uint32_t)E)
            atomicAdd(&c[e], 1u);
        else if (e != 0xFFFFFFFFu)  // UINT32_MAX marks an empty slot: skipped silently
            atomicOr(err, kErrBadExpert);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) cnt[blockIdx.x * kSortMaxExperts + e] = c[e];
}

// Pass 2, one CTA: expert order (by sort key, then id), per-expert offsets and
// counts, groups, tiles, and each chunk's first destination per expert
// (cnt[chunk][e] is replaced by that base).
__global__ void __launch_bounds__(kSortMaxExperts) route_plan_kernel(
    uint32_t* cnt, int nb, int E, int tile_e, const unsigned long long* __restrict__ sort_keys, uint32_t* offsets,
    uint32_t* counts, tf_moe_group* groups, uint32_t* n_groups, tf_moe_tile* tiles, uint32_t* n_tiles) {
    __shared__ uint32_t tot[kSortMaxExperts];
    __shared__ uint32_t order[kSortMaxExperts];
    __shared__ uint32_t start[kSortMaxExperts];
    __shared__ uint32_t gidx[kSortMaxExperts];
    const int e = threadIdx.x;
    if (e < E) {
        uint32_t t = 0;
        for (int b = 0; b < nb; ++b) t += cnt[b * kSortMaxExperts + e];
        tot[e] = t;
        int pos = e;
        if (sort_keys) {
            const unsigned long long k = sort_keys[e];
            pos = 0;
            for (int j = 0; j < E; ++j) {
                const unsigned long long kj = sort_keys[j];
                pos += (kj < k || (kj == k && j < e)) ? 1 : 0;
            }
        }
        order[pos] = (uint32_t)e;
    }
    __syncthreads();
    // position i (thread i) in sort order: exclusive scans of the counts and of
    // the non-empty flags give each expert's first pair and its group index
    // (block scan: warp inclusive scans, then the earlier warps' totals)
    __shared__ uint32_t wsum[kSortMaxExperts / 32], wnz[kSortMaxExperts / 32];
    __shared__ uint32_t s_ng;
    const int lane = e & 31, wid = e >> 5;
    const uint32_t x = e < E ? order[e] : 0u;
    const uint32_t tx = e < E ? tot[x] : 0u, nz = tx ? 1u : 0u;
    uint32_t ia = tx, in = nz;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t va = __shfl_up_sync(0xffffffffu, ia, o), vn = __shfl_up_sync(0xffffffffu, in, o);
        if (lane >= o) {
            ia += va;
            in += vn;
        }
    }
    if (lane == 31) {
        wsum[wid] = ia;
        wnz[wid] = in;
    }
    __syncthreads();
    uint32_t pa = 0, pn = 0;
    for (int w = 0; w < wid; ++w) {
        pa += wsum[w];
        pn += wnz[w];
    }
    const uint32_t acc = pa + ia - tx, g = pn + in - nz;  // exclusive
    if (e < E) {
        start[x] = acc;
        offsets[x] = tx ? acc : 0xFFFFFFFFu;
        counts[x] = tx;
        if (tx) {
            groups[g] = tf_moe_group{x, acc, tx};
            gidx[g] = x;
        }
    }
    if (e == (E > 0 ? E - 1 : 0)) s_ng = E > 0 ? g + nz : 0u;
    __syncthreads();
    const uint32_t ng = s_ng;
    const uint32_t nt = (ng + (uint32_t)tile_e - 1) / (uint32_t)tile_e;
    for (uint32_t j = (uint32_t)e; j < nt; j += blockDim.x) {
        const uint32_t g0 = j * (uint32_t)tile_e, g1 = min(ng, g0 + (uint32_t)tile_e);
        const uint32_t ps = start[gidx[g0]];
        const uint32_t pe = start[gidx[g1 - 1]] + tot[gidx[g1 - 1]];
        tiles[j] = tf_moe_tile{g0, g1 - g0, ps, pe - ps};
    }
    if (e == 0) {
        *n_groups = ng;
        *n_tiles = nt;
    }
    __syncthreads();
    if (e < E) {
        uint32_t run = start[e];
        for (int b = 0; b < nb; ++b) {
            const uint32_t v = cnt[b * kSortMaxExperts + e];
            cnt[b * kSortMaxExperts + e] = run;
            run += v;
        }
    }
}

// Pass 3, one CTA per chunk: stable scatter.  Within a 1024-pair round the
// rank of a pair among equal experts is (earlier warps' count + lanes below
// it in its own warp), so the (expert, token, rank) order of the reference
// is reproduced exactly.
__global__ void __launch_bounds__(kSortThreads) route_scatter_kernel(
    const uint32_t* __restrict__ ids, const __half* __restrict__ w, int n, int K, int chunk, int E,
    const uint32_t* __restrict__ base, tf_token_expert_pair* sorted) {
    __shared__ uint32_t run[kSortMaxExperts];
    __shared__ uint32_t wcnt[kSortThreads / 32][kSortMaxExperts];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < E; e += blockDim.x) run[e] = base[blockIdx.x * kSortMaxExperts + e];
    __syncthreads();
    const int p0 = blockIdx.x * chunk, p1 = min(n, p0 + chunk);
    for (int r0 = p0; r0 < p1; r0 += blockDim.x) {
        const int p = r0 + tid;
        const bool valid = p < p1;
        const uint32_t e = valid ? ids[p] : 0xFFFFFFFFu;
        const bool ok = valid && e < (uint32_t)E;
        const unsigned int same = __match_any_sync(0xffffffffu, ok ? e : 0xFFFFFFFFu);
        const uint32_t intra = __popc(same & ((1u << lane) - 1u));
        for (int i = lane; i < E; i += 32) wcnt[warp][i] = 0;
        __syncwarp();
        if (ok && intra == 0) wcnt[warp][e] = __popc(same);
        __syncthreads();
        if (ok) {
            uint32_t before = 0;
            for (int w2 = 0; w2 < warp; ++w2) before += wcnt[w2][e];
            tf_token_expert_pair pr;
            pr.token = (uint32_t)(p / K);
            pr.expert = e;
            pr.rank = (uint32_t)(p % K);
            pr.weight_bits = (uint32_t)__half_as_ushort(w[p]);
            sorted[run[e] + before + intra] = pr;
        }
        __syncthreads();
        for (int i = tid; i < E; i += blockDim.x) {
            uint32_t s = 0;
            for (int w2 = 0; w2 < kSortThreads / 32; ++w2) s += wcnt[w2][i];
            run[i] += s;
        }
        __syncthreads();
    }
}

}  // namespace

extern "C" {

tf_status tf_group_token_expert_pairs(const tf_token_expert_pair* pairs, uint32_t n_pairs, int32_t T, int32_t K,
                                      int32_t E, int32_t tile_e, const uint64_t* sort_keys, uint32_t n_keys,
                                      tf_token_expert_pair* sorted, uint32_t* offsets, uint32_t* counts,
                                      tf_moe_group* groups, uint32_t* n_groups, tf_moe_tile* tiles, uint32_t* n_tiles,
                                      tf_grouping_error* error) {
    tf_grouping_error local;
    tf_grouping_error* er = error ? error : &local;
    *er = tf_grouping_error{TF_GROUPING_OK, 0, 0};
    auto reject = [&](tf_grouping_code c, uint32_t a = 0, uint32_t b = 0) {
        *er = tf_grouping_error{c, a, b};
        return TF_ERR_GROUPING;
    };
    if (T < 0) return reject(TF_GROUPING_INVALID_QUERY_COUNT, (uint32_t)T);
    if (K <= 0) return reject(TF_GROUPING_INVALID_TOP_K, (uint32_t)K);
    if (E <= 0) return reject(TF_GROUPING_INVALID_NUM_EXPERTS, (uint32_t)E);
    if (tile_e < 1 || tile_e > 16) return reject(TF_GROUPING_INVALID_TILE_EXPERT_COUNT, (uint32_t)tile_e);
    if (sort_keys && n_keys != (uint32_t)E) return reject(TF_GROUPING_SORT_KEY_COUNT_MISMATCH, (uint32_t)E, n_keys);
    if ((uint64_t)n_pairs != (uint64_t)T * (uint64_t)K)
        return reject(TF_GROUPING_PAIR_COUNT_MISMATCH, (uint32_t)(T * K), n_pairs);
    if (n_pairs && (!pairs || !sorted)) return TF_ERR_INVALID_ARG;
    if (!offsets || !counts || !groups || !n_groups || !tiles || !n_tiles) return TF_ERR_INVALID_ARG;
    std::unordered_set<uint64_t> seen;
    seen.reserve(n_pairs * 2 + 1);
    for (uint32_t i = 0; i < n_pairs; ++i) {
        const tf_token_expert_pair& p = pairs[i];
        if (p.token >= (uint32_t)T) return reject(TF_GROUPING_TOKEN_OUT_OF_RANGE, p.token);
        if (p.rank >= (uint32_t)K) return reject(TF_GROUPING_RANK_OUT_OF_RANGE, p.rank);
        if (p.expert >= (uint32_t)E) return reject(TF_GROUPING_EXPERT_OUT_OF_RANGE, p.expert);
        if (!seen.insert(((uint64_t)p.token << 32) | p.rank).second)
            return reject(TF_GROUPING_DUPLICATE_TOKEN_RANK, p.token, p.rank);
    }
    std::vector<tf_token_expert_pair> v(pairs, pairs + n_pairs);
    std::sort(v.begin(), v.end(), [&](const tf_token_expert_pair& a, const tf_token_expert_pair& b) {
        if (sort_keys) {
            const uint64_t ka = sort_keys[a.expert], kb = sort_keys[b.expert];
            if (ka != kb) return ka < kb;
        }
        if (a.expert != b.expert) return a.expert < b.expert;
        if (a.token != b.token) return a.token < b.token;
        return a.rank < b.rank;
    });
    std::copy(v.begin(), v.end(), sorted);
    for (int e = 0; e < E; ++e) {
        offsets[e] = 0xFFFFFFFFu;
        counts[e] = 0;
    }
    uint32_t ng = 0;
    for (uint32_t i = 0; i < n_pairs;) {
        const uint32_t ex = v[i].expert, s = i;
        while (i < n_pairs && v[i].expert == ex) ++i;
        offsets[ex] = s;
        counts[ex] = i - s;
        groups[ng++] = tf_moe_group{ex, s, i - s};
    }
    uint32_t nt = 0;
    for (uint32_t g0 = 0; g0 < ng; g0 += (uint32_t)tile_e) {
        const uint32_t g1 = std::min(ng, g0 + (uint32_t)tile_e);
        const uint32_t ps = groups[g0].pair_start;
        tiles[nt++] = tf_moe_tile{g0, g1 - g0, ps, groups[g1 - 1].pair_start + groups[g1 - 1].pair_count - ps};
    }
    *n_groups = ng;
    *n_tiles = nt;
    return TF_OK;
}

tf_status tf_moe_route_sort(tf_context* ctx, const void* expert_ids, const void* weights, uint32_t T, uint32_t K,
                            uint32_t E, uint32_t tile_expert_count, const void* sort_keys, void* sorted_pairs,
                            void* offsets, void* counts, void* groups, void* n_groups, void* tiles, void* n_tiles,
                            void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    const char* name = "tf_moe_route_sort";
    if (E == 0 || E > (uint32_t)kSortMaxExperts) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: num_experts must be in 1..256", name);
    if (K == 0 || tile_expert_count < 1 || tile_expert_count > 16)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: top_k >= 1 and tile_expert_count in 1..16", name);
    if ((uint64_t)T * K > (1u << 24)) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: too many pairs", name);
    if ((T && (!expert_ids || !weights || !sorted_pairs)) || !offsets || !counts || !groups || !n_groups || !tiles ||
        !n_tiles)
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    const int n = (int)(T * K);
    int nb = 0, chunk = kSortThreads;
    if (n > 0) {
        nb = std::min(kRouteSortChunks, (n + kSortThreads - 1) / kSortThreads);
        chunk = ((n + nb - 1) / nb + kSortThreads - 1) / kSortThreads * kSortThreads;
        nb = (n + chunk - 1) / chunk;
        route_count_kernel<<<nb, kSortThreads, 0, cs>>>(static_cast<const uint32_t*>(expert_ids), n, chunk, (int)E,
                                                         ctx->d_sort_cnt, ctx->d_err);
    }
    route_plan_kernel<<<1, kSortMaxExperts, 0, cs>>>(
        ctx->d_sort_cnt, nb, (int)E, (int)tile_expert_count, static_cast<const unsigned long long*>(sort_keys),
        static_cast<uint32_t*>(offsets), static_cast<uint32_t*>(counts), static_cast<tf_moe_group*>(groups),
        static_cast<uint32_t*>(n_groups), static_cast<tf_moe_tile*>(tiles), static_cast<uint32_t*>(n_tiles));
    if (n > 0)
        route_scatter_kernel<<<nb, kSortThreads, 0, cs>>>(
            static_cast<const uint32_t*>(expert_ids), static_cast<const __half*>(weights), n, (int)K, chunk, (int)E,
            ctx->d_sort_cnt, static_cast<tf_token_expert_pair*>(sorted_pairs));
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // extern "C"
