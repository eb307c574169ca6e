// tf_sampling.cu -- output-head sampling (Sources/TurboFieldfare/Metal/Sampling/logit.metal:42-617;
// LogitSoftcapSoftmax / Sample / SampleTopK64, Kernels/Sampling/LogitOutput.swift):
//   tf_softcap_softmax   p = softmax(softcap * tanh(z / softcap)), fp16 out
//   tf_sample            greedy argmax, Gumbel-max plain temperature, or the
//                        truncating path (top-k <= 256 / top-p, then the seeded
//                        inverse-CDF draw)
//   tf_sample_topk64     the three-stage top-64 sampler
//
// The reference runs each of these in one 256-thread threadgroup; here the
// vocabulary (262144) is spread over the SMs: the softmax takes two passes
// (per-block online (m, d), then every block merges the partials and writes
// its range), the argmax folds blocks with a 64-bit atomicMax of
// (ordered value, ~index), and top-K selection keeps the best K of every
// 1024-entry tile (bitonic sort in shared memory) until one tile is left.
#include "tf_context.cuh"

using namespace tf;

namespace {

constexpr int kSmxBlocks = 128;   // blocks per row of the softmax
constexpr int kTile = 1024;       // candidates sorted per block
constexpr int kMaxVocab = 262144;

__device__ __forceinline__ float softcap_value(float z, float cap) { return cap * tanhf(z / cap); }

template <bool F32>
__device__ __forceinline__ float load_logit(const void* p, long long i) {
    if constexpr (F32)
        return static_cast<const float*>(p)[i];
    else
        return __half2float(static_cast<const __half*>(p)[i]);
}

// online (m, d) merge; an empty side (m == -inf) contributes nothing
__device__ __forceinline__ void md_merge(float& m, float& d, float m2, float d2) {
    if (m2 == -INFINITY) return;
    if (m == -INFINITY) {
        m = m2;
        d = d2;
        return;
    }
    const float mn = fmaxf(m, m2);
    d = d * __expf(m - mn) + d2 * __expf(m2 - mn);
    m = mn;
}

template <bool F32>
__global__ void __launch_bounds__(256) softmax_partial_kernel(const void* __restrict__ logits, int V, float cap,
                                                              float* __restrict__ md) {
    const int r = blockIdx.y, b = blockIdx.x, nb = gridDim.x;
    const int per = (V + nb - 1) / nb;
    const int i0 = b * per, i1 = min(V, i0 + per);
    float m = -INFINITY, d = 0.f;
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float z = softcap_value(load_logit<F32>(logits, (long long)r * V + i), cap);
        md_merge(m, d, z, 1.f);
    }
    for (int o = 16; o; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), d2 = __shfl_xor_sync(0xffffffffu, d, o);
        md_merge(m, d, m2, d2);
    }
    __shared__ float sm[8], sd[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sm[warp] = m;
        sd[warp] = d;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) md_merge(m, d, sm[w], sd[w]);
        md[((size_t)r * nb + b) * 2] = m;
        md[((size_t)r * nb + b) * 2 + 1] = d;
    }
}

template <bool F32>
__global__ void __launch_bounds__(256) softmax_write_kernel(const void* __restrict__ logits, int V, float cap,
                                                            const float* __restrict__ md, __half* __restrict__ probs) {
    const int r = blockIdx.y, b = blockIdx.x, nb = gridDim.x;
    __shared__ float s_m, s_inv;
    if (threadIdx.x < 32) {
        float m = -INFINITY, d = 0.f;
        for (int j = threadIdx.x; j < nb; j += 32) md_merge(m, d, md[((size_t)r * nb + j) * 2], md[((size_t)r * nb + j) * 2 + 1]);
        for (int o = 16; o; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o), d2 = __shfl_xor_sync(0xffffffffu, d, o);
            md_merge(m, d, m2, d2);
        }
        if (threadIdx.x == 0) {
            s_m = m;
            s_inv = 1.f / d;
        }
    }
    __syncthreads();
    const float m = s_m, inv = s_inv;
    const int per = (V + nb - 1) / nb;
    const int i0 = b * per, i1 = min(V, i0 + per);
    for (int i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
        const float z = softcap_value(load_logit<F32>(logits, (long long)r * V + i), cap);
        probs[(long long)r * V + i] = __float2half_rn(__expf(z - m) * inv);
    }
}

// ---- argmax (greedy, Gumbel-max) ------------------------------------------
__device__ __forceinline__ unsigned long long key_of(float v, uint32_t row) {
    uint32_t b = __float_as_uint(v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - row);
}

// lmhead_gumbel_for (logit.metal:164-181): a counter-based draw per (seed, position, row)
__device__ __forceinline__ float gumbel_for(unsigned long long seed, uint32_t position, uint32_t row) {
    unsigned long long x = seed ^ ((unsigned long long)position * 0xD2B74407B1CE6E93ull) ^ (unsigned long long)row;
    x = x + 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    x = x ^ (x >> 31);
    const uint32_t bits = (uint32_t)(x >> 40);
    const float u = ((float)bits + 0.5f) * (1.0f / 16777216.0f);
    return -logf(-logf(u));
}

// MODE 0: argmax p (temperature 0); MODE 1: argmax inv_t*log p + gumbel (p > 0 only).
// The last block (ticket) writes the token (0 when nothing qualified) and
// leaves the key and ticket at zero.
template <int MODE>
__global__ void __launch_bounds__(256) sample_argmax_kernel(const __half* __restrict__ probs, int V, float inv_t,
                                                            unsigned long long seed, uint32_t position,
                                                            unsigned long long* key, unsigned int* ticket,
                                                            uint32_t* out) {
    unsigned long long best = 0ull;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
        const float p = __half2float(probs[i]);
        float s;
        if (MODE == 0) {
            s = p;
        } else {
            if (!(p > 0.f)) continue;
            s = inv_t * logf(p) + gumbel_for(seed, position, (uint32_t)i);
        }
        const unsigned long long k = key_of(s, (uint32_t)i);
        best = k > best ? k : best;
    }
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    __shared__ unsigned long long wb[8];
    __shared__ bool last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) wb[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) b = wb[w] > b ? wb[w] : b;
        if (b) atomicMax(key, b);
        __threadfence();
        last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        const unsigned long long k = atomicExch(key, 0ull);
        out[0] = k ? 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull) : 0u;
        *ticket = 0u;
    }
}

// ---- top-K candidates ------------------------------------------------------
// (value desc, index asc): the order of repeated argmax extraction
__device__ __forceinline__ bool better(float va, uint32_t ia, float vb, uint32_t ib) {
    return va > vb || (va == vb && ia < ib);
}

__device__ void sort_tile(float* v, uint32_t* ix) {
    for (int width = 2; width <= kTile; width <<= 1) {
        for (int stride = width >> 1; stride > 0; stride >>= 1) {
            __syncthreads();
            for (int i = threadIdx.x; i < kTile; i += blockDim.x) {
                const int partner = i ^ stride;
                if (partner <= i) continue;
                const float lv = v[i], rv = v[partner];
                const uint32_t li = ix[i], ri = ix[partner];
                const bool desc = (i & width) == 0;
                const bool swap = desc ? better(rv, ri, lv, li) : better(lv, li, rv, ri);
                if (swap) {
                    v[i] = rv;
                    ix[i] = ri;
                    v[partner] = lv;
                    ix[partner] = li;
                }
            }
        }
    }
    __syncthreads();
}

// One 1024-entry tile per block -> its best `keep` candidates.  FROM_PROBS:
// the tile comes from the fp16 probabilities (indices = positions).
template <bool FROM_PROBS>
__global__ void __launch_bounds__(256) topk_tile_kernel(const __half* __restrict__ probs, const float* __restrict__ in_v,
                                                        const uint32_t* __restrict__ in_i, int count, int keep,
                                                        float* __restrict__ out_v, uint32_t* __restrict__ out_i) {
    __shared__ float v[kTile];
    __shared__ uint32_t ix[kTile];
    const int base = blockIdx.x * kTile;
    for (int i = threadIdx.x; i < kTile; i += blockDim.x) {
        const int s = base + i;
        const bool ok = s < count;
        if (FROM_PROBS) {
            v[i] = ok ? __half2float(probs[s]) : -INFINITY;
            ix[i] = ok ? (uint32_t)s : 0xFFFFFFFFu;
        } else {
            v[i] = ok ? in_v[s] : -INFINITY;
            ix[i] = ok ? in_i[s] : 0xFFFFFFFFu;
        }
    }
    sort_tile(v, ix);
    for (int i = threadIdx.x; i < keep; i += blockDim.x) {
        out_v[(size_t)blockIdx.x * keep + i] = v[i];
        out_i[(size_t)blockIdx.x * keep + i] = ix[i];
    }
}

__device__ __forceinline__ uint64_t xorshift64(uint64_t& s) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s * 2685821657736338717ULL;
}

// The last tile (<= 1024 candidates) sorted, then the reference's truncating
// draw on its first k: finite entries only, top-p against the full-vocabulary
// mass, p^(1/T), one xorshift step, inverse-CDF walk (default: the argmax).
__global__ void __launch_bounds__(256) topk_final_kernel(const __half* __restrict__ probs, const float* __restrict__ in_v,
                                                         const uint32_t* __restrict__ in_i, int count, int from_probs,
                                                         int k, int V, float temperature, float top_p,
                                                         unsigned long long seed, uint32_t* out) {
    __shared__ float v[kTile];
    __shared__ uint32_t ix[kTile];
    for (int i = threadIdx.x; i < kTile; i += blockDim.x) {
        const bool ok = i < count;
        if (from_probs) {
            v[i] = ok ? __half2float(probs[i]) : -INFINITY;
            ix[i] = ok ? (uint32_t)i : 0xFFFFFFFFu;
        } else {
            v[i] = ok ? in_v[i] : -INFINITY;
            ix[i] = ok ? in_i[i] : 0xFFFFFFFFu;
        }
    }
    sort_tile(v, ix);
    if (threadIdx.x != 0) return;
    int kept = 0;
    while (kept < k && ix[kept] < (uint32_t)V && isfinite(v[kept])) ++kept;
    if (top_p > 0.f && top_p < 1.f) {
        float cum = 0.f;
        int cut = kept;
        for (int i = 0; i < kept; ++i) {
            cum += v[i];
            if (cum >= top_p) {
                cut = i + 1;
                break;
            }
        }
        kept = cut;
    }
    const float inv_t = 1.f / temperature;
    if (temperature != 1.f)
        for (int i = 0; i < kept; ++i) v[i] = powf(v[i], inv_t);
    float surviving = 0.f;
    for (int i = 0; i < kept; ++i) surviving += v[i];
    uint64_t rng = seed;
    (void)xorshift64(rng);
    const float u = (float)(uint32_t)(xorshift64(rng) >> 40) * (1.0f / 16777216.0f) * surviving;
    float run = 0.f;
    uint32_t picked = ix[0];
    for (int i = 0; i < kept; ++i) {
        run += v[i];
        if (u <= run) {
            picked = ix[i];
            break;
        }
    }
    out[0] = picked;
}

tf_status check(tf_context* ctx, const char* name) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "%s: cudaSetDevice failed", name);
    return TF_OK;
}

// top-`keep` candidates of the row, then the final draw on the first k
tf_status topk_draw(tf_context* ctx, const __half* probs, int V, int keep, int k, float temperature, float top_p,
                    unsigned long long seed, uint32_t* out, cudaStream_t s, const char* name) {
    if (V <= kTile) {
        topk_final_kernel<<<1, 256, 0, s>>>(probs, nullptr, nullptr, V, 1, k, V, temperature, top_p, seed, out);
        return cuda_check(ctx, cudaGetLastError(), name);
    }
    float* bv[2] = {ctx->d_cand_v, ctx->d_cand_v + kCandCap};
    uint32_t* bi[2] = {ctx->d_cand_i, ctx->d_cand_i + kCandCap};
    int tiles = (V + kTile - 1) / kTile;
    topk_tile_kernel<true><<<tiles, 256, 0, s>>>(probs, nullptr, nullptr, V, keep, bv[0], bi[0]);
    int count = tiles * keep, cur = 0;
    while (count > kTile) {
        tiles = (count + kTile - 1) / kTile;
        topk_tile_kernel<false><<<tiles, 256, 0, s>>>(nullptr, bv[cur], bi[cur], count, keep, bv[cur ^ 1], bi[cur ^ 1]);
        count = tiles * keep;
        cur ^= 1;
    }
    topk_final_kernel<<<1, 256, 0, s>>>(nullptr, bv[cur], bi[cur], count, 0, k, V, temperature, top_p, seed, out);
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // namespace

extern "C" {

tf_status tf_softcap_softmax(tf_context* ctx, const void* logits, int logits_fp32, void* probs, uint32_t V,
                             uint32_t rows, float softcap, void* stream) {
    const char* name = "tf_softcap_softmax";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (V == 0 || rows > (uint32_t)kMaxLmTokens || !(softcap > 0.f))
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: V > 0, rows <= %d, softcap > 0", name, kMaxLmTokens);
    if (rows == 0) return TF_OK;
    if (!logits || !probs) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    const int nb = (int)std::min<uint32_t>((uint32_t)kSmxBlocks, (V + 1023) / 1024);
    const dim3 grid(nb, rows);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (logits_fp32) {
        softmax_partial_kernel<true><<<grid, 256, 0, cs>>>(logits, (int)V, softcap, ctx->d_smx);
        softmax_write_kernel<true><<<grid, 256, 0, cs>>>(logits, (int)V, softcap, ctx->d_smx, static_cast<__half*>(probs));
    } else {
        softmax_partial_kernel<false><<<grid, 256, 0, cs>>>(logits, (int)V, softcap, ctx->d_smx);
        softmax_write_kernel<false><<<grid, 256, 0, cs>>>(logits, (int)V, softcap, ctx->d_smx, static_cast<__half*>(probs));
    }
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_sample(tf_context* ctx, const void* probs, uint32_t V, float temperature, uint32_t top_k, float top_p,
                    uint64_t seed, uint32_t position, void* out_token, void* stream) {
    const char* name = "tf_sample";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (V == 0 || V > (uint32_t)kMaxVocab) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: 0 < V <= %d", name, kMaxVocab);
    if (!probs || !out_token) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    const __half* p = static_cast<const __half*>(probs);
    uint32_t* out = static_cast<uint32_t*>(out_token);
    const int blocks = std::max(1, std::min((int)((V + 255) / 256), 2 * ctx->num_sms));
    if (temperature <= 0.f) {
        sample_argmax_kernel<0><<<blocks, 256, 0, cs>>>(p, (int)V, 0.f, seed, position, ctx->d_lm_keys,
                                                        ctx->d_lm_tickets, out);
        return cuda_check(ctx, cudaGetLastError(), name);
    }
    if (top_k == 0 && (top_p <= 0.f || top_p >= 1.f)) {
        sample_argmax_kernel<1><<<blocks, 256, 0, cs>>>(p, (int)V, 1.f / temperature, seed, position, ctx->d_lm_keys,
                                                        ctx->d_lm_tickets, out);
        return cuda_check(ctx, cudaGetLastError(), name);
    }
    int k = top_k == 0 ? (int)V : (int)top_k;
    k = std::min(k, 256);
    k = std::min(k, (int)V);
    return topk_draw(ctx, p, (int)V, k <= 64 ? 64 : 256, k, temperature, top_p, seed, out, cs, name);
}

tf_status tf_sample_topk64(tf_context* ctx, const void* probs, uint32_t V, float temperature, float top_p,
                           uint64_t seed, void* out_token, void* stream) {
    const char* name = "tf_sample_topk64";
    tf_status s = check(ctx, name);
    if (s) return s;
    if (V == 0 || V > (uint32_t)kMaxVocab) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: 0 < V <= %d", name, kMaxVocab);
    if (!probs || !out_token) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    return topk_draw(ctx, static_cast<const __half*>(probs), (int)V, 64, std::min(64, (int)V), temperature, top_p, seed,
                     static_cast<uint32_t*>(out_token), static_cast<cudaStream_t>(stream), name);
}

}  // extern "C"
