// tf_ep.cu -- device pieces of the expert-parallel MoE step (routed experts
// sharded across GPUs in contiguous id ranges, experts_per_rank each).
//
// The reference has no multi-GPU path; this is the B200 replacement for its
// SSD expert streaming when experts are spread over several GPUs.  A step on
// each rank is:
//   route + tf_moe_route_sort over its own tokens  (pairs sorted by expert,
//       hence by destination rank)
//   tf_ep_send_counts     pairs per destination rank
//   tf_ep_pack            the pairs' token rows in sorted order + the local
//                         expert id at the destination (the send buffer)
//   all-to-all (NCCL)     rows and ids to the expert owners
//   tf_moe_route_sort (K = 1) + tf_moe_grouped_routed (top_k = 1) on the
//                         received rows: one output row per received row
//   all-to-all (NCCL)     output rows back, in the sender's sorted order
//   tf_moe_combine_sorted h2[t] = half(sum_r fma(w[t][r], part[pair(t, r)])),
//                         the token-major reduce of prefill.metal:575-596 in
//                         the same rank order, reading the partials through
//                         the sorted-pair permutation
#include "tf_context.cuh"

using namespace tf;

namespace {

__global__ void send_counts_kernel(const uint32_t* __restrict__ counts, int E, int per_rank, int P,
                                   uint32_t* out) {
    const int r = threadIdx.x;
    if (r >= P) return;
    uint32_t s = 0;
    for (int e = r * per_rank; e < min(E, (r + 1) * per_rank); ++e) s += counts[e];
    out[r] = s;
}

// rows[p][:] = hidden[pairs[p].token][:], local[p] = pairs[p].expert % per_rank
__global__ void ep_pack_kernel(const __half* __restrict__ x, long long ldx,
                               const tf_token_expert_pair* __restrict__ pairs, int n, int d, int T, int per_rank,
                               __half* __restrict__ rows, uint32_t* __restrict__ local, uint32_t* err) {
    const int d8 = d >> 3;
    const long long total = (long long)n * d8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(i / d8), c = (int)(i - (long long)p * d8);
        const tf_token_expert_pair pr = pairs[p];
        uint4 v = make_uint4(0, 0, 0, 0);
        if (pr.token < (uint32_t)T)
            v = __ldg(reinterpret_cast<const uint4*>(x + (long long)pr.token * ldx) + c);
        else if (c == 0 && err)
            atomicOr(err, kErrBadExpert);
        reinterpret_cast<uint4*>(rows + (long long)p * d)[c] = v;
        if (c == 0) local[p] = pr.expert % (uint32_t)per_rank;
    }
}

// inv[token * K + rank] = sorted position of that pair
__global__ void invert_pairs_kernel(const tf_token_expert_pair* __restrict__ pairs, int n, int K, int T,
                                    uint32_t* inv, uint32_t* err) {
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n; p += gridDim.x * blockDim.x) {
        const tf_token_expert_pair pr = pairs[p];
        if (pr.token < (uint32_t)T && pr.rank < (uint32_t)K)
            inv[pr.token * K + pr.rank] = (uint32_t)p;
        else if (err)
            atomicOr(err, kErrBadExpert);
    }
}

__global__ void combine_sorted_kernel(const __half* __restrict__ part, const uint32_t* __restrict__ inv,
                                      const __half* __restrict__ w, __half* __restrict__ h2, int T, int K, int D) {
    const int d8 = D >> 3;
    const long long n = (long long)T * d8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / d8), dv = (int)(i - (long long)t * d8);
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int r = 0; r < K; ++r) {
            const float wr = __half2float(w[(long long)t * K + r]);
            const uint32_t p = __ldg(&inv[(long long)t * K + r]);
            const uint4 q = __ldcs(reinterpret_cast<const uint4*>(part + (long long)p * D) + dv);
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

int grid_for(const tf_context* ctx, long long n) {
    return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)ctx->num_sms * 8));
}

}  // namespace

extern "C" {

tf_status tf_ep_send_counts(tf_context* ctx, const void* counts, uint32_t num_experts, uint32_t experts_per_rank,
                            uint32_t world, void* send_counts, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_send_counts";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (!counts || !send_counts) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (world == 0 || world > 1024 || experts_per_rank == 0 || experts_per_rank * world != num_experts)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: num_experts must equal experts_per_rank * world", name);
    send_counts_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint32_t*>(counts), (int)num_experts, (int)experts_per_rank, (int)world,
        static_cast<uint32_t*>(send_counts));
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_ep_pack(tf_context* ctx, const void* hidden, uint32_t hidden_stride, const void* sorted_pairs,
                     uint32_t n_pairs, uint32_t d, uint32_t T, uint32_t experts_per_rank, void* rows,
                     void* local_expert, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_pack";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || experts_per_rank == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0", name);
    if (hidden_stride == 0) hidden_stride = d;
    if (hidden_stride < d || hidden_stride % 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: hidden stride", name);
    if (n_pairs == 0) return TF_OK;
    if (!hidden || !sorted_pairs || !rows || !local_expert) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(hidden) || !aligned16(rows) || !aligned4(sorted_pairs) || !aligned4(local_expert))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: hidden/rows 16-byte aligned", name);
    const long long n = (long long)n_pairs * (d / 8);
    ep_pack_kernel<<<grid_for(ctx, n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(hidden), hidden_stride, static_cast<const tf_token_expert_pair*>(sorted_pairs),
        (int)n_pairs, (int)d, (int)T, (int)experts_per_rank, static_cast<__half*>(rows),
        static_cast<uint32_t*>(local_expert), ctx->d_err);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_moe_combine_sorted(tf_context* ctx, const void* sorted_pairs, const void* partials_sorted,
                                const void* routing_weights, void* inv_scratch, void* h2, uint32_t T,
                                uint32_t top_k, uint32_t d, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_moe_combine_sorted";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0, top_k > 0", name);
    if (T == 0) return TF_OK;
    if (!sorted_pairs || !partials_sorted || !routing_weights || !inv_scratch || !h2)
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(partials_sorted) || !aligned16(h2) || !aligned2(routing_weights) || !aligned4(inv_scratch) ||
        !aligned4(sorted_pairs))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: partials/h2 16-byte aligned", name);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int n = (int)(T * top_k);
    invert_pairs_kernel<<<grid_for(ctx, n), 256, 0, s>>>(static_cast<const tf_token_expert_pair*>(sorted_pairs), n,
                                                         (int)top_k, (int)T, static_cast<uint32_t*>(inv_scratch),
                                                         ctx->d_err);
    tf_status rc = cuda_check(ctx, cudaGetLastError(), name);
    if (rc != TF_OK) return rc;
    const long long m = (long long)T * (d / 8);
    combine_sorted_kernel<<<grid_for(ctx, m), 256, 0, s>>>(
        static_cast<const __half*>(partials_sorted), static_cast<const uint32_t*>(inv_scratch),
        static_cast<const __half*>(routing_weights), static_cast<__half*>(h2), (int)T, (int)top_k, (int)d);
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // extern "C"
