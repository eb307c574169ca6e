// tf_ep.cu -- device pieces of the expert-parallel MoE step (routed experts
// sharded across GPUs in contiguous id ranges, experts_per_rank each).
//
// The reference has no multi-GPU path; this is the B200 replacement for its
// SSD expert streaming when experts are spread over several GPUs.  A layer on
// each rank, with a fixed capacity of rows per (sender, owner) pair so the
// exchange sizes never leave the device:
//   tf_ep_dispatch_pack    token t -> slot (owner r, t) when one of its experts
//                          lives on r: fp16 row + header (local ids, weights)
//   all-to-all (NCCL)      equal splits: capacity rows to every rank
//   tf_ep_dispatch_unpack  received headers -> [rows][top_k] routing
//   tf_moe_route_sort + tf_moe_grouped_routed on the received rows (the
//                          grouped gate/up/GELU and down of the reference's
//                          prefill.metal:336-440,598-670)
//   tf_ep_expert_combine   per received row: fp32 sum over its slots here, in
//                          slot order, of fma(w, half partial)
//   all-to-all (NCCL)      the fp32 rows back to their senders
//   tf_ep_return_reduce    h2[t] = half(sum over owner ranks, in rank order)
#include "tf_context.cuh"

using namespace tf;

namespace {

// ---- fixed-capacity dispatch (device-resident counts, graph-capturable) ----
// A dispatch row is the token's fp16 hidden row (d halves) followed by a
// tf_ep_row_header.  Slot (r, t) of the send buffer carries token t to rank r
// when at least one of its top-k experts lives there; otherwise only the
// header is written (n_valid = 0) and the payload is left as it was.
__global__ void ep_dispatch_pack_kernel(const __half* __restrict__ x, long long ldx,
                                        const uint32_t* __restrict__ ids, const __half* __restrict__ w, int T, int K,
                                        int E, int per_rank, int cap, int d, uint8_t* __restrict__ send,
                                        uint32_t* err) {
    const int slot = blockIdx.x;  // r * cap + t
    const int r = slot / cap, t = slot - r * cap;
    const size_t row_bytes = (size_t)d * 2 + sizeof(tf_ep_row_header);
    uint8_t* row = send + (size_t)slot * row_bytes;
    __shared__ int s_n;
    if (threadIdx.x == 0) {
        tf_ep_row_header h;
        uint32_t n = 0;
        for (int k = 0; k < 8; ++k) {
            h.local_expert[k] = 0xFFFFFFFFu;
            h.weight_bits[k] = 0;
        }
        if (t < T) {
            for (int k = 0; k < K; ++k) {
                const uint32_t e = ids[(size_t)t * K + k];
                if (e >= (uint32_t)E) {
                    if (err) atomicOr(err, kErrBadExpert);
                    continue;
                }
                if ((int)(e / (uint32_t)per_rank) == r) {
                    h.local_expert[k] = e - (uint32_t)(r * per_rank);
                    h.weight_bits[k] = __half_as_ushort(w[(size_t)t * K + k]);
                    ++n;
                }
            }
        }
        h.n_valid = n;
        h.src_token = (uint32_t)t;
        h.reserved[0] = h.reserved[1] = 0;
        *reinterpret_cast<tf_ep_row_header*>(row + (size_t)d * 2) = h;
        s_n = (int)n;
    }
    __syncthreads();
    if (s_n == 0) return;
    const uint4* src = reinterpret_cast<const uint4*>(x + (long long)t * ldx);
    uint4* dst = reinterpret_cast<uint4*>(row);
    for (int c = threadIdx.x; c < d / 8; c += blockDim.x) dst[c] = __ldg(src + c);
}

// ids_out[i][k] / w_out[i][k] from the received headers (UINT32_MAX = empty slot)
__global__ void ep_dispatch_unpack_kernel(const uint8_t* __restrict__ recv, int rows, int d, int K,
                                          uint32_t* __restrict__ ids_out, __half* __restrict__ w_out) {
    const size_t row_bytes = (size_t)d * 2 + sizeof(tf_ep_row_header);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows * K; i += gridDim.x * blockDim.x) {
        const int row = i / K, k = i - row * K;
        const tf_ep_row_header* h = reinterpret_cast<const tf_ep_row_header*>(recv + (size_t)row * row_bytes + (size_t)d * 2);
        ids_out[i] = h->local_expert[k];
        w_out[i] = __ushort_as_half(h->weight_bits[k]);
    }
}

// out[row][:] = sum over the row's valid slots, in slot (rank) order, of
// fma(w, partial[row*K + slot]) in fp32; 0 for a row with none.
__global__ void ep_expert_combine_kernel(const __half* __restrict__ part, const uint32_t* __restrict__ ids,
                                         const __half* __restrict__ w, int rows, int K, int d,
                                         float* __restrict__ out) {
    const int d8 = d >> 3;
    const long long n = (long long)rows * d8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / d8), dv = (int)(i - (long long)row * d8);
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int k = 0; k < K; ++k) {
            if (__ldg(&ids[(size_t)row * K + k]) == 0xFFFFFFFFu) continue;
            const float wr = __half2float(w[(size_t)row * K + k]);
            const uint4 q = __ldcs(reinterpret_cast<const uint4*>(part + ((long long)row * K + k) * d) + dv);
            const __half2* hp = reinterpret_cast<const __half2*>(&q);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f2 = __half22float2(hp[j]);
                acc[2 * j] = fmaf(wr, f2.x, acc[2 * j]);
                acc[2 * j + 1] = fmaf(wr, f2.y, acc[2 * j + 1]);
            }
        }
        float4* o = reinterpret_cast<float4*>(out + (long long)row * d) + dv * 2;
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

// h2[t][:] = half(sum_r back[r][t][:]) in rank order (+ nothing else)
__global__ void ep_return_reduce_kernel(const float* __restrict__ back, int world, int cap, int T, int d,
                                        __half* __restrict__ h2, long long ldh) {
    const int d4 = d >> 2;
    const long long n = (long long)T * d4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / d4), dv = (int)(i - (long long)t * d4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int r = 0; r < world; ++r) {
            const float4 v = __ldcs(reinterpret_cast<const float4*>(back + ((long long)r * cap + t) * d) + dv);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        __half2* o = reinterpret_cast<__half2*>(h2 + (long long)t * ldh) + dv * 2;
        o[0] = __floats2half2_rn(acc.x, acc.y);
        o[1] = __floats2half2_rn(acc.z, acc.w);
    }
}


// ---- peer-memory exchange (one GPU per rank, CUDA IPC mappings over NVLink) ----
// Each rank owns a flag block of 2 x world counters, one 128-byte line each:
// recv_cnt[src] counts the dispatch CTAs of rank src whose rows have landed in
// this rank's receive buffer, back_cnt[owner] the combine CTAs of rank owner
// whose rows have landed in this rank's return buffer.  Writers store their
// rows to the peer, fence at system scope, then add 1 to the peer's counter;
// readers wait (bounded by time) for the expected count, and the counter is
// reset by the one CTA whose signal the resetting rank's partner cannot do
// without, so no reset can race with the next step's signals.
constexpr int kEpFlagStride = 32;  // uint32 per counter line
constexpr unsigned long long kEpWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long ep_now() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t ep_ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ep_signal(uint32_t* peer_counter) {
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(peer_counter) : "memory");
}
// bounded wait for *cnt >= want; false (and the error bit) when it times out
__device__ __forceinline__ bool ep_wait_count(const uint32_t* cnt, uint32_t want, uint32_t* err) {
    const unsigned long long t0 = ep_now();
    while (ep_ld_acquire(cnt) < want) {
        if (ep_now() - t0 > kEpWaitNs) {
            if (err) atomicOr(err, kErrMbarTimeout);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// Dispatch: warp w of CTA (block b, owner r) takes slot t = 8b + w and writes
// the token's row straight into rank r's receive buffer at [my_rank][t]
// (lane k < top_k maps routing slot k; the header's fields are one lane
// each); the CTA then signals recv_cnt[my_rank] on rank r by its slot count,
// so rank r waits for cap.  CTA 0 of each owner first resets this rank's
// back_cnt[r] (rank r cannot answer before that CTA's signal arrives).
constexpr int kEpDispatchWarps = 8;
__global__ void __launch_bounds__(32 * kEpDispatchWarps) ep_dispatch_p2p_kernel(
    const __half* __restrict__ x, long long ldx, const uint32_t* __restrict__ ids, const __half* __restrict__ w,
    int T, int K, int E, int per_rank, int cap, int d, int my_rank, uint8_t* const* __restrict__ peer_recv,
    uint32_t* const* __restrict__ peer_flags, uint32_t* my_flags, int world, uint32_t* err) {
    const int r = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kEpDispatchWarps + warp;
    if (blockIdx.x == 0 && threadIdx.x == 0) my_flags[(world + r) * kEpFlagStride] = 0u;  // back_cnt[r]
    if (t < cap) {
        const size_t row_bytes = (size_t)d * 2 + sizeof(tf_ep_row_header);
        uint8_t* row = peer_recv[r] + ((size_t)my_rank * cap + t) * row_bytes;
        uint32_t local = 0xFFFFFFFFu;
        uint16_t wbits = 0;
        if (t < T && lane < K) {
            const uint32_t e = ids[(size_t)t * K + lane];
            if (e >= (uint32_t)E) {
                if (err) atomicOr(err, kErrBadExpert);
            } else if ((int)(e / (uint32_t)per_rank) == r) {
                local = e - (uint32_t)(r * per_rank);
                wbits = __half_as_ushort(w[(size_t)t * K + lane]);
            }
        }
        const uint32_t n = (uint32_t)__popc(__ballot_sync(0xffffffffu, local != 0xFFFFFFFFu));
        tf_ep_row_header* h = reinterpret_cast<tf_ep_row_header*>(row + (size_t)d * 2);
        if (lane < 8) {
            h->local_expert[lane] = local;
            h->weight_bits[lane] = wbits;
        } else if (lane == 8) {
            h->n_valid = n;
        } else if (lane == 9) {
            h->src_token = (uint32_t)t;
        } else if (lane < 12) {
            h->reserved[lane - 10] = 0;
        }
        if (n) {
            const uint4* src = reinterpret_cast<const uint4*>(x + (long long)t * ldx);
            uint4* dst = reinterpret_cast<uint4*>(row);
            for (int c = lane; c < d / 8; c += 32) dst[c] = __ldg(src + c);
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int nslots = min(kEpDispatchWarps, cap - (int)blockIdx.x * kEpDispatchWarps);
        asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(peer_flags[r] + (size_t)my_rank * kEpFlagStride),
                     "r"((uint32_t)nslots)
                     : "memory");  // recv_cnt[my_rank] on r
    }
}

// Owner side: wait until every sender's cap rows have landed, then the
// headers -> [rows][K] routing (as ep_dispatch_unpack_kernel).
__global__ void ep_unpack_p2p_kernel(const uint8_t* __restrict__ recv, const uint32_t* my_flags, int world, int cap,
                                     int d, int K, uint32_t* __restrict__ ids_out, __half* __restrict__ w_out,
                                     uint32_t* err) {
    __shared__ bool ok;
    if (threadIdx.x == 0) {
        ok = true;
        for (int s = 0; s < world && ok; ++s) ok = ep_wait_count(my_flags + (size_t)s * kEpFlagStride, (uint32_t)cap, err);
    }
    __syncthreads();
    const int rows = world * cap;
    const size_t row_bytes = (size_t)d * 2 + sizeof(tf_ep_row_header);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows * K; i += gridDim.x * blockDim.x) {
        const int row = i / K, k = i - row * K;
        const tf_ep_row_header* h =
            reinterpret_cast<const tf_ep_row_header*>(recv + (size_t)row * row_bytes + (size_t)d * 2);
        // volatile loads: the rows were written by other GPUs
        ids_out[i] = ok ? __ldcv(&h->local_expert[k]) : 0xFFFFFFFFu;
        w_out[i] = ok ? __ushort_as_half(__ldcv(&h->weight_bits[k])) : __float2half_rn(0.f);
    }
}

// Owner side, after the grouped experts: CTA (src s, block b) sums its rows'
// slots (as ep_expert_combine_kernel) and stores the fp32 rows straight into
// rank s's return buffer at [my_rank][t]; then signals back_cnt[my_rank] on
// rank s.  The b == 0 CTA of each sender first resets this rank's
// recv_cnt[s] (every reader of the receive buffer ran before this kernel).
__global__ void ep_combine_p2p_kernel(const __half* __restrict__ part, const uint32_t* __restrict__ ids,
                                      const __half* __restrict__ w, int cap, int K, int d, int my_rank,
                                      float* const* __restrict__ peer_back, uint32_t* const* __restrict__ peer_flags,
                                      uint32_t* my_flags, int world) {
    const int s = blockIdx.y, b = blockIdx.x, nb = gridDim.x;
    if (b == 0 && threadIdx.x == 0) my_flags[(size_t)s * kEpFlagStride] = 0u;  // recv_cnt[s]
    const int d8 = d >> 3;
    const long long n = (long long)cap * d8;
    float* dst_base = peer_back[s] + (size_t)my_rank * cap * d;
    for (long long i = b * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)nb * blockDim.x) {
        const int t = (int)(i / d8), dv = (int)(i - (long long)t * d8);
        const int row = s * cap + t;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int k = 0; k < K; ++k) {
            if (__ldg(&ids[(size_t)row * K + k]) == 0xFFFFFFFFu) continue;
            const float wr = __half2float(w[(size_t)row * K + k]);
            const uint4 q = __ldcs(reinterpret_cast<const uint4*>(part + ((long long)row * K + k) * d) + dv);
            const __half2* hp = reinterpret_cast<const __half2*>(&q);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 f2 = __half22float2(hp[j]);
                acc[2 * j] = fmaf(wr, f2.x, acc[2 * j]);
                acc[2 * j + 1] = fmaf(wr, f2.y, acc[2 * j + 1]);
            }
        }
        float4* o = reinterpret_cast<float4*>(dst_base + (size_t)t * d) + dv * 2;
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) ep_signal(peer_flags[s] + (size_t)(world + my_rank) * kEpFlagStride);  // back_cnt[my_rank]
}

// Sender side: wait for every owner's nb combine CTAs, then the rank-order reduce.
__global__ void ep_reduce_p2p_kernel(const float* __restrict__ back, const uint32_t* my_flags, int world, int cap,
                                     int T, int d, int nb, __half* __restrict__ h2, long long ldh, uint32_t* err) {
    __shared__ bool ok;
    if (threadIdx.x == 0) {
        ok = true;
        for (int o = 0; o < world && ok; ++o)
            ok = ep_wait_count(my_flags + (size_t)(world + o) * kEpFlagStride, (uint32_t)nb, err);
    }
    __syncthreads();
    const int d4 = d >> 2;
    const long long n = (long long)T * d4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / d4), dv = (int)(i - (long long)t * d4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ok) {
            for (int r = 0; r < world; ++r) {
                const float4 v = __ldcv(reinterpret_cast<const float4*>(back + ((long long)r * cap + t) * d) + dv);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
        }
        __half2* o = reinterpret_cast<__half2*>(h2 + (long long)t * ldh) + dv * 2;
        o[0] = __floats2half2_rn(acc.x, acc.y);
        o[1] = __floats2half2_rn(acc.z, acc.w);
    }
}

// Combine CTAs per sender (the sender's reduce waits for this many signals
// from every owner): about two 16-byte items per thread, 8 to 128 CTAs.  A
// function of the shape only, so every rank derives the same count.
int ep_combine_blocks(uint32_t capacity, uint32_t d) {
    const long long items = (long long)capacity * (d / 8);
    return (int)std::max<long long>(8, std::min<long long>(128, (items + 511) / 512));
}

int grid_for(const tf_context* ctx, long long n) {
    return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)ctx->num_sms * 8));
}

}  // namespace

extern "C" {

tf_status tf_ep_dispatch_pack(tf_context* ctx, const void* hidden, uint32_t hidden_stride, const void* expert_ids,
                              const void* weights, uint32_t T, uint32_t top_k, uint32_t num_experts,
                              uint32_t experts_per_rank, uint32_t world, uint32_t capacity, uint32_t d, void* send,
                              void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_dispatch_pack";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0 || top_k > 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0, 1 <= top_k <= 8", name);
    if (world == 0 || experts_per_rank == 0 || (uint64_t)experts_per_rank * world != num_experts)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: num_experts must equal experts_per_rank * world", name);
    if (T > capacity) return fail(ctx, TF_ERR_INVALID_ARG, "%s: T (%u) exceeds the capacity (%u)", name, T, capacity);
    if (hidden_stride == 0) hidden_stride = d;
    if (hidden_stride < d || hidden_stride % 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: hidden stride", name);
    if (capacity == 0) return TF_OK;
    if (!send || (T && (!hidden || !expert_ids || !weights))) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(send) || (T && (!aligned16(hidden) || !aligned4(expert_ids) || !aligned2(weights))))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: hidden/send 16-byte aligned", name);
    ep_dispatch_pack_kernel<<<world * capacity, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(hidden), hidden_stride, static_cast<const uint32_t*>(expert_ids),
        static_cast<const __half*>(weights), (int)T, (int)top_k, (int)num_experts, (int)experts_per_rank,
        (int)capacity, (int)d, static_cast<uint8_t*>(send), ctx->d_err);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_ep_dispatch_unpack(tf_context* ctx, const void* recv, uint32_t rows, uint32_t d, uint32_t top_k,
                                void* expert_ids_out, void* weights_out, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_dispatch_unpack";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0 || top_k > 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0, 1 <= top_k <= 8", name);
    if (rows == 0) return TF_OK;
    if (!recv || !expert_ids_out || !weights_out) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(recv) || !aligned4(expert_ids_out) || !aligned2(weights_out))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: misaligned buffer", name);
    ep_dispatch_unpack_kernel<<<grid_for(ctx, (long long)rows * top_k), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(recv), (int)rows, (int)d, (int)top_k, static_cast<uint32_t*>(expert_ids_out),
        static_cast<__half*>(weights_out));
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_ep_expert_combine(tf_context* ctx, const void* route_partials, const void* expert_ids,
                               const void* weights, uint32_t rows, uint32_t top_k, uint32_t d, void* out,
                               void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_expert_combine";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0, top_k > 0", name);
    if (rows == 0) return TF_OK;
    if (!route_partials || !expert_ids || !weights || !out) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(route_partials) || !aligned16(out) || !aligned4(expert_ids) || !aligned2(weights))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: partials/out 16-byte aligned", name);
    const long long n = (long long)rows * (d / 8);
    ep_expert_combine_kernel<<<grid_for(ctx, n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(route_partials), static_cast<const uint32_t*>(expert_ids),
        static_cast<const __half*>(weights), (int)rows, (int)top_k, (int)d, static_cast<float*>(out));
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_ep_return_reduce(tf_context* ctx, const void* back, uint32_t world, uint32_t capacity, uint32_t T,
                              uint32_t d, void* h2, uint32_t h2_stride, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_return_reduce";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || world == 0) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0", name);
    if (T > capacity) return fail(ctx, TF_ERR_INVALID_ARG, "%s: T exceeds the capacity", name);
    if (h2_stride == 0) h2_stride = d;
    if (h2_stride < d || h2_stride % 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: h2 stride", name);
    if (T == 0) return TF_OK;
    if (!back || !h2) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(back) || !aligned16(h2)) return fail(ctx, TF_ERR_MISALIGNED, "%s: back/h2 16-byte aligned", name);
    const long long n = (long long)T * (d / 4);
    ep_return_reduce_kernel<<<grid_for(ctx, n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float*>(back), (int)world, (int)capacity, (int)T, (int)d, static_cast<__half*>(h2),
        (long long)h2_stride);
    return cuda_check(ctx, cudaGetLastError(), name);
}

size_t tf_ep_flag_bytes(uint32_t world) { return sizeof(uint32_t) * 2 * (size_t)world * kEpFlagStride; }

tf_status tf_ep_ipc_alloc(tf_context* ctx, size_t bytes, void** dev_ptr, void* ipc_handle) {
    if (!ctx || !dev_ptr || !ipc_handle || bytes == 0) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return cuda_check(ctx, e, "tf_ep_ipc_alloc");
    }
    *dev_ptr = p;
    return TF_OK;
}

tf_status tf_ep_ipc_open(tf_context* ctx, const void* ipc_handle, void** peer_ptr) {
    if (!ctx || !ipc_handle || !peer_ptr) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return cuda_check(ctx, cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess), "tf_ep_ipc_open");
}

tf_status tf_ep_ipc_close(tf_context* ctx, void* peer_ptr) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    return cuda_check(ctx, cudaIpcCloseMemHandle(peer_ptr), "tf_ep_ipc_close");
}

tf_status tf_ep_ipc_free(tf_context* ctx, void* dev_ptr) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    return cuda_check(ctx, cudaFree(dev_ptr), "tf_ep_ipc_free");
}

tf_status tf_ep_dispatch_p2p(tf_context* ctx, const void* hidden, uint32_t hidden_stride, const void* expert_ids,
                             const void* weights, uint32_t T, uint32_t top_k, uint32_t num_experts,
                             uint32_t experts_per_rank, uint32_t world, uint32_t rank, uint32_t capacity, uint32_t d,
                             const void* peer_recv, const void* peer_flags, void* my_flags, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_dispatch_p2p";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0 || top_k > 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: d %% 8 == 0, 1 <= top_k <= 8", name);
    if (world == 0 || rank >= world || experts_per_rank == 0 || (uint64_t)experts_per_rank * world != num_experts)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: num_experts must equal experts_per_rank * world", name);
    if (capacity == 0 || T > capacity) return fail(ctx, TF_ERR_INVALID_ARG, "%s: 0 < capacity, T <= capacity", name);
    if (hidden_stride == 0) hidden_stride = d;
    if (hidden_stride < d || hidden_stride % 8) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: hidden stride", name);
    if (!peer_recv || !peer_flags || !my_flags || (T && (!hidden || !expert_ids || !weights)))
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (T && (!aligned16(hidden) || !aligned4(expert_ids) || !aligned2(weights)))
        return fail(ctx, TF_ERR_MISALIGNED, "%s: hidden 16-byte aligned", name);
    const dim3 dgrid((capacity + kEpDispatchWarps - 1) / kEpDispatchWarps, world);
    ep_dispatch_p2p_kernel<<<dgrid, 32 * kEpDispatchWarps, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(hidden), hidden_stride, static_cast<const uint32_t*>(expert_ids),
        static_cast<const __half*>(weights), (int)T, (int)top_k, (int)num_experts, (int)experts_per_rank,
        (int)capacity, (int)d, (int)rank, static_cast<uint8_t* const*>(peer_recv),
        static_cast<uint32_t* const*>(peer_flags), static_cast<uint32_t*>(my_flags), (int)world, ctx->d_err);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_ep_dispatch_unpack_p2p(tf_context* ctx, const void* recv, const void* my_flags, uint32_t world,
                                    uint32_t capacity, uint32_t d, uint32_t top_k, void* expert_ids_out,
                                    void* weights_out, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_dispatch_unpack_p2p";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0 || top_k > 8 || world == 0 || capacity == 0)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: bad shape", name);
    if (!recv || !my_flags || !expert_ids_out || !weights_out) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    const long long rows = (long long)world * capacity;
    ep_unpack_p2p_kernel<<<grid_for(ctx, rows * top_k), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(recv), static_cast<const uint32_t*>(my_flags), (int)world, (int)capacity, (int)d,
        (int)top_k, static_cast<uint32_t*>(expert_ids_out), static_cast<__half*>(weights_out), ctx->d_err);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_ep_combine_p2p(tf_context* ctx, const void* route_partials, const void* expert_ids, const void* weights,
                            uint32_t world, uint32_t rank, uint32_t capacity, uint32_t top_k, uint32_t d,
                            const void* peer_back, const void* peer_flags, void* my_flags, void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_combine_p2p";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || top_k == 0 || world == 0 || rank >= world || capacity == 0)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: bad shape", name);
    if (!route_partials || !expert_ids || !weights || !peer_back || !peer_flags || !my_flags)
        return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(route_partials)) return fail(ctx, TF_ERR_MISALIGNED, "%s: partials 16-byte aligned", name);
    ep_combine_p2p_kernel<<<dim3(ep_combine_blocks(capacity, d), world), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(route_partials), static_cast<const uint32_t*>(expert_ids),
        static_cast<const __half*>(weights), (int)capacity, (int)top_k, (int)d, (int)rank,
        static_cast<float* const*>(peer_back), static_cast<uint32_t* const*>(peer_flags),
        static_cast<uint32_t*>(my_flags), (int)world);
    return cuda_check(ctx, cudaGetLastError(), name);
}

tf_status tf_ep_return_reduce_p2p(tf_context* ctx, const void* back, const void* my_flags, uint32_t world,
                                  uint32_t capacity, uint32_t T, uint32_t d, void* h2, uint32_t h2_stride,
                                  void* stream) {
    if (!ctx) return TF_ERR_INVALID_ARG;
    const char* name = "tf_ep_return_reduce_p2p";
    if (cudaSetDevice(ctx->device) != cudaSuccess) return fail(ctx, TF_ERR_CUDA, "cudaSetDevice failed");
    if (d == 0 || d % 8 || world == 0 || capacity == 0 || T > capacity)
        return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: bad shape", name);
    if (h2_stride == 0) h2_stride = d;
    if (!back || !my_flags || (T && !h2)) return fail(ctx, TF_ERR_INVALID_ARG, "%s: null pointer", name);
    if (!aligned16(back) || (T && !aligned16(h2))) return fail(ctx, TF_ERR_MISALIGNED, "%s: back/h2 16-byte aligned", name);
    // one CTA at least, so the wait runs even when this rank has no tokens
    const long long n = std::max<long long>(1, (long long)T * (d / 4));
    ep_reduce_p2p_kernel<<<grid_for(ctx, n), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const float*>(back), static_cast<const uint32_t*>(my_flags), (int)world, (int)capacity, (int)T,
        (int)d, ep_combine_blocks(capacity, d), static_cast<__half*>(h2), (long long)h2_stride, ctx->d_err);
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // extern "C"
