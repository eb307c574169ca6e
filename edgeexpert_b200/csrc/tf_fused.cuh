// tf_fused.cuh -- one decode MoE layer (router -> routed experts -> down +
// combine, with the shared expert) as a single persistent cooperative kernel.
//
// The three dependent stages of the reference's per-layer encoders
// (MoE.encodeRouterGemma4, encodeRoutedPersistentPhase1U16Load,
// encodeRoutedPersistentPhase2Reduce, SharedExpertRuntime.encode) run as
// phases of one launch, one CTA per SM, separated by grid barriers:
//   phase 0  router logits (int8 GEMV) and the shared expert's gate/up/GELU,
//            neither of which depends on the routing
//   barrier  every CTA selects the top-k itself from the 128 logits
//   phase 1  routed gate/up/GELU of the selected experts
//   barrier
//   phase 2  routed down projections weighted by the routing, plus the shared
//            expert's down projection and the residual
// The routing never leaves the GPU (the reference reads it back on the CPU,
// RealForwardRunner.swift:2491-2520).  The grid barrier spins with a bound:
// if it gives up it raises an error bit and the kernel runs on to the end.
#pragma once
#include "tf_policies.cuh"

namespace tf {

struct LayerParams {
    RouterParams r;     // fused mode: logits only
    Phase1Params sh;    // shared expert gate/up (top_k = 0)
    Phase1Params p1;    // routed gate/up, ids from shared memory
    Phase2Params p2;    // down + combine, ids and weights from shared memory
    int has_shared;
    unsigned int* bar_count;  // grid barrier words (context workspace)
    unsigned int* bar_flags;  // [gridDim.x * kFlagStride] release flags
    uint32_t* out_idx;        // routing for the caller (written by CTA 0)
    __half* out_w;
    uint32_t* err;
};

__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_gpu(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

constexpr uint32_t kGridSpinLimit = 1u << 24;
constexpr int kFlagStride = 32;  // words between per-CTA release flags (128 B)

// Generation barrier over all CTAs of a cooperative launch.  Arrivals count
// on one word; the last arriver releases every CTA through its own flag word
// (128 B apart) so the waiting CTAs do not all poll one L2 line.
__device__ __forceinline__ void grid_barrier(unsigned int* count, unsigned int* flags, uint32_t* err) {
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned int* mine = flags + blockIdx.x * kFlagStride;
        const unsigned int g = ld_acquire_gpu(mine);
        __threadfence();
        const unsigned int arrived = atomicAdd(count, 1u);
        if (arrived == gridDim.x - 1) {
            atomicExch(count, 0u);
            __threadfence();
            for (unsigned int b = 0; b < gridDim.x; ++b)
                *reinterpret_cast<volatile unsigned int*>(flags + b * kFlagStride) = g + 1u;
        } else {
            uint32_t i = 0;
            for (; i < kGridSpinLimit; ++i)
                if (ld_acquire_gpu(mine) != g) break;
            if (i == kGridSpinLimit) atomicOr(err, kErrMbarTimeout);
        }
        __threadfence();
    }
    __syncthreads();
}

template <typename ST>
__global__ void __launch_bounds__(kWarps * 32, 1) fused_layer_kernel(const __grid_constant__ LayerParams p) {
    EngineState es;
    TF_T(0);
    engine_init(es);
    run_phase<RouterPolicy<ST>, ST>(p.r, es);
    TF_T(1);
    if (p.has_shared) run_phase<Phase1Policy<ST>, ST>(p.sh, es);
    TF_T(2);
    grid_barrier(p.bar_count, p.bar_flags, p.err);
    TF_T(3);
    {
        // every CTA selects the routing itself (no second barrier needed)
        float* scratch = reinterpret_cast<float*>(engine_xarea_of(es));
        cta_topk_softmax(p.r.logits + (blockIdx.x % max(1, p.r.replicas)) * 256, p.r.E, p.r.top_k,
                         p.r.per_expert_scale, ids_smem(), rw_smem(), scratch);
        if (blockIdx.x == 0 && threadIdx.x < p.r.top_k) {
            p.out_idx[threadIdx.x] = ids_smem()[threadIdx.x];
            p.out_w[threadIdx.x] = rw_smem()[threadIdx.x];
        }
    }
    __syncthreads();
    TF_T(4);
    run_phase<Phase1Policy<ST>, ST>(p.p1, es);
    TF_T(5);
    grid_barrier(p.bar_count, p.bar_flags, p.err);
    TF_T(6);
    run_phase<Phase2Policy<ST>, ST>(p.p2, es);
    TF_T(7);
}

}  // namespace tf
