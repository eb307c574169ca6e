// tf_context.cuh -- host-side context, status plumbing and the engine launcher.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <string>

#include "../../include/tfcuda.h"
#include "tf_policies.cuh"

struct tf_context {
    int device = 0;
    int num_sms = 148;
    size_t max_smem_optin = 0;
    std::string last_error;
    // Device workspace (allocated once at create time).
    uint32_t* d_err = nullptr;         // error bits raised by kernels
    float* d_logits = nullptr;         // [kMaxRouterExperts] router logits
    unsigned int* d_ticket = nullptr;  // router selection ticket (always left 0)
    uint32_t* d_idx = nullptr;         // [8] decode routing ids
    __half* d_w = nullptr;             // [8] decode routing weights
    __half* d_acts = nullptr;          // [8][kMaxF] routed activations
    __half* d_shared_act = nullptr;    // [kMaxFs] shared-expert activation
};

namespace tf {

constexpr int kMaxRouterExperts = 256;
constexpr int kMaxF = 4096;
constexpr int kMaxFs = 16384;
constexpr int kMaxTopKDecode = 8;

inline tf_status fail(tf_context* ctx, tf_status s, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return s;
}

inline tf_status cuda_check(tf_context* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return TF_OK;
    return fail(ctx, TF_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned2(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 1u) == 0; }
inline bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Launch one engine instantiation: picks the ring depth that fits, sets the
// dynamic shared-memory attribute once per instantiation, sizes the grid to
// min(super-jobs, SMs) (one 256-thread CTA per SM).
template <class Pol, typename ST>
tf_status launch_engine(tf_context* ctx, typename Pol::Params p, size_t x_bytes, int superjobs,
                        cudaStream_t stream, const char* name) {
    if (superjobs <= 0) return TF_OK;
    // Dynamic shared memory may use what the kernel's static shared memory leaves.
    static size_t static_smem = (size_t)-1;
    if (static_smem == (size_t)-1) {
        cudaFuncAttributes fa;
        cudaError_t e = cudaFuncGetAttributes(&fa, engine_kernel<Pol, ST>);
        if (e != cudaSuccess) return cuda_check(ctx, e, name);
        static_smem = fa.sharedSizeBytes;
    }
    const size_t limit = ctx->max_smem_optin - static_smem;
    int ns = 3;
    size_t smem = engine_fixed_smem(ns) + x_bytes;
    if (smem > limit) {
        ns = 2;
        smem = engine_fixed_smem(ns) + x_bytes;
    }
    if (smem > limit) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: activation too large for shared memory", name);
    p.ns = ns;
    static bool configured[64] = {};  // per instantiation, per device
    const int dev = ctx->device & 63;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(engine_kernel<Pol, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)limit);
        if (e != cudaSuccess) return cuda_check(ctx, e, name);
        configured[dev] = true;
    }
    const int grid = superjobs < ctx->num_sms ? superjobs : ctx->num_sms;
    engine_kernel<Pol, ST><<<grid, kWarps * 32, smem, stream>>>(p);
    return cuda_check(ctx, cudaGetLastError(), name);
}

}  // namespace tf
