// tf_context.cuh -- host-side context, status plumbing and the engine launcher.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdlib.h>
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
    float* d_rt_logits = nullptr;      // [kRtLogitsCap] batched-router logits scratch
    float* d_qmm_part = nullptr;       // [kQmmPartCap] split-K partial sums of the dense GEMMs
    unsigned int* d_ticket = nullptr;  // router selection ticket (always left 0), barrier count
    unsigned int* d_flags = nullptr;   // fused-layer barrier release flags, 128 B apart
    uint32_t* d_idx = nullptr;         // [8] decode routing ids
    __half* d_w = nullptr;             // [8] decode routing weights
    __half* d_acts = nullptr;          // [8][kMaxF] routed activations
    __half* d_shared_act = nullptr;    // [kMaxFs] shared-expert activation
    uint32_t* d_sort_cnt = nullptr;    // [kRouteSortChunks][256] per-chunk expert counts / bases
    unsigned long long* d_lm_keys = nullptr;  // [kMaxLmTokens] LM-head argmax keys (left 0)
    unsigned int* d_lm_tickets = nullptr;     // [kMaxLmTokens] LM-head argmax block tickets (left 0)
    float* d_smx = nullptr;                   // [kMaxLmTokens][128][2] softmax partials (m, d)
    float* d_cand_v = nullptr;                // [2][kCandCap] top-K candidate values (sampling)
    uint32_t* d_cand_i = nullptr;             // [2][kCandCap] top-K candidate indices
};

// Device grouping: pairs are split into at most this many chunks (one CTA each).
constexpr int kRouteSortChunks = 1024;

namespace tf {

constexpr int kMaxRouterExperts = 256;
constexpr int kMaxF = 4096;
constexpr int kMaxFs = 16384;
constexpr int kMaxTopKDecode = 8;
constexpr int kMaxLmTokens = 256;
constexpr size_t kRtLogitsCap = 1u << 20;  // floats: 4096 tokens x 256 experts
constexpr size_t kQmmPartCap = 8u << 20;   // floats (32 MB)
constexpr int kCandCap = 65536;  // 256 tiles x 256 candidates: a 262144-entry vocabulary

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

// Largest dynamic shared memory an engine launch may request.
template <class Pol, typename ST, int H = 0>
size_t engine_smem_limit(tf_context* ctx) {
    static size_t static_smem = (size_t)-1;
    if (static_smem == (size_t)-1) {
        cudaFuncAttributes fa;
        if (cudaFuncGetAttributes(&fa, engine_kernel<Pol, ST, H>) != cudaSuccess) return 0;
        static_smem = fa.sharedSizeBytes;
    }
    return ctx->max_smem_optin - static_smem;
}

// Launch one engine instantiation: sets the dynamic shared-memory attribute
// once per instantiation and device, sizes the grid to min(super-jobs, SMs)
// (one CTA of kWarps warps, or 2 * kWarps with helper warps, per SM).
template <class Pol, typename ST, int H = 0>
tf_status launch_engine(tf_context* ctx, const typename Pol::Params& p, size_t x_bytes, int superjobs,
                        cudaStream_t stream, const char* name) {
    if (superjobs <= 0) return TF_OK;
    const size_t limit = engine_smem_limit<Pol, ST, H>(ctx);
    const size_t smem = engine_fixed_smem(H) + x_bytes + 1024;  // + slack for 1 KB alignment
    if (smem > limit) return fail(ctx, TF_ERR_UNSUPPORTED_SHAPE, "%s: activation too large for shared memory", name);
    static bool configured[64] = {};  // per instantiation, per device
    const int dev = ctx->device & 63;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(engine_kernel<Pol, ST, H>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)limit);
        if (e != cudaSuccess) return cuda_check(ctx, e, name);
        configured[dev] = true;
    }
    const int grid = superjobs < ctx->num_sms ? superjobs : ctx->num_sms;
    // Programmatic dependent launch (TFCUDA_PDL=0 turns it off): this grid's
    // launch and set-up overlap the preceding kernel's tail; the kernel waits
    // (griddepcontrol.wait) before reading anything that kernel produced.
    const char* pdl_env = getenv("TFCUDA_PDL");
    const bool pdl = !(pdl_env && pdl_env[0] == '0');
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kWarps * 32 * (1 + H));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cuda_check(ctx, cudaLaunchKernelEx(&cfg, engine_kernel<Pol, ST, H>, p), name);
}

// ---------------------------------------------------------------------------
// TMA descriptors.  A weight tensor is viewed as uint8 [depth][rows][row_bytes]
// (depth = experts of a pool or matrices of a batch) and read in boxes of
// 8 rows x 128 bytes with the 128-byte swizzle.
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
    static EncodeTiledFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

// Returns false when the tensor cannot be described (the caller then takes the
// synchronous copy path).
inline bool make_weight_map(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint64_t depth,
                            uint64_t depth_stride) {
    memset(m, 0, sizeof(*m));
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || !aligned16(base) || row_bytes % 16 || rows == 0 || depth == 0) return false;
    const uint64_t ds = depth > 1 ? depth_stride : row_bytes * rows;
    if (ds % 16 || ds >= (1ull << 40)) return false;
    cuuint64_t dims[3] = {row_bytes, rows, depth};
    cuuint64_t strides[2] = {row_bytes, ds};
    cuuint32_t box[3] = {(cuuint32_t)kBox, (cuuint32_t)kBoxRows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D fp16 activation map [rows][cols] with row pitch `ld` elements, boxes of
// 64 columns (128 B) x 64 rows in the 128-byte swizzle (the K-major operand
// layout of tcgen05.mma).  Out-of-range rows read as zero.
inline bool make_act_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld,
                         uint32_t box_rows = 64) {
    memset(m, 0, sizeof(*m));
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || !aligned16(base) || cols == 0 || rows == 0 || (ld * 2) % 16 || ld < cols) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t es[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D uint8 map over packed int4 weight rows [depth][rows][row_bytes]
// (depth = experts of a pool, depth_stride = blob stride), boxes of 32 bytes
// (one 64-element quantisation group) x box_rows rows, unswizzled.
inline bool make_raw_map(CUtensorMap* m, const void* base, uint64_t row_bytes, uint64_t rows, uint64_t depth,
                         uint64_t depth_stride, uint32_t box_rows = 64) {
    memset(m, 0, sizeof(*m));
    EncodeTiledFn fn = encode_tiled_fn();
    if (!fn || !aligned16(base) || row_bytes % 32 || rows == 0 || depth == 0) return false;
    const uint64_t ds = depth > 1 ? depth_stride : row_bytes * rows;
    if (ds % 16 || ds >= (1ull << 40)) return false;
    cuuint64_t dims[3] = {row_bytes, rows, depth};
    cuuint64_t strides[2] = {row_bytes, ds};
    cuuint32_t box[3] = {32, box_rows, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tf
