// tf_api_noalloc.cu -- tf_router_topk_noalloc: the fused router + top-k with
// its scratch (router logits, selection ticket, device error words) in a
// fixed file-scope device array instead of a tf_context workspace.
//
// Why: some callers cannot call cudaMalloc at all -- code that runs inside a
// host that owns every device allocation (a custom allocator or a memory pool
// that forbids side allocations), or a process that must not allocate after
// start-up.  This entry point needs no context and allocates nothing; every
// GPU that loads the library carries the small array below until exit.
#include <mutex>

#include "tf_context.cuh"

using namespace tf;

namespace {

constexpr int kNoAllocMaxExperts = 256;  // largest num_experts accepted
// Layout: [logits: 256 floats][ticket: 1 uint][error words: 4 uint], padded.
constexpr size_t kNoAllocLogitsOff = 0;
constexpr size_t kNoAllocTicketOff = kNoAllocMaxExperts * sizeof(float);
constexpr size_t kNoAllocErrOff = kNoAllocTicketOff + 16;
constexpr size_t kNoAllocBytes = kNoAllocErrOff + 16;

static __device__ __align__(256) uint8_t g_router_scratch[kNoAllocBytes];

struct DeviceSetup {
    bool done = false;
    uint8_t* scratch = nullptr;  // device address of g_router_scratch on this device
    int num_sms = 0;
    size_t max_smem_optin = 0;
};
std::mutex g_setup_mutex;
DeviceSetup g_setup[64];

// Once per device, with that device current: resolve the array's device
// address (its host-side name is a stand-in, not a device pointer) and read
// the launch limits.  Nothing is written: a __device__ array without an
// initialiser is zero when the module loads, and every launch leaves the
// ticket at 0 again.  The cached address assumes the module stays loaded, so
// cudaDeviceReset between calls is not supported.
tf_status setup_device(int dev, DeviceSetup** out) {
    if (dev < 0 || dev >= 64) return TF_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> lk(g_setup_mutex);
    DeviceSetup& s = g_setup[dev];
    if (!s.done) {
        int major = 0, sms = 0, optin = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major < 10)
            return TF_ERR_NO_DEVICE;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return TF_ERR_CUDA;
        if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
            return TF_ERR_CUDA;
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_router_scratch) != cudaSuccess || ptr == nullptr) return TF_ERR_CUDA;
        s.scratch = static_cast<uint8_t*>(ptr);
        s.num_sms = sms;
        s.max_smem_optin = (size_t)optin;
        s.done = true;
    }
    *out = &s;
    return TF_OK;
}

}  // namespace

extern "C" {

tf_status tf_router_topk_noalloc(const void* W, const void* S, const void* B, const void* hidden, const void* es,
                                 const void* pes, void* out_idx, void* out_w, uint32_t E, uint32_t d,
                                 uint32_t top_k, tf_scale_type st, void* stream) {
    if (!W || !S || !B || !hidden || !es || !pes || !out_idx || !out_w) return TF_ERR_INVALID_ARG;
    if (st != TF_SCALE_BF16 && st != TF_SCALE_F16) return TF_ERR_INVALID_ARG;
    if (E == 0 || E > (uint32_t)kNoAllocMaxExperts) return TF_ERR_UNSUPPORTED_SHAPE;  // beyond the fixed scratch
    if (d == 0 || d % 64) return TF_ERR_UNSUPPORTED_SHAPE;
    if (top_k == 0 || top_k > 32 || top_k > E) return TF_ERR_UNSUPPORTED_SHAPE;
    if (!aligned2(W) || !aligned2(S) || !aligned2(B) || !aligned2(hidden) || !aligned2(es) || !aligned2(pes) ||
        (reinterpret_cast<uintptr_t>(out_idx) & 3u))
        return TF_ERR_MISALIGNED;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TF_ERR_NO_DEVICE;
    DeviceSetup* s = nullptr;
    tf_status rc = setup_device(dev, &s);
    if (rc) return rc;

    // A stack-only context carries the launch limits; it owns no memory.
    tf_context ctx;
    ctx.device = dev;
    ctx.num_sms = s->num_sms;
    ctx.max_smem_optin = s->max_smem_optin;

    RouterParams p;
    memset(&p, 0, sizeof(p));
    p.W = static_cast<const uint8_t*>(W);
    p.S = S;
    p.B = B;
    p.hidden = static_cast<const __half*>(hidden);
    p.eff_scale = static_cast<const __nv_bfloat16*>(es);
    p.per_expert_scale = static_cast<const __nv_bfloat16*>(pes);
    p.E = (int)E;
    p.D = (int)d;
    p.top_k = (int)top_k;
    p.logits = reinterpret_cast<float*>(s->scratch + kNoAllocLogitsOff);
    p.ticket = reinterpret_cast<unsigned int*>(s->scratch + kNoAllocTicketOff);  // left at 0 by every launch
    p.out_idx = static_cast<uint32_t*>(out_idx);
    p.out_w = static_cast<__half*>(out_w);
    p.aligned = make_weight_map(&p.map, W, d, E, 1, 0);
    p.err = reinterpret_cast<uint32_t*>(s->scratch + kNoAllocErrOff);
    p.sched = make_sched(((int)E + 15) / 16, units_for_K((int)d, 8), 0, 1, ctx.num_sms);
    const int sj = p.sched.S_total;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (st == TF_SCALE_F16)
        return launch_engine<RouterPolicy<__half>, __half>(&ctx, p, RouterPolicy<__half>::x_bytes((int)d), sj, cs,
                                                           "tf_router_topk_noalloc");
    return launch_engine<RouterPolicy<__nv_bfloat16>, __nv_bfloat16>(
        &ctx, p, RouterPolicy<__nv_bfloat16>::x_bytes((int)d), sj, cs, "tf_router_topk_noalloc");
}

tf_status tf_router_topk_noalloc_check(void* stream, uint32_t* flags_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return TF_ERR_NO_DEVICE;
    DeviceSetup* s = nullptr;
    tf_status rc = setup_device(dev, &s);
    if (rc) return rc;
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    uint32_t* err = reinterpret_cast<uint32_t*>(s->scratch + kNoAllocErrOff);
    uint32_t words[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemcpyAsync(words, err, sizeof(words), cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) e = cudaMemsetAsync(err, 0, sizeof(words), cs);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cs);
    if (e != cudaSuccess) return TF_ERR_CUDA;
    if (flags_out) *flags_out = words[0];
    if (words[0] & kErrMbarTimeout) return TF_ERR_TIMEOUT;
    if (words[0] & kErrAlign) return TF_ERR_MISALIGNED;
    if (words[0] & kErrBadExpert) return TF_ERR_INVALID_ARG;
    return TF_OK;
}

}  // extern "C"
