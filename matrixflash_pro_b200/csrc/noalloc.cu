// mfb_sgemm_noalloc: the strict-FP32 / TF32 tcgen05 GEMM with its operand scratch in a
// fixed, statically allocated device array instead of memory from cudaMalloc.
//
// Some callers cannot allocate device memory when they call a GEMM: code running
// under a framework that owns the whole device-memory budget and forbids library
// allocations, latency-critical paths where cudaMalloc/cudaFree (which synchronize
// the device) or an out-of-memory failure in the middle of a call are not
// acceptable, and plugins hosted in a process whose allocator they may not touch.
// This entry point serves them: it calls no cudaMalloc, cudaFree or allocating
// library routine. Its scratch is g_noalloc_scratch below, MFB_NOALLOC_SCRATCH_BYTES
// (64 MiB) that every GPU loading libmfb.so holds until the process exits.
//
// Rules (also in include/mfb.h):
//   * The first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it under the id of the
//     device's current CUDA context; make that first call before any stream capture. A
//     device reset or a new primary context gets a new id, so the next call looks the
//     address up again instead of reusing a stale one (where the driver cannot report a
//     context id, every call looks it up).
//   * All calls share the one array and it keeps the last call's contents. Nothing in
//     it needs to start at zero: the prepass rewrites every element the GEMM reads.
//     Calls that overlap on the GPU (different streams, or host threads without
//     ordering) race on it: order them on one stream or synchronize between them.
//   * A problem whose operand planes need more than the array holds is rejected with
//     MFB_EINVAL and a message that gives both sizes.
#include "gemm_tc.cuh"
#include "mfb_internal.h"

#include <map>
#include <mutex>

namespace mfb {

namespace {

// The address of this array is valid only in device code; host code must ask the
// runtime for it (cudaGetSymbolAddress) per device before passing it to a kernel.
static __device__ __align__(256) float g_noalloc_scratch[MFB_NOALLOC_SCRATCH_BYTES / sizeof(float)];

std::mutex g_noalloc_mutex;
std::map<unsigned long long, void*> g_noalloc_ptrs;  // context id -> the array's device address

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current CUDA context (never reused within a process),
// or false when the driver cannot say.
bool current_context_id(unsigned long long* id) {
    static CtxGetCurrentFn get_current = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    static CtxGetIdFn get_id = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetIdFn>(p);
    }();
    CUcontext ctx = nullptr;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
    return get_id(ctx, id) == CUDA_SUCCESS;
}

// Must run with `device` current (select_device has made it so, and the runtime has made
// its primary context current on this thread).
mfb_status_t noalloc_scratch(void** out) {
    unsigned long long ctx_id = 0;
    const bool keyed = current_context_id(&ctx_id);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (keyed) {
        auto it = g_noalloc_ptrs.find(ctx_id);
        if (it != g_noalloc_ptrs.end()) {
            *out = it->second;
            return MFB_OK;
        }
    }
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    if (ptr == nullptr) return fail(MFB_ECUDA, "cudaGetSymbolAddress returned a null scratch address");
    if (keyed) g_noalloc_ptrs[ctx_id] = ptr;
    *out = ptr;
    return MFB_OK;
}

}  // namespace

}  // namespace mfb

extern "C" MFB_API mfb_status_t mfb_sgemm_noalloc(int device, mfb_stream_t stream_h, const mfb_gemm_desc* desc,
                                                  const float* a, const float* b, float* c, const float* bias) {
    using namespace mfb;
    clear_error();
    MFB_TRY(validate_desc(desc, a, b, c, bias, true));
    const mfb_gemm_desc& d = *desc;
    if (d.m == 0 || d.n == 0) return MFB_OK;
    const bool scale_only = d.k == 0 || d.alpha == 0.0f;
    const size_t need = scale_only ? 0 : tc_workspace_bytes(d);
    if (need > MFB_NOALLOC_SCRATCH_BYTES)
        return fail(MFB_EINVAL, "mfb_sgemm_noalloc: this problem needs " + std::to_string(need) +
                                    " bytes of operand scratch; the allocation-free entry point holds " +
                                    std::to_string(static_cast<size_t>(MFB_NOALLOC_SCRATCH_BYTES)) +
                                    " bytes (use mfb_sgemm or a plan for larger problems)");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    if (scale_only) return scale_output(d, stream, c, bias);
    TcConfig cfg[4];
    if (tc_candidates(d, cfg, 4) == 0) return fail(MFB_EUNSUPPORTED, "no tcgen05 configuration");
    void* scratch = nullptr;
    MFB_TRY(noalloc_scratch(&scratch));
    return tc_gemm(d, cfg[0], stream, a, b, c, bias, scratch, MFB_NOALLOC_SCRATCH_BYTES);
}
