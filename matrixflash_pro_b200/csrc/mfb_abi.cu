// C-ABI entry points of libmfb.so (declared in include/mfb.h): argument validation
// with the reference's rules, device selection, scratch ownership, plans, the
// hw::cuda_gemm-compatible slot streams, and the device status word.
#include "gemm_tc.cuh"
#include "mfb_internal.h"

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <vector>

namespace mfb {

namespace {
thread_local std::string t_last_error;
std::atomic<uint64_t> g_wait_limit_ns{4000000000ull};
}  // namespace

mfb_status_t fail(mfb_status_t status, const std::string& msg) {
    t_last_error = msg;
    return status;
}

mfb_status_t cuda_fail(cudaError_t err, const char* what) {
    t_last_error = std::string(what) + ": " + cudaGetErrorString(err);
    if (err == cudaErrorMemoryAllocation) return MFB_ENOMEM;
    return MFB_ECUDA;
}

void clear_error() { t_last_error.clear(); }

uint64_t wait_limit_ns() { return g_wait_limit_ns.load(std::memory_order_relaxed); }

namespace {

struct DeviceInfo {
    bool checked = false;
    bool sm100 = false;
    int sms = 0;
};

std::mutex g_dev_mutex;
std::vector<DeviceInfo> g_devices;

}  // namespace

mfb_status_t select_device(int device) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= count) return fail(MFB_EINVAL, "CUDA device index out of range");
    {
        std::lock_guard<std::mutex> lock(g_dev_mutex);
        if (static_cast<int>(g_devices.size()) < count) g_devices.resize(count);
        DeviceInfo& info = g_devices[device];
        if (!info.checked) {
            cudaDeviceProp prop;
            e = cudaGetDeviceProperties(&prop, device);
            if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
            info.sm100 = prop.major == 10 && prop.minor == 0;
            info.sms = prop.multiProcessorCount;
            info.checked = true;
        }
        if (!info.sm100)
            return fail(MFB_EUNSUPPORTED, "libmfb kernels are built for sm_100a (B200); this device is not sm_100");
    }
    MFB_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
    return MFB_OK;
}

int sm_count(int device) {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (device >= 0 && device < static_cast<int>(g_devices.size()) && g_devices[device].checked)
        return g_devices[device].sms;
    return 148;
}

bool stream_capturing(cudaStream_t stream) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &st) != cudaSuccess) return false;
    return st != cudaStreamCaptureStatusNone;
}

// ------------------------------------------------------------------------------------
// Per-(device, stream) scratch for calls without a plan. Only one stream ever uses a
// buffer, so stream order alone keeps reuse safe (same rule as the reference's
// Environment, src/ops/gemm/plan/environment.inc:21-23).
// ------------------------------------------------------------------------------------
namespace {
struct Scratch {
    void* ptr = nullptr;
    size_t bytes = 0;
};
std::mutex g_scratch_mutex;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;
}  // namespace

mfb_status_t stream_workspace(int device, cudaStream_t stream, size_t bytes, void** out) {
    *out = nullptr;
    if (bytes == 0) return MFB_OK;
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    Scratch& s = g_scratch[{device, stream}];
    if (s.bytes >= bytes) {
        *out = s.ptr;
        return MFB_OK;
    }
    if (stream_capturing(stream))
        return fail(MFB_EINVAL,
                    "operation needs more scratch than this stream has while the stream is being captured; "
                    "create a plan (or run once) before capture");
    if (s.ptr) {
        // The old buffer may still be read by work queued on this stream.
        MFB_CUDA_TRY(cudaStreamSynchronize(stream), "scratch resize sync");
        cudaFree(s.ptr);
        s.ptr = nullptr;
        s.bytes = 0;
    }
    const size_t rounded = (bytes + (1u << 20) - 1) & ~static_cast<size_t>((1u << 20) - 1);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, rounded);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(e, "scratch cudaMalloc");
    }
    s.ptr = p;
    s.bytes = rounded;
    *out = p;
    return MFB_OK;
}

mfb_status_t validate_desc(const mfb_gemm_desc* d, const float* a, const float* b, const float* c,
                           const float* bias, bool need_bias_check) {
    if (!d) return fail(MFB_EINVAL, "null GEMM descriptor");
    if (d->m < 0 || d->n < 0 || d->k < 0) return fail(MFB_EINVAL, "GEMM dimensions must be non-negative");
    if (d->precision != MFB_PRECISION_FP32 && d->precision != MFB_PRECISION_TF32)
        return fail(MFB_EINVAL, "Invalid GEMM precision policy");
    if (d->epilogue < MFB_EPILOGUE_NONE || d->epilogue > MFB_EPILOGUE_BIAS_GELU)
        return fail(MFB_EINVAL, "Invalid GEMM epilogue");
    if ((d->trans_a != 0 && d->trans_a != 1) || (d->trans_b != 0 && d->trans_b != 1))
        return fail(MFB_EINVAL, "transpose flags must be 0 or 1");
    const int a_cols = d->trans_a ? d->m : d->k;
    const int b_cols = d->trans_b ? d->k : d->n;
    if (d->lda < std::max(1, a_cols)) return fail(MFB_EINVAL, "lda is smaller than the stored row length of A");
    if (d->ldb < std::max(1, b_cols)) return fail(MFB_EINVAL, "ldb is smaller than the stored row length of B");
    if (d->ldc < std::max(1, d->n)) return fail(MFB_EINVAL, "ldc is smaller than n");
    if (!need_bias_check) return MFB_OK;
    if (d->m > 0 && d->n > 0) {
        if (!c) return fail(MFB_EINVAL, "null C pointer");
        if (d->k > 0 && (!a || !b)) return fail(MFB_EINVAL, "null A or B pointer");
        if (c == a || c == b) return fail(MFB_EINVAL, "GEMM output cannot alias an input");
    }
    if (d->epilogue != MFB_EPILOGUE_NONE) {
        if (!bias) return fail(MFB_ESHAPE, "GEMM bias length must equal N");
        if (bias == c && d->m > 0 && d->n > 0) return fail(MFB_EINVAL, "GEMM output cannot alias bias");
    }
    return MFB_OK;
}

mfb_status_t read_and_clear_status(uint32_t* bits) {
    uint32_t v = 0;
    MFB_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_status, sizeof(v)), "status read");
    const uint32_t zero = 0;
    MFB_CUDA_TRY(cudaMemcpyToSymbol(g_status, &zero, sizeof(zero)), "status clear");
    if (bits) *bits = v;
    return v ? fail(MFB_ETIMEOUT, "a bounded device wait gave up (status 0x" + std::to_string(v) + ")") : MFB_OK;
}

// ------------------------------------------------------------------------------------
// GEMM dispatch shared by mfb_sgemm and plans
// ------------------------------------------------------------------------------------
enum Path { kPathTc = 0, kPathGemv = 1, kPathScale = 2, kPathEmpty = 3 };

int choose_path(const mfb_gemm_desc& d) {
    if (d.m == 0 || d.n == 0) return kPathEmpty;
    if (d.k == 0 || d.alpha == 0.0f) return kPathScale;
    if (gemv_eligible(d)) return kPathGemv;
    return kPathTc;
}

}  // namespace mfb

// ======================================================================================
// C ABI
// ======================================================================================
using namespace mfb;

struct mfb_plan {
    int device = 0;
    mfb_gemm_desc desc{};
    int path = kPathTc;
    TcConfig cfg{};
    TcConfig candidates[16];
    int n_candidates = 0;
    int sm_limit = 0;
    void* ws = nullptr;
    size_t ws_bytes = 0;
};

namespace {

// Shared body of mfb_plan_execute / mfb_plan_prepare / mfb_plan_multiply.
mfb_status_t plan_run(mfb_plan_t plan, mfb_stream_t stream_h, const float* a, const float* b, float* c,
                      float alpha, float beta, const float* bias, int phases) {
    clear_error();
    if (!plan) return fail(MFB_EINVAL, "Cannot execute a null or destroyed GEMM plan");
    mfb_gemm_desc d = plan->desc;
    d.alpha = alpha;
    d.beta = beta;
    const bool multiply = (phases & kPhaseMultiply) != 0;
    if (multiply) {
        MFB_TRY(validate_desc(&d, a, b, c, bias, true));
    } else if (d.m > 0 && d.n > 0 && d.k > 0 && !a && !b) {
        return fail(MFB_EINVAL, "mfb_plan_prepare needs A, B or both");
    }
    DeviceGuard guard;
    MFB_TRY(select_device(plan->device));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    int path = plan->path;
    if ((path == kPathTc || path == kPathGemv) && alpha == 0.0f && multiply) path = kPathScale;
    switch (path) {
        case kPathEmpty: return MFB_OK;
        case kPathScale: return multiply ? scale_output(d, stream, c, bias) : MFB_OK;
        case kPathGemv: return multiply ? gemv_launch(d, stream, a, b, c, bias, plan->ws, plan->ws_bytes) : MFB_OK;
        default: break;
    }
    // The plan's scratch was sized for this shape at creation; execute allocates nothing.
    if (tc_workspace_bytes(d) > plan->ws_bytes) return fail(MFB_EINVAL, "plan scratch does not cover this shape");
    return tc_gemm(d, plan->cfg, stream, a, b, c, bias, plan->ws, plan->ws_bytes, phases, plan->sm_limit);
}

}  // namespace

extern "C" {

MFB_API const char* mfb_status_string(mfb_status_t s) {
    switch (s) {
        case MFB_OK: return "MFB_OK";
        case MFB_EINVAL: return "MFB_EINVAL: invalid argument";
        case MFB_ECUDA: return "MFB_ECUDA: CUDA error";
        case MFB_ETIMEOUT: return "MFB_ETIMEOUT: bounded device wait timed out";
        case MFB_ENCCL: return "MFB_ENCCL: NCCL error";
        case MFB_EUNSUPPORTED: return "MFB_EUNSUPPORTED: unsupported request";
        case MFB_ENOMEM: return "MFB_ENOMEM: out of device memory";
        case MFB_ESHAPE: return "MFB_ESHAPE: operand shape mismatch";
    }
    return "MFB_UNKNOWN";
}

MFB_API const char* mfb_last_error(void) { return t_last_error.c_str(); }

MFB_API const char* mfb_version(void) {
    return "mfb 0.1 (sm_100a: tcgen05 tf32/3xtf32 GEMM, GEMV, implicit-GEMM conv2d, naive FFMA oracle)";
}

MFB_API mfb_status_t mfb_set_wait_limit_ns(uint64_t limit_ns) {
    if (limit_ns < 1000) return fail(MFB_EINVAL, "wait limit must be at least 1 microsecond");
    g_wait_limit_ns.store(limit_ns);
    return MFB_OK;
}

MFB_API uint64_t mfb_get_wait_limit_ns(void) { return wait_limit_ns(); }

MFB_API mfb_status_t mfb_device_status(int device, uint32_t* bits) {
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    MFB_CUDA_TRY(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    return read_and_clear_status(bits);
}

MFB_API mfb_status_t mfb_sync(int device, mfb_stream_t stream) {
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    MFB_CUDA_TRY(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
    MFB_CUDA_TRY(cudaGetLastError(), "pending CUDA error");
    return read_and_clear_status(nullptr);
}

MFB_API mfb_status_t mfb_sgemm(int device, mfb_stream_t stream_h, const mfb_gemm_desc* desc, const float* a,
                               const float* b, float* c, const float* bias) {
    clear_error();
    MFB_TRY(validate_desc(desc, a, b, c, bias, true));
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    const mfb_gemm_desc& d = *desc;
    switch (choose_path(d)) {
        case kPathEmpty: return MFB_OK;
        case kPathScale: return scale_output(d, stream, c, bias);
        case kPathGemv: {
            void* ws = nullptr;
            MFB_TRY(stream_workspace(device, stream, gemv_workspace_bytes(d), &ws));
            return gemv_launch(d, stream, a, b, c, bias, ws, gemv_workspace_bytes(d));
        }
        default: break;
    }
    TcConfig cfgs[4];
    if (tc_candidates(d, cfgs, 4) == 0) return fail(MFB_EUNSUPPORTED, "no tcgen05 configuration");
    const size_t need = tc_workspace_bytes_for(d, cfgs[0]);
    void* ws = nullptr;
    MFB_TRY(stream_workspace(device, stream, need, &ws));
    return tc_gemm(d, cfgs[0], stream, a, b, c, bias, ws, need);
}

MFB_API mfb_status_t mfb_sgemm_strided_batched(int device, mfb_stream_t stream_h, const mfb_gemm_desc* desc,
                                               const float* a, long long stride_a, const float* b,
                                               long long stride_b, float* c, long long stride_c, int batch_count,
                                               const float* bias) {
    clear_error();
    MFB_TRY(validate_desc(desc, a, b, c, bias, true));
    const mfb_gemm_desc& d = *desc;
    if (batch_count < 0) return fail(MFB_EINVAL, "batch count must be non-negative");
    if (batch_count > 65535) return fail(MFB_EINVAL, "batch count must be at most 65535");
    if (stride_a < 0 || stride_b < 0 || stride_c < 0) return fail(MFB_EINVAL, "batch strides must be non-negative");
    if (batch_count == 0 || d.m == 0 || d.n == 0) return MFB_OK;
    // Consecutive outputs may not overlap: C_i spans (m - 1) * ldc + n floats.
    if (batch_count > 1 && stride_c < static_cast<long long>(d.m - 1) * d.ldc + d.n)
        return fail(MFB_EINVAL, "stride_c makes the batch's outputs overlap");
    if (batch_count > 1 && d.k > 0 && d.alpha != 0.0f) {
        // No output may alias an input of any batch entry.
        const long long a_rows = d.trans_a ? d.k : d.m, b_rows = d.trans_b ? d.n : d.k;
        const float* a_end = a + stride_a * (batch_count - 1) + (a_rows - 1) * d.lda + (d.trans_a ? d.m : d.k);
        const float* b_end = b + stride_b * (batch_count - 1) + (b_rows - 1) * d.ldb + (d.trans_b ? d.k : d.n);
        const float* c_end = c + stride_c * (batch_count - 1) + static_cast<long long>(d.m - 1) * d.ldc + d.n;
        if ((c < a_end && a < c_end) || (c < b_end && b < c_end))
            return fail(MFB_EINVAL, "GEMM output cannot alias an input");
    }
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    if (d.k == 0 || d.alpha == 0.0f) {
        for (int i = 0; i < batch_count; ++i) MFB_TRY(scale_output(d, stream, c + stride_c * i, bias));
        return MFB_OK;
    }
    TcBatch batch;
    batch.count = batch_count;
    batch.stride_a = stride_a;
    batch.stride_b = stride_b;
    batch.stride_c = stride_c;
    TcConfig cfgs[4];
    if (tc_candidates(d, cfgs, 4, batch_count) == 0) return fail(MFB_EUNSUPPORTED, "no tcgen05 configuration");
    const size_t need = tc_workspace_bytes_for(d, cfgs[0], batch_count);
    void* ws = nullptr;
    MFB_TRY(stream_workspace(device, stream, need, &ws));
    return tc_gemm(d, cfgs[0], stream, a, b, c, bias, ws, need, kPhaseAll, 0, batch);
}

MFB_API mfb_status_t mfb_gemv(int device, mfb_stream_t stream_h, const mfb_gemm_desc* desc, const float* a,
                              const float* b, float* c, const float* bias) {
    clear_error();
    MFB_TRY(validate_desc(desc, a, b, c, bias, true));
    const mfb_gemm_desc& d = *desc;
    if (d.trans_a || d.trans_b) return fail(MFB_EINVAL, "mfb_gemv takes untransposed operands");
    if (!(d.n <= 16 || d.m == 1)) return fail(MFB_EINVAL, "mfb_gemv serves n <= 16 or m == 1");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    const int path = choose_path(d);
    if (path == kPathEmpty) return MFB_OK;
    if (path == kPathScale) return scale_output(d, stream, c, bias);
    void* ws = nullptr;
    MFB_TRY(stream_workspace(device, stream, gemv_workspace_bytes(d), &ws));
    return gemv_launch(d, stream, a, b, c, bias, ws, gemv_workspace_bytes(d));
}

MFB_API mfb_status_t mfb_naive_sgemm(int device, mfb_stream_t stream_h, const mfb_gemm_desc* desc, const float* a,
                                     const float* b, float* c, const float* bias) {
    clear_error();
    MFB_TRY(validate_desc(desc, a, b, c, bias, true));
    if (desc->trans_a || desc->trans_b) return fail(MFB_EINVAL, "the naive oracle takes untransposed operands");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    return naive_launch(*desc, reinterpret_cast<cudaStream_t>(stream_h), a, b, c, bias);
}

MFB_API mfb_status_t mfb_probe_wait_timeout(int device, mfb_stream_t stream_h, uint64_t limit_ns) {
    clear_error();
    if (limit_ns == 0 || limit_ns > 10000000000ull) return fail(MFB_EINVAL, "probe limit must be in (0, 10 s]");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    return probe_wait_launch(reinterpret_cast<cudaStream_t>(stream_h), limit_ns);
}

// ---------------------------------------------------------------------------- plans
MFB_API mfb_status_t mfb_plan_create(int device, const mfb_gemm_desc* desc, mfb_plan_t* out) {
    clear_error();
    if (!out) return fail(MFB_EINVAL, "null plan output");
    *out = nullptr;
    MFB_TRY(validate_desc(desc, nullptr, nullptr, nullptr, nullptr, false));
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    std::unique_ptr<mfb_plan> plan(new (std::nothrow) mfb_plan());
    if (!plan) return fail(MFB_ENOMEM, "plan allocation");
    plan->device = device;
    plan->desc = *desc;
    mfb_gemm_desc probe = *desc;
    probe.alpha = 1.0f;
    plan->path = choose_path(probe);
    size_t need = 0;
    if (plan->path == kPathTc) {
        plan->n_candidates = tc_candidates(probe, plan->candidates, 16);
        if (plan->n_candidates == 0) return fail(MFB_EUNSUPPORTED, "no tcgen05 configuration");
        plan->cfg = plan->candidates[0];
        // operand planes (hi/lo strict, or rounded TF32) and the partial slots of the largest
        // stream-K candidate, so that tuning may pick any candidate
        need = tc_workspace_bytes(probe);
        for (int i = 0; i < plan->n_candidates; ++i)
            need = std::max(need, tc_workspace_bytes_for(probe, plan->candidates[i]));
    } else if (plan->path == kPathGemv) {
        need = gemv_workspace_bytes(probe);
    }
    if (need) {
        cudaError_t e = cudaMalloc(&plan->ws, need);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return cuda_fail(e, "plan workspace cudaMalloc");
        }
        plan->ws_bytes = need;
    }
    *out = plan.release();
    return MFB_OK;
}

MFB_API mfb_status_t mfb_plan_execute(mfb_plan_t plan, mfb_stream_t stream_h, const float* a, const float* b,
                                      float* c, float alpha, float beta, const float* bias) {
    return plan_run(plan, stream_h, a, b, c, alpha, beta, bias, kPhaseAll);
}

MFB_API mfb_status_t mfb_plan_prepare(mfb_plan_t plan, mfb_stream_t stream_h, const float* a, const float* b) {
    return plan_run(plan, stream_h, a, b, nullptr, 1.0f, 0.0f, nullptr, kPhasePrepare);
}

MFB_API mfb_status_t mfb_plan_multiply(mfb_plan_t plan, mfb_stream_t stream_h, const float* a, const float* b,
                                       float* c, float alpha, float beta, const float* bias) {
    return plan_run(plan, stream_h, a, b, c, alpha, beta, bias, kPhaseMultiply);
}

MFB_API mfb_status_t mfb_plan_prepare_cols(mfb_plan_t plan, mfb_stream_t stream_h, const float* b, int ldb_src,
                                           int n0, int n1) {
    clear_error();
    if (!plan) return fail(MFB_EINVAL, "Cannot execute a null or destroyed GEMM plan");
    const mfb_gemm_desc& d = plan->desc;
    if (plan->path != kPathTc) return fail(MFB_EUNSUPPORTED, "column-range calls need a plan on the tcgen05 path");
    if (d.trans_b) return fail(MFB_EUNSUPPORTED, "column-range calls need a non-transposed B");
    if (n0 < 0 || n1 <= n0 || n1 > d.n || n0 % 32 != 0 || (n1 != d.n && n1 % 32 != 0))
        return fail(MFB_EINVAL, "column range must satisfy 0 <= n0 < n1 <= n with n0 and n1 (unless n) multiples "
                                "of 32");
    if (!b || ldb_src < n1 - n0) return fail(MFB_EINVAL, "B column block needs a pointer and ldb >= n1 - n0");
    DeviceGuard guard;
    MFB_TRY(select_device(plan->device));
    TcColumns cols;
    cols.n0 = n0;
    cols.n1 = n1;
    cols.b_src = b;
    cols.b_ld = ldb_src;
    return tc_gemm(d, plan->cfg, reinterpret_cast<cudaStream_t>(stream_h), nullptr, nullptr, nullptr, nullptr,
                   plan->ws, plan->ws_bytes, kPhasePrepare, plan->sm_limit, TcBatch(), TcPrologue(), cols);
}

MFB_API mfb_status_t mfb_plan_multiply_cols(mfb_plan_t plan, mfb_stream_t stream_h, const float* a, float* c,
                                            float alpha, float beta, const float* bias, int n0, int n1) {
    clear_error();
    if (!plan) return fail(MFB_EINVAL, "Cannot execute a null or destroyed GEMM plan");
    mfb_gemm_desc d = plan->desc;
    d.alpha = alpha;
    d.beta = beta;
    if (plan->path != kPathTc) return fail(MFB_EUNSUPPORTED, "column-range calls need a plan on the tcgen05 path");
    if (d.trans_b) return fail(MFB_EUNSUPPORTED, "column-range calls need a non-transposed B");
    if (n0 < 0 || n1 <= n0 || n1 > d.n || n0 % 32 != 0 || (n1 != d.n && n1 % 32 != 0))
        return fail(MFB_EINVAL, "column range must satisfy 0 <= n0 < n1 <= n with n0 and n1 (unless n) multiples "
                                "of 32");
    if (!a || !c) return fail(MFB_EINVAL, "null A or C pointer");
    if (c == a) return fail(MFB_EINVAL, "GEMM output cannot alias an input");
    if (d.epilogue != MFB_EPILOGUE_NONE && !bias) return fail(MFB_ESHAPE, "GEMM bias length must equal N");
    DeviceGuard guard;
    MFB_TRY(select_device(plan->device));
    TcColumns cols;
    cols.n0 = n0;
    cols.n1 = n1;
    return tc_gemm(d, plan->cfg, reinterpret_cast<cudaStream_t>(stream_h), a, nullptr, c, bias, plan->ws,
                   plan->ws_bytes, kPhaseMultiply, plan->sm_limit, TcBatch(), TcPrologue(), cols);
}

MFB_API mfb_status_t mfb_plan_set_sm_limit(mfb_plan_t plan, int sms) {
    clear_error();
    if (!plan) return fail(MFB_EINVAL, "null plan");
    if (sms < 0) return fail(MFB_EINVAL, "SM limit must be >= 0 (0 = all SMs)");
    plan->sm_limit = sms;
    return MFB_OK;
}

MFB_API mfb_status_t mfb_plan_tune(mfb_plan_t plan, mfb_stream_t stream_h, const float* a, const float* b,
                                   float* scratch_c, int repeats, int* candidates_tested, float* best_ms) {
    clear_error();
    if (!plan) return fail(MFB_EINVAL, "null plan");
    if (candidates_tested) *candidates_tested = 0;
    if (best_ms) *best_ms = 0.0f;
    if (plan->path != kPathTc) return MFB_OK;
    if (repeats < 1) repeats = 1;
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    if (stream_capturing(stream)) return fail(MFB_EINVAL, "Construct/tune GEMM plans before CUDA Graph capture");
    mfb_gemm_desc d = plan->desc;
    d.alpha = 1.0f;
    d.beta = 0.0f;
    d.epilogue = MFB_EPILOGUE_NONE;
    MFB_TRY(validate_desc(&d, a, b, scratch_c, nullptr, true));
    DeviceGuard guard;
    MFB_TRY(select_device(plan->device));
    const size_t need = tc_workspace_bytes(d);
    if (need > plan->ws_bytes) return fail(MFB_EINVAL, "plan workspace does not cover these operands");
    cudaEvent_t e0, e1;
    MFB_CUDA_TRY(cudaEventCreate(&e0), "event create");
    MFB_CUDA_TRY(cudaEventCreate(&e1), "event create");
    float best = -1.0f;
    int best_idx = 0;
    mfb_status_t st = MFB_OK;
    for (int i = 0; i < plan->n_candidates && st == MFB_OK; ++i) {
        std::vector<float> samples;
        st = tc_gemm(d, plan->candidates[i], stream, a, b, scratch_c, nullptr, plan->ws, plan->ws_bytes);  // warm
        for (int r = 0; r < repeats && st == MFB_OK; ++r) {
            cudaEventRecord(e0, stream);
            st = tc_gemm(d, plan->candidates[i], stream, a, b, scratch_c, nullptr, plan->ws, plan->ws_bytes);
            cudaEventRecord(e1, stream);
            if (cudaEventSynchronize(e1) != cudaSuccess) st = cuda_fail(cudaGetLastError(), "tune sync");
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, e0, e1);
            samples.push_back(ms);
        }
        if (st != MFB_OK) break;
        std::sort(samples.begin(), samples.end());
        const float med = samples[samples.size() / 2];
        if (best < 0.0f || med < best) {
            best = med;
            best_idx = i;
        }
        if (candidates_tested) *candidates_tested = i + 1;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    MFB_TRY(st);
    uint32_t bits = 0;
    MFB_TRY(read_and_clear_status(&bits));
    plan->cfg = plan->candidates[best_idx];
    if (best_ms) *best_ms = best;
    return MFB_OK;
}

MFB_API mfb_status_t mfb_plan_select_candidate(mfb_plan_t plan, int index) {
    clear_error();
    if (!plan) return fail(MFB_EINVAL, "null plan");
    if (plan->path != kPathTc) return index == 0 ? MFB_OK : fail(MFB_EINVAL, "this plan has one candidate");
    if (index < 0 || index >= plan->n_candidates) return fail(MFB_EINVAL, "candidate index out of range");
    plan->cfg = plan->candidates[index];
    return MFB_OK;
}

MFB_API mfb_status_t mfb_plan_info_get(mfb_plan_t plan, mfb_plan_info* info) {
    if (!plan || !info) return fail(MFB_EINVAL, "null plan or info");
    std::memset(info, 0, sizeof(*info));
    info->m = plan->desc.m;
    info->n = plan->desc.n;
    info->k = plan->desc.k;
    info->precision = plan->desc.precision;
    info->trans_a = plan->desc.trans_a;
    info->trans_b = plan->desc.trans_b;
    info->epilogue = plan->desc.epilogue;
    info->path = plan->path;
    info->tile_n = plan->path == kPathTc ? plan->cfg.bn : 0;
    info->stages = plan->path == kPathTc ? plan->cfg.stages : 0;
    info->candidates = plan->n_candidates;
    info->workspace_bytes = plan->ws_bytes;
    const char* name = plan->path == kPathTc
                           ? (plan->cfg.planes == 2 ? "tcgen05_3xtf32" : "tcgen05_tf32")
                           : plan->path == kPathGemv ? "gemv_fp32" : plan->path == kPathScale ? "scale" : "empty";
    std::snprintf(info->kernel, sizeof(info->kernel), "%s", name);
    info->sm_pair = plan->path == kPathTc ? plan->cfg.pair : 0;
    info->split_k = 1;
    info->stream_k_tiles = 0;
    info->workers = 0;
    if (plan->path == kPathTc) {
        DeviceGuard guard;
        MFB_TRY(select_device(plan->device));
        TcSchedule sc;
        MFB_TRY(tc_schedule(plan->desc, plan->cfg, plan->device, plan->sm_limit, 1, plan->desc.n, &sc));
        const size_t planes = static_cast<size_t>((tc_workspace_bytes(plan->desc) + 255) / 256 * 256);
        if (sc.sk_tiles > 0 && planes + sc.partial_bytes <= plan->ws_bytes) {
            info->split_k = sc.split;
            info->stream_k_tiles = sc.sk_tiles;
        }
        info->workers = sc.workers;
    }
    return MFB_OK;
}

MFB_API mfb_status_t mfb_plan_destroy(mfb_plan_t plan) {
    if (!plan) return MFB_OK;
    if (plan->ws) {
        DeviceGuard guard;
        cudaSetDevice(plan->device);
        cudaFree(plan->ws);  // waits for queued work that still reads it
    }
    delete plan;
    return MFB_OK;
}

// ---------------------------------------------------------------- hw::cuda_gemm drop-in
namespace {
struct Slot {
    cudaStream_t stream = nullptr;
    std::mutex mutex;
};
std::mutex g_slot_table_mutex;
std::vector<std::unique_ptr<Slot>> g_slots;

mfb_status_t slot_for(int device, Slot** out) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= count) return fail(MFB_EINVAL, "CUDA device index out of range");
    std::lock_guard<std::mutex> lock(g_slot_table_mutex);
    if (static_cast<int>(g_slots.size()) < count) {
        for (int i = static_cast<int>(g_slots.size()); i < count; ++i) g_slots.emplace_back(new Slot());
    }
    Slot& s = *g_slots[device];
    if (s.stream == nullptr) {
        DeviceGuard guard;
        MFB_TRY(select_device(device));
        MFB_CUDA_TRY(cudaStreamCreate(&s.stream), "cudaStreamCreate");
    }
    *out = &s;
    return MFB_OK;
}
}  // namespace

MFB_API mfb_status_t mfb_cuda_device_count(int* count) {
    if (!count) return fail(MFB_EINVAL, "null count");
    *count = 0;
    if (cudaGetDeviceCount(count) != cudaSuccess) {
        cudaGetLastError();
        *count = 0;
    }
    return MFB_OK;
}

MFB_API mfb_status_t mfb_cuda_gemm(int device, int m, int n, int k, const float* a, int lda, const float* b,
                                   int ldb, float* c, int ldc, float alpha, float beta) {
    clear_error();
    Slot* slot = nullptr;
    MFB_TRY(slot_for(device, &slot));
    std::lock_guard<std::mutex> lock(slot->mutex);
    mfb_gemm_desc d{};
    d.m = m;
    d.n = n;
    d.k = k;
    d.lda = lda;
    d.ldb = ldb;
    d.ldc = ldc;
    d.alpha = alpha;
    d.beta = beta;
    d.precision = MFB_PRECISION_FP32;
    return mfb_sgemm(device, reinterpret_cast<mfb_stream_t>(slot->stream), &d, a, b, c, nullptr);
}

MFB_API mfb_status_t mfb_cuda_sync(int device) {
    clear_error();
    Slot* slot = nullptr;
    MFB_TRY(slot_for(device, &slot));
    std::lock_guard<std::mutex> lock(slot->mutex);
    return mfb_sync(device, reinterpret_cast<mfb_stream_t>(slot->stream));
}

// ---------------------------------------------------------------- conv2d
MFB_API mfb_status_t mfb_conv2d_fwd(int device, mfb_stream_t stream_h, int n, int c, int h, int w, int k, int r,
                                    int s, int stride, int pad, const float* x, const float* wgt,
                                    const float* bias, float* y, int precision) {
    clear_error();
    if (n < 0 || c <= 0 || h <= 0 || w <= 0 || k <= 0 || r <= 0 || s <= 0 || pad < 0)
        return fail(MFB_EINVAL, "conv2d expects positive C, H, W, K, R, S and non-negative N and padding");
    if (stride <= 0) return fail(MFB_ESHAPE, "conv2d channel or stride mismatch");
    if (h + 2 * pad < r || w + 2 * pad < s) return fail(MFB_ESHAPE, "conv2d kernel is larger than padded input");
    if (precision != MFB_PRECISION_FP32 && precision != MFB_PRECISION_TF32)
        return fail(MFB_EINVAL, "Invalid conv precision policy");
    if (n > 0 && (!x || !wgt || !bias || !y)) return fail(MFB_EINVAL, "null conv2d pointer");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    return conv2d_launch(device, reinterpret_cast<cudaStream_t>(stream_h), n, c, h, w, k, r, s, stride, pad, x, wgt,
                         bias, y, precision);
}

namespace {
// Shape checks of the reference's validate_conv (src/nn/backward/convolution_kernels.cuh:98-115).
mfb_status_t validate_conv_bwd(int n, int c, int h, int w, int k, int r, int s, int stride, int pad, int precision) {
    if (n < 0 || c <= 0 || h <= 0 || w <= 0 || k <= 0 || r <= 0 || s <= 0 || pad < 0)
        return fail(MFB_EINVAL, "conv2d backward expects positive C, H, W, K, R, S and non-negative N and padding");
    if (stride <= 0) return fail(MFB_EINVAL, "conv2d backward stride must be positive");
    if (h + 2 * pad < r || w + 2 * pad < s) return fail(MFB_ESHAPE, "conv2d backward shape mismatch");
    if (precision != MFB_PRECISION_FP32 && precision != MFB_PRECISION_TF32)
        return fail(MFB_EINVAL, "Invalid conv precision policy");
    return MFB_OK;
}
}  // namespace

MFB_API mfb_status_t mfb_conv2d_bwd_data(int device, mfb_stream_t stream_h, int n, int c, int h, int w, int k, int r,
                                         int s, int stride, int pad, const float* dy, const float* wgt, float* dx,
                                         int precision) {
    clear_error();
    MFB_TRY(validate_conv_bwd(n, c, h, w, k, r, s, stride, pad, precision));
    if (n > 0 && (!dy || !wgt || !dx)) return fail(MFB_EINVAL, "null conv2d backward pointer");
    if (n > 0 && (dx == dy || dx == wgt)) return fail(MFB_EINVAL, "conv2d input gradient cannot alias an input");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    return conv2d_bwd_data_launch(device, reinterpret_cast<cudaStream_t>(stream_h), n, c, h, w, k, r, s, stride, pad,
                                  dy, wgt, dx, precision);
}

MFB_API mfb_status_t mfb_conv2d_bwd_filter(int device, mfb_stream_t stream_h, int n, int c, int h, int w, int k,
                                           int r, int s, int stride, int pad, const float* x, const float* dy,
                                           float* dw, int precision) {
    clear_error();
    MFB_TRY(validate_conv_bwd(n, c, h, w, k, r, s, stride, pad, precision));
    if (!dw || (n > 0 && (!x || !dy))) return fail(MFB_EINVAL, "null conv2d backward pointer");
    if (dw == x || dw == dy) return fail(MFB_EINVAL, "conv2d weight gradient cannot alias an input");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    return conv2d_bwd_filter_launch(device, reinterpret_cast<cudaStream_t>(stream_h), n, c, h, w, k, r, s, stride, pad,
                                    x, dy, dw, precision);
}

MFB_API mfb_status_t mfb_conv2d_bwd_bias(int device, mfb_stream_t stream_h, int n, int k, int p, int q,
                                         const float* dy, float* db) {
    clear_error();
    if (n < 0 || k < 0 || p < 0 || q < 0) return fail(MFB_EINVAL, "conv2d bias backward expects a rank-4 gradient");
    if (k > 0 && (!db || (n > 0 && p > 0 && q > 0 && !dy))) return fail(MFB_EINVAL, "null conv2d backward pointer");
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    return conv2d_bwd_bias_launch(device, reinterpret_cast<cudaStream_t>(stream_h), n, k, p, q, dy, db);
}

}  // extern "C"
