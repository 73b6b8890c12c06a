// GEMM on operands that may live in host memory: mfb_sgemm_host.
//
// The reference's host-side GEMM with a GPU share, HeterogeneousScheduler::gemm
// (src/hw/scheduler.cpp:236-312), copies B, then the GPU rows of A (and C when
// beta != 0) to the device, runs hw::cuda_gemm, copies C back and synchronizes: every
// transfer and the GEMM run one after another. Here the rows of C stream through the
// GPU in panels: a copy-in stream brings panel i's rows of A and C into a ring of
// device slots while the caller's stream runs the GEMM of panel i-1 and a copy-out
// stream returns panel i-2's rows of C, so PCIe traffic in both directions overlaps
// the tensor-core work and the call costs about max(bytes in / H2D bandwidth, GEMM)
// plus one panel. B (and the bias) is copied once per call and split once per call
// (one plan per panel shape, B prepared once, A per panel).
//
// Each operand may be host memory (pinned for full speed; pageable memory works, its
// copies are staged by the driver) or memory of `device`. The call is stream-ordered
// on `stream`: host C holds the result once `stream` has been synchronized.
#include "mfb_internal.h"

#include <cstdlib>
#include <map>
#include <memory>
#include <mutex>

namespace mfb {
namespace {

constexpr int kRing = 3;                           // device slots per streamed operand
constexpr size_t kPanelTargetBytes = 48ull << 20;  // host bytes moved per panel (both directions)
constexpr int kMaxPanels = 64;

// Host bytes per panel: kPanelTargetBytes, or MFB_HOST_PANEL_MB from the environment.
size_t panel_target_bytes() {
    static const size_t v = [] {
        const char* e = std::getenv("MFB_HOST_PANEL_MB");
        const long long mb = e ? std::atoll(e) : 0;
        return mb > 0 ? static_cast<size_t>(mb) << 20 : kPanelTargetBytes;
    }();
    return v;
}

size_t round_up_sz(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Host (pinned, registered or pageable) or memory of `device` (managed counts as device).
mfb_status_t on_device(const void* p, int device, bool* dev, const char* what) {
    *dev = false;
    if (!p) return MFB_OK;
    cudaPointerAttributes at{};
    const cudaError_t e = cudaPointerGetAttributes(&at, p);
    if (e != cudaSuccess) {
        cudaGetLastError();  // an unknown pointer is plain host memory
        return MFB_OK;
    }
    if (at.type == cudaMemoryTypeDevice) {
        if (at.device != device) return fail(MFB_EINVAL, std::string(what) + " is memory of another device");
        *dev = true;
    } else if (at.type == cudaMemoryTypeManaged) {
        *dev = true;
    }
    return MFB_OK;
}

struct Stager {
    std::mutex mutex;
    cudaStream_t in = nullptr, out = nullptr;
    cudaEvent_t entry = nullptr, b_ready = nullptr, done = nullptr;
    cudaEvent_t ev_in[kRing] = {}, ev_gemm[kRing] = {}, ev_out[kRing] = {};
    bool pending = false;  // `done` holds the previous call's last copy-out
    void* buf = nullptr;
    size_t bytes = 0;
    mfb_plan_t plan = nullptr;
    mfb_gemm_desc plan_desc{};
};

std::mutex g_stagers_mutex;
std::map<int, std::unique_ptr<Stager>> g_stagers;

mfb_status_t stager_for(int device, Stager** out) {
    std::lock_guard<std::mutex> lock(g_stagers_mutex);
    std::unique_ptr<Stager>& s = g_stagers[device];
    if (!s) {
        auto fresh = std::make_unique<Stager>();
        MFB_CUDA_TRY(cudaStreamCreateWithFlags(&fresh->in, cudaStreamNonBlocking), "host GEMM copy-in stream");
        MFB_CUDA_TRY(cudaStreamCreateWithFlags(&fresh->out, cudaStreamNonBlocking), "host GEMM copy-out stream");
        cudaEvent_t* evs[] = {&fresh->entry, &fresh->b_ready, &fresh->done};
        for (cudaEvent_t* e : evs) MFB_CUDA_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "event");
        for (int i = 0; i < kRing; ++i) {
            MFB_CUDA_TRY(cudaEventCreateWithFlags(&fresh->ev_in[i], cudaEventDisableTiming), "event");
            MFB_CUDA_TRY(cudaEventCreateWithFlags(&fresh->ev_gemm[i], cudaEventDisableTiming), "event");
            MFB_CUDA_TRY(cudaEventCreateWithFlags(&fresh->ev_out[i], cudaEventDisableTiming), "event");
        }
        s = std::move(fresh);
    }
    *out = s.get();
    return MFB_OK;
}

bool same_desc(const mfb_gemm_desc& x, const mfb_gemm_desc& y) {
    return x.m == y.m && x.n == y.n && x.k == y.k && x.lda == y.lda && x.ldb == y.ldb && x.ldc == y.ldc &&
           x.precision == y.precision && x.trans_a == y.trans_a && x.trans_b == y.trans_b &&
           x.epilogue == y.epilogue;
}

// Copies `rows` rows of `width_bytes` between pitched buffers on `stream`.
mfb_status_t copy_rows(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width_bytes, size_t rows,
                       cudaMemcpyKind kind, cudaStream_t stream) {
    if (rows == 0 || width_bytes == 0) return MFB_OK;
    MFB_CUDA_TRY(cudaMemcpy2DAsync(dst, dpitch, src, spitch, width_bytes, rows, kind, stream), "host GEMM copy");
    return MFB_OK;
}

}  // namespace
}  // namespace mfb

using namespace mfb;

extern "C" MFB_API mfb_status_t mfb_sgemm_host(int device, mfb_stream_t stream_h, const mfb_gemm_desc* desc,
                                               const float* a, const float* b, float* c, const float* bias) {
    clear_error();
    MFB_TRY(validate_desc(desc, a, b, c, bias, true));
    const mfb_gemm_desc d = *desc;
    if (d.m == 0 || d.n == 0) return MFB_OK;
    DeviceGuard guard;
    MFB_TRY(select_device(device));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    const bool uses_ab = d.k > 0 && d.alpha != 0.0f;
    bool a_dev = true, b_dev = true, c_dev = false, bias_dev = true;
    if (uses_ab) {
        MFB_TRY(on_device(a, device, &a_dev, "A"));
        MFB_TRY(on_device(b, device, &b_dev, "B"));
    }
    MFB_TRY(on_device(c, device, &c_dev, "C"));
    if (d.epilogue != MFB_EPILOGUE_NONE) MFB_TRY(on_device(bias, device, &bias_dev, "bias"));
    if (a_dev && b_dev && c_dev && bias_dev) return mfb_sgemm(device, stream_h, desc, a, b, c, bias);

    // ---- panel size: ~kPanelTargetBytes of host traffic, whole 256-row pair tiles, <= 64 panels
    const bool c_in = !c_dev && d.beta != 0.0f;
    const size_t row_bytes = (uses_ab && !a_dev ? 4ull * d.k : 0) + (!c_dev ? 4ull * d.n : 0) * (c_in ? 2 : 1);
    long long rows = row_bytes ? static_cast<long long>(panel_target_bytes() / row_bytes) / 256 * 256 : d.m;
    rows = std::max<long long>(rows, 256);
    rows = std::max<long long>(rows, round_up_sz((d.m + kMaxPanels - 1) / kMaxPanels, 256));
    const int rc = static_cast<int>(std::min<long long>(rows, d.m));
    const int panels = (d.m + rc - 1) / rc;

    // ---- device layout: [B][bias][A slots][C slots], each 256-byte aligned
    const int b_rows = d.trans_b ? d.n : d.k, b_cols = d.trans_b ? d.k : d.n;
    const size_t bld = round_up_sz(b_cols, 4);
    const size_t ald = d.trans_a ? round_up_sz(rc, 4) : round_up_sz(d.k, 4);
    const size_t a_slot_rows = d.trans_a ? d.k : rc;
    const size_t cld = round_up_sz(d.n, 4);
    const size_t b_bytes = uses_ab && !b_dev ? round_up_sz(4 * bld * b_rows, 256) : 0;
    const size_t bias_bytes = !bias_dev ? round_up_sz(4ull * d.n, 256) : 0;
    const size_t a_slot = uses_ab && !a_dev ? round_up_sz(4 * ald * a_slot_rows, 256) : 0;
    const size_t c_slot = !c_dev ? round_up_sz(4 * cld * rc, 256) : 0;
    const size_t need = b_bytes + bias_bytes + kRing * (a_slot + c_slot);

    Stager* st = nullptr;
    MFB_TRY(stager_for(device, &st));
    std::lock_guard<std::mutex> lock(st->mutex);
    if (need > st->bytes) {
        // The previous call's copies and GEMMs may still use the old buffer.
        if (st->pending) MFB_CUDA_TRY(cudaEventSynchronize(st->done), "host GEMM buffer resize");
        if (st->buf) cudaFree(st->buf);
        st->buf = nullptr;
        st->bytes = 0;
        const cudaError_t e = cudaMalloc(&st->buf, need);
        if (e != cudaSuccess) {
            cudaGetLastError();
            st->buf = nullptr;
            return cuda_fail(e, "host GEMM device buffers");
        }
        st->bytes = need;
    }
    char* base = static_cast<char*>(st->buf);
    float* b_d = b_bytes ? reinterpret_cast<float*>(base) : const_cast<float*>(b);
    const long long b_ld = b_bytes ? static_cast<long long>(bld) : d.ldb;
    float* bias_d = bias_bytes ? reinterpret_cast<float*>(base + b_bytes) : const_cast<float*>(bias);
    char* a_slots = base + b_bytes + bias_bytes;
    char* c_slots = a_slots + kRing * a_slot;

    // ---- entry: wait for the caller's stream and for the previous call's last copy-out
    MFB_CUDA_TRY(cudaEventRecord(st->entry, stream), "event record");
    MFB_CUDA_TRY(cudaStreamWaitEvent(st->in, st->entry, 0), "stream wait");
    if (st->pending) MFB_CUDA_TRY(cudaStreamWaitEvent(st->in, st->done, 0), "stream wait");
    if (b_bytes)
        MFB_TRY(copy_rows(b_d, 4 * bld, b, 4ull * d.ldb, 4ull * b_cols, b_rows, cudaMemcpyHostToDevice, st->in));
    if (bias_bytes) MFB_CUDA_TRY(cudaMemcpyAsync(bias_d, bias, 4ull * d.n, cudaMemcpyHostToDevice, st->in), "bias");
    MFB_CUDA_TRY(cudaEventRecord(st->b_ready, st->in), "event record");
    MFB_CUDA_TRY(cudaStreamWaitEvent(stream, st->b_ready, 0), "stream wait");

    // ---- one plan for full panels; B split once per call
    mfb_gemm_desc pd = d;
    pd.m = rc;
    pd.lda = uses_ab ? (a_dev ? d.lda : static_cast<int>(ald)) : d.lda;
    pd.ldb = static_cast<int>(b_ld);
    pd.ldc = c_dev ? d.ldc : static_cast<int>(cld);
    const bool full_panels = d.m / rc > 0 && panels > 1;
    if (full_panels && uses_ab) {
        if (!st->plan || !same_desc(st->plan_desc, pd)) {
            if (st->plan) mfb_plan_destroy(st->plan);
            st->plan = nullptr;
            MFB_TRY(mfb_plan_create(device, &pd, &st->plan));
            st->plan_desc = pd;
        }
        MFB_TRY(mfb_plan_prepare(st->plan, stream_h, nullptr, b_d));
    }

    mfb_status_t status = MFB_OK;
    auto cu = [](cudaError_t e, const char* what) { return e == cudaSuccess ? MFB_OK : cuda_fail(e, what); };
    for (int i = 0; i < panels && status == MFB_OK; ++i) {
        const int slot = i % kRing;
        const int r0 = i * rc;
        const int pr = std::min(rc, d.m - r0);
        // copy in (slot reuse waits for the copy-out of panel i - kRing, which followed its GEMM)
        if (i >= kRing && (status = cu(cudaStreamWaitEvent(st->in, st->ev_out[slot], 0), "stream wait")) != MFB_OK)
            break;
        const float* a_p = a;
        long long a_ld = d.lda;
        if (uses_ab && a_dev) {
            a_p = d.trans_a ? a + r0 : a + static_cast<size_t>(r0) * d.lda;
        } else if (uses_ab) {
            float* dst = reinterpret_cast<float*>(a_slots + slot * a_slot);
            status = d.trans_a ? copy_rows(dst, 4 * ald, a + r0, 4ull * d.lda, 4ull * pr, d.k,
                                           cudaMemcpyHostToDevice, st->in)
                               : copy_rows(dst, 4 * ald, a + static_cast<size_t>(r0) * d.lda, 4ull * d.lda,
                                           4ull * d.k, pr, cudaMemcpyHostToDevice, st->in);
            a_p = dst;
            a_ld = static_cast<long long>(ald);
        }
        float* c_p = c_dev ? c + static_cast<size_t>(r0) * d.ldc : reinterpret_cast<float*>(c_slots + slot * c_slot);
        if (status == MFB_OK && c_in)
            status = copy_rows(c_p, 4 * cld, c + static_cast<size_t>(r0) * d.ldc, 4ull * d.ldc, 4ull * d.n, pr,
                               cudaMemcpyHostToDevice, st->in);
        if (status == MFB_OK) status = cu(cudaEventRecord(st->ev_in[slot], st->in), "event record");
        // GEMM of the panel on the caller's stream
        if (status == MFB_OK) status = cu(cudaStreamWaitEvent(stream, st->ev_in[slot], 0), "stream wait");
        if (status != MFB_OK) break;
        if (pr == rc && full_panels && uses_ab) {
            status = mfb_plan_prepare(st->plan, stream_h, a_p, nullptr);
            if (status == MFB_OK)
                status = mfb_plan_multiply(st->plan, stream_h, a_p, b_d, c_p, d.alpha, d.beta, bias_d);
        } else {
            mfb_gemm_desc td = pd;
            td.m = pr;
            td.lda = static_cast<int>(a_ld);
            status = mfb_sgemm(device, stream_h, &td, a_p, b_d, c_p, bias_d);
        }
        if (status == MFB_OK) status = cu(cudaEventRecord(st->ev_gemm[slot], stream), "event record");
        // copy out
        if (status == MFB_OK) status = cu(cudaStreamWaitEvent(st->out, st->ev_gemm[slot], 0), "stream wait");
        if (status == MFB_OK && !c_dev)
            status = copy_rows(c + static_cast<size_t>(r0) * d.ldc, 4ull * d.ldc, c_p, 4 * cld, 4ull * d.n, pr,
                               cudaMemcpyDeviceToHost, st->out);
        if (status == MFB_OK) status = cu(cudaEventRecord(st->ev_out[slot], st->out), "event record");
    }
    // exit (also after an error, for what was queued): the caller's stream waits for the last
    // copy-out, and the next call waits for it before reusing the slots
    const mfb_status_t fin = cu(cudaEventRecord(st->done, st->out), "event record");
    st->pending = fin == MFB_OK;
    if (fin == MFB_OK) cudaStreamWaitEvent(stream, st->done, 0);
    if (status == MFB_OK && fin != MFB_OK) status = fin;
    return status;
}
