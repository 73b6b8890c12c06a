// mfb_sgemm_multi: the row-split GEMM over several GPUs of one process.
//
// C = epilogue(alpha * A * B + beta * C) with A and C split by rows into one block per GPU
// and B on one of them (the root). This is the multi-GPU form of the reference's row split
// between devices (HeterogeneousScheduler::gemm, src/hw/scheduler.cpp:238-312, which gives
// one CUDA device a block of rows and sends it B over PCIe), with B broadcast over
// NVLink/NVSwitch by NCCL instead of host-staged copies (src/hw/collectives.cpp:219-235).
//
// Schedule per call (the same one as matrixflash_pro_b200.distributed.RowSplitGemm, which
// runs one process per GPU):
//   * B travels in column panels: the root packs B[:, n0:n1] into a contiguous k x (n1 - n0)
//     buffer and every panel is an NCCL broadcast on the set's communication streams; a small
//     leading panel makes the first transfer, the only one not hidden, short, and for a large B
//     the panels after it double in width so each arrives during the previous panel's GEMM.
//   * Each GPU splits its A block into TF32 planes on its compute stream while B is in flight,
//     splits each panel into the plan's B planes on a second stream as soon as it has arrived,
//     and multiplies C[:, n0:n1] on the compute stream (mfb_plan_multiply_cols). GEMMs that
//     run while later panels are still broadcasting leave kCommSms SMs to NCCL: every panel but
//     the last at first, then only those whose GEMM started before the last panel had landed
//     in the previous call with the same schedule (timed events).
//   * Blocking: work already queued on the devices finishes first, and the call returns when
//     every GPU is done, like the reference's scheduler.
#include "mfb_internal.h"

#include <algorithm>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

namespace mfb {
namespace {

constexpr int kCommSms = 32;      // SMs left to NCCL while later panels are in flight
constexpr int kPanelTile = 256;   // panel widths are whole SM-pair tiles
constexpr int kMaxBlocks = 64;

// Column panels of B (the same schedule as matrixflash_pro_b200.distributed.col_panels): a
// leading panel of a tenth of the columns in whole 256-column tiles and at most 128 MB of B (its
// broadcast is the only one nothing hides); then, while the rest of B is over 512 MB and over four
// times the last panel, a panel twice as wide as the last (a panel's GEMM takes 2 * rows * k FLOP
// per column, its transfer 4 * k bytes, so a doubled panel arrives during the previous GEMM);
// then the rest. One panel without peers or for narrow B.
std::vector<std::pair<int, int>> col_panels(int n, int world, long long k) {
    std::vector<std::pair<int, int>> p;
    if (world <= 1 || n <= 2 * kPanelTile) {
        p.emplace_back(0, n);
        return p;
    }
    int first = std::max(kPanelTile, static_cast<int>(n * 0.1) / kPanelTile * kPanelTile);
    if (k > 0)
        first = std::min<long long>(first, std::max<long long>(kPanelTile, (128LL << 20) / (4 * k) / kPanelTile * kPanelTile));
    if (first >= n) {
        p.emplace_back(0, n);
        return p;
    }
    p.emplace_back(0, first);
    long long width = first, start = first;
    while (4 * k * (n - start) > (512LL << 20) && n - start > 4 * width) {
        width *= 2;
        p.emplace_back(static_cast<int>(start), static_cast<int>(start + width));
        start += width;
    }
    p.emplace_back(static_cast<int>(start), n);
    return p;
}

// Library-owned state of one device: a plan for the last shape, panel and bias buffers,
// a compute and a prepare stream, one event per panel.
struct DevState {
    int device = 0;
    mfb_plan_t plan = nullptr;
    mfb_gemm_desc plan_desc{};
    float* panels = nullptr;  // all panels back to back: panel [n0, n1) at panels + k * n0
    size_t panel_floats = 0;
    float* bias = nullptr;
    size_t bias_floats = 0;
    cudaStream_t compute = nullptr;
    cudaStream_t prepare = nullptr;
    std::vector<cudaEvent_t> arrived;   // per panel, on the communication stream
    std::vector<cudaEvent_t> prepared;  // per panel, on the prepare stream
    cudaEvent_t bias_ready = nullptr;
    // Adaptive SM cap (timed events): when the last panel landed, when each panel's GEMM started,
    // and which panels still leave SMs to NCCL, for the panel schedule of the last call.
    cudaEvent_t last_arrived = nullptr;
    std::vector<cudaEvent_t> gemm_start;
    std::vector<std::pair<int, int>> schedule;
    std::vector<char> capped;
    bool recorded = false;
};

// A panel's GEMM that started at least 50 us after the last panel landed (previous call) runs on
// every SM from now on; the others keep leaving kCommSms SMs to NCCL.
void update_caps(DevState& s) {
    if (!s.recorded || cudaEventQuery(s.last_arrived) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    for (size_t i = 0; i + 1 < s.schedule.size(); ++i) {
        float ms = 0.0f;
        if (s.capped[i] && cudaEventQuery(s.gemm_start[i]) == cudaSuccess &&
            cudaEventElapsedTime(&ms, s.gemm_start[i], s.last_arrived) == cudaSuccess && ms <= -0.05f)
            s.capped[i] = 0;
    }
    cudaGetLastError();
}

std::mutex g_multi_mutex;  // one call at a time: the per-device state is shared
std::map<int, std::unique_ptr<DevState>> g_states;

bool same_plan_shape(const mfb_gemm_desc& x, const mfb_gemm_desc& y) {
    return x.m == y.m && x.n == y.n && x.k == y.k && x.lda == y.lda && x.ldb == y.ldb && x.ldc == y.ldc &&
           x.precision == y.precision && x.trans_a == y.trans_a && x.trans_b == y.trans_b && x.epilogue == y.epilogue;
}

mfb_status_t grow(float** ptr, size_t* have, size_t floats) {
    if (*have >= floats) return MFB_OK;
    if (*ptr) {
        MFB_CUDA_TRY(cudaDeviceSynchronize(), "multi-GPU buffer resize sync");
        cudaFree(*ptr);
        *ptr = nullptr;
        *have = 0;
    }
    MFB_CUDA_TRY(cudaMalloc(ptr, floats * 4), "multi-GPU buffer cudaMalloc");
    *have = floats;
    return MFB_OK;
}

// The state of `device` (current) sized for `panels` panels, `k x n` of panel storage and
// `bias_n` floats of bias.
mfb_status_t device_state(int device, size_t panel_count, size_t b_floats, size_t bias_n, DevState** out) {
    auto& slot = g_states[device];
    if (!slot) {
        slot.reset(new DevState());
        slot->device = device;
        MFB_CUDA_TRY(cudaStreamCreateWithFlags(&slot->compute, cudaStreamNonBlocking), "multi-GPU compute stream");
        MFB_CUDA_TRY(cudaStreamCreateWithFlags(&slot->prepare, cudaStreamNonBlocking), "multi-GPU prepare stream");
        MFB_CUDA_TRY(cudaEventCreateWithFlags(&slot->bias_ready, cudaEventDisableTiming), "event");
        MFB_CUDA_TRY(cudaEventCreate(&slot->last_arrived), "event");
    }
    DevState* st = slot.get();
    while (st->arrived.size() < panel_count) {
        cudaEvent_t a = nullptr, p = nullptr, g = nullptr;
        MFB_CUDA_TRY(cudaEventCreateWithFlags(&a, cudaEventDisableTiming), "event");
        MFB_CUDA_TRY(cudaEventCreateWithFlags(&p, cudaEventDisableTiming), "event");
        MFB_CUDA_TRY(cudaEventCreate(&g), "event");
        st->arrived.push_back(a);
        st->prepared.push_back(p);
        st->gemm_start.push_back(g);
    }
    MFB_TRY(grow(&st->panels, &st->panel_floats, std::max<size_t>(b_floats, 1)));
    if (bias_n) MFB_TRY(grow(&st->bias, &st->bias_floats, bias_n));
    *out = st;
    return MFB_OK;
}

mfb_status_t device_plan(DevState* st, const mfb_gemm_desc& d) {
    if (st->plan && same_plan_shape(st->plan_desc, d)) return MFB_OK;
    if (st->plan) {
        MFB_CUDA_TRY(cudaDeviceSynchronize(), "multi-GPU plan replace sync");
        mfb_plan_destroy(st->plan);
        st->plan = nullptr;
    }
    MFB_TRY(mfb_plan_create(st->device, &d, &st->plan));
    st->plan_desc = d;
    return MFB_OK;
}

// Argument checks that need no device (the reference's validation: shapes, strides, options,
// pointers), then the devices themselves.
mfb_status_t check_args(const mfb_row_block* blocks, int count, int root, const mfb_gemm_desc* desc, const float* b,
                        const float* bias) {
    if (!blocks || count < 1 || count > kMaxBlocks) return fail(MFB_EINVAL, "mfb_sgemm_multi: 1 to 64 row blocks");
    if (root < 0 || root >= count) return fail(MFB_EINVAL, "mfb_sgemm_multi: root out of range");
    MFB_TRY(validate_desc(desc, nullptr, nullptr, nullptr, nullptr, false));
    const mfb_gemm_desc& d = *desc;
    if (d.trans_a || d.trans_b) return fail(MFB_EUNSUPPORTED, "mfb_sgemm_multi: the row split takes untransposed A and B");
    long long rows = 0;
    std::vector<int> devs;
    for (int r = 0; r < count; ++r) {
        const mfb_row_block& blk = blocks[r];
        if (blk.rows < 0) return fail(MFB_EINVAL, "mfb_sgemm_multi: negative row count");
        rows += blk.rows;
        if (blk.rows > 0 && d.n > 0) {
            if (!blk.c) return fail(MFB_EINVAL, "mfb_sgemm_multi: null C block");
            if (d.k > 0 && !blk.a) return fail(MFB_EINVAL, "mfb_sgemm_multi: null A block");
            if (blk.c == blk.a || blk.c == b) return fail(MFB_EINVAL, "GEMM output cannot alias an input");
        }
        devs.push_back(blk.device);
    }
    if (rows != d.m) return fail(MFB_ESHAPE, "mfb_sgemm_multi: the blocks' rows must add up to m");
    std::sort(devs.begin(), devs.end());
    if (std::adjacent_find(devs.begin(), devs.end()) != devs.end())
        return fail(MFB_EINVAL, "mfb_sgemm_multi: one row block per GPU (devices must be distinct)");
    if (d.m > 0 && d.n > 0 && d.k > 0 && !b) return fail(MFB_EINVAL, "null B pointer");
    if (d.epilogue != MFB_EPILOGUE_NONE && !bias) return fail(MFB_ESHAPE, "GEMM bias length must equal N");
    return MFB_OK;
}

mfb_status_t run_multi(const mfb_row_block* blocks, int count, int root, const mfb_gemm_desc& d, const float* b,
                       const float* bias) {
    std::vector<int> devices(count);
    for (int r = 0; r < count; ++r) {
        devices[r] = blocks[r].device;
        MFB_TRY(select_device(devices[r]));
        MFB_CUDA_TRY(cudaDeviceSynchronize(), "multi-GPU entry sync");  // blocking, like the reference
    }
    if (d.m == 0 || d.n == 0) return MFB_OK;
    const bool with_bias = d.epilogue != MFB_EPILOGUE_NONE;
    const auto panels = col_panels(d.n, count, d.k);
    const size_t b_floats = static_cast<size_t>(d.k) * static_cast<size_t>(d.n);
    std::vector<DevState*> st(count, nullptr);
    for (int r = 0; r < count; ++r) {
        MFB_CUDA_TRY(cudaSetDevice(devices[r]), "cudaSetDevice");
        MFB_TRY(device_state(devices[r], panels.size(), count > 1 ? b_floats : 0, with_bias ? d.n : 0, &st[r]));
        if (blocks[r].rows > 0) {
            mfb_gemm_desc pd = d;
            pd.m = blocks[r].rows;
            MFB_TRY(device_plan(st[r], pd));
        }
    }
    if (count == 1) {
        const mfb_row_block& blk = blocks[0];
        MFB_TRY(mfb_plan_execute(st[0]->plan, reinterpret_cast<mfb_stream_t>(st[0]->compute), blk.a, b, blk.c,
                                 d.alpha, d.beta, bias));
        MFB_CUDA_TRY(cudaStreamSynchronize(st[0]->compute), "multi-GPU sync");
        return read_and_clear_status(nullptr);
    }

    for (int r = 0; r < count; ++r) {
        DevState& s = *st[r];
        if (s.schedule != panels) {  // a new panel schedule: cap every panel but the last again
            s.schedule = panels;
            s.capped.assign(panels.size(), 1);
            s.capped.back() = 0;
            s.recorded = false;
        } else {
            update_caps(s);
        }
    }
    std::vector<cudaStream_t> comm;
    MFB_TRY(nccl_streams(devices, &comm));
    // Root: each panel packed contiguous on its communication stream, ahead of its broadcast.
    MFB_CUDA_TRY(cudaSetDevice(devices[root]), "cudaSetDevice");
    for (const auto& pn : panels) {
        const int w = pn.second - pn.first;
        MFB_CUDA_TRY(cudaMemcpy2DAsync(st[root]->panels + static_cast<size_t>(d.k) * pn.first, static_cast<size_t>(w) * 4,
                                       b + pn.first, static_cast<size_t>(d.ldb) * 4, static_cast<size_t>(w) * 4, d.k,
                                       cudaMemcpyDeviceToDevice, comm[root]),
                     "panel pack");
    }
    if (with_bias) {
        MFB_CUDA_TRY(cudaMemcpyAsync(st[root]->bias, bias, static_cast<size_t>(d.n) * 4, cudaMemcpyDeviceToDevice,
                                     comm[root]),
                     "bias copy");
        std::vector<float*> bufs(count);
        for (int r = 0; r < count; ++r) bufs[r] = st[r]->bias;
        MFB_TRY(nccl_broadcast_group(devices, bufs, static_cast<size_t>(d.n), root));
        for (int r = 0; r < count; ++r) {
            MFB_CUDA_TRY(cudaSetDevice(devices[r]), "cudaSetDevice");
            MFB_CUDA_TRY(cudaEventRecord(st[r]->bias_ready, comm[r]), "event record");
        }
    }
    for (size_t i = 0; i < panels.size(); ++i) {
        const size_t off = static_cast<size_t>(d.k) * panels[i].first;
        const size_t cnt = static_cast<size_t>(d.k) * (panels[i].second - panels[i].first);
        std::vector<float*> bufs(count);
        for (int r = 0; r < count; ++r) bufs[r] = st[r]->panels + off;
        MFB_TRY(nccl_broadcast_group(devices, bufs, cnt, root));
        for (int r = 0; r < count; ++r) {
            MFB_CUDA_TRY(cudaSetDevice(devices[r]), "cudaSetDevice");
            MFB_CUDA_TRY(cudaEventRecord(st[r]->arrived[i], comm[r]), "event record");
            if (i + 1 == panels.size()) MFB_CUDA_TRY(cudaEventRecord(st[r]->last_arrived, comm[r]), "event record");
        }
    }
    // Per GPU: A's planes while B is in flight, each panel's planes as it lands, its GEMM.
    for (int r = 0; r < count; ++r) {
        const mfb_row_block& blk = blocks[r];
        if (blk.rows == 0) continue;
        DevState& s = *st[r];
        MFB_CUDA_TRY(cudaSetDevice(devices[r]), "cudaSetDevice");
        const int sms = sm_count(devices[r]);
        mfb_stream_t cs = reinterpret_cast<mfb_stream_t>(s.compute);
        mfb_stream_t ps = reinterpret_cast<mfb_stream_t>(s.prepare);
        MFB_TRY(mfb_plan_prepare(s.plan, cs, blk.a, nullptr));
        for (size_t i = 0; i < panels.size(); ++i) {
            const int n0 = panels[i].first, n1 = panels[i].second;
            MFB_CUDA_TRY(cudaStreamWaitEvent(s.prepare, s.arrived[i], 0), "wait panel");
            MFB_TRY(mfb_plan_prepare_cols(s.plan, ps, s.panels + static_cast<size_t>(d.k) * n0, n1 - n0, n0, n1));
            MFB_CUDA_TRY(cudaEventRecord(s.prepared[i], s.prepare), "event record");
        }
        if (with_bias) MFB_CUDA_TRY(cudaStreamWaitEvent(s.compute, s.bias_ready, 0), "wait bias");
        for (size_t i = 0; i < panels.size(); ++i) {
            const int n0 = panels[i].first, n1 = panels[i].second;
            MFB_CUDA_TRY(cudaStreamWaitEvent(s.compute, s.prepared[i], 0), "wait planes");
            MFB_TRY(mfb_plan_set_sm_limit(s.plan, s.capped[i] ? std::max(1, sms - kCommSms) : 0));
            MFB_CUDA_TRY(cudaEventRecord(s.gemm_start[i], s.compute), "event record");
            MFB_TRY(mfb_plan_multiply_cols(s.plan, cs, blk.a, blk.c, d.alpha, d.beta, with_bias ? s.bias : nullptr,
                                           n0, n1));
        }
    }
    for (int r = 0; r < count; ++r) st[r]->recorded = true;
    mfb_status_t result = MFB_OK;
    for (int r = 0; r < count; ++r) {
        MFB_CUDA_TRY(cudaSetDevice(devices[r]), "cudaSetDevice");
        MFB_CUDA_TRY(cudaStreamSynchronize(comm[r]), "multi-GPU broadcast sync");
        MFB_CUDA_TRY(cudaStreamSynchronize(st[r]->prepare), "multi-GPU prepare sync");
        MFB_CUDA_TRY(cudaStreamSynchronize(st[r]->compute), "multi-GPU compute sync");
        const mfb_status_t s = read_and_clear_status(nullptr);
        if (result == MFB_OK) result = s;
    }
    return result;
}

}  // namespace
}  // namespace mfb

extern "C" MFB_API mfb_status_t mfb_sgemm_multi(const mfb_row_block* blocks, int block_count, int root,
                                                const mfb_gemm_desc* desc, const float* b, const float* bias) {
    using namespace mfb;
    clear_error();
    MFB_TRY(check_args(blocks, block_count, root, desc, b, bias));
    DeviceGuard guard;
    std::lock_guard<std::mutex> lock(g_multi_mutex);
    return run_multi(blocks, block_count, root, *desc, b, bias);
}
