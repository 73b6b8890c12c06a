// Collectives over an array of per-GPU buffers of one process, on NCCL over NVLink/NVSwitch.
//
// Replaces matrix_pro::all_reduce / broadcast / all_gather / reduce_scatter / scatter / gather
// (include/matrix_pro/distributed/collectives.hpp:27-32, src/hw/collectives.cpp:185-311), which
// download every rank's buffer to the host, combine there and upload again, and the stubbed
// hw::cuda_nccl_allreduce (src/hw/cuda_backend.cu:252). The results land in the same places the
// reference writes them (including reduce_scatter leaving the all-reduced tail behind each rank's
// chunk, and Mean as Sum times the float 1/ranks). Ranks on distinct GPUs run as one NCCL
// communicator per device set (ncclCommInitAll, created once and cached) with grouped calls on a
// stream per device; ranks that all sit on one GPU run device-local copies and a fixed-order
// reduction kernel. Every call is blocking, as in the reference: each device is synchronized
// before (so earlier work on its buffers has finished) and after.
//
// NCCL is opened at run time (dlopen "libnccl.so.2"): in a process that already loaded NCCL
// (e.g. through torch) the same library is used.
#include "mfb_internal.h"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

namespace mfb {
namespace {

struct NcclApi {
    ncclResult_t (*comm_init_all)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

const NcclApi& nccl_api() {
    static NcclApi api = [] {
        NcclApi a;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return a;
        a.comm_init_all = reinterpret_cast<decltype(a.comm_init_all)>(dlsym(h, "ncclCommInitAll"));
        a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
        a.broadcast = reinterpret_cast<decltype(a.broadcast)>(dlsym(h, "ncclBroadcast"));
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
        a.send = reinterpret_cast<decltype(a.send)>(dlsym(h, "ncclSend"));
        a.recv = reinterpret_cast<decltype(a.recv)>(dlsym(h, "ncclRecv"));
        a.group_start = reinterpret_cast<decltype(a.group_start)>(dlsym(h, "ncclGroupStart"));
        a.group_end = reinterpret_cast<decltype(a.group_end)>(dlsym(h, "ncclGroupEnd"));
        a.error_string = reinterpret_cast<decltype(a.error_string)>(dlsym(h, "ncclGetErrorString"));
        a.ok = a.comm_init_all && a.all_reduce && a.broadcast && a.all_gather && a.send && a.recv && a.group_start &&
               a.group_end;
        return a;
    }();
    return api;
}

#define MFB_NCCL_TRY(expr, what)                                                                             \
    do {                                                                                                     \
        ncclResult_t mfb_nr_ = (expr);                                                                       \
        if (mfb_nr_ != ncclSuccess)                                                                          \
            return fail(MFB_ENCCL, std::string(what) + ": " +                                                \
                                       (nccl_api().error_string ? nccl_api().error_string(mfb_nr_) : "error")); \
    } while (0)

// One communicator, stream and scratch buffer per device of a device set.
struct CommSet {
    std::vector<int> devices;
    std::vector<ncclComm_t> comms;
    std::vector<cudaStream_t> streams;
};

std::mutex g_comm_mutex;
std::map<std::vector<int>, std::unique_ptr<CommSet>> g_comms;

mfb_status_t comm_set(const std::vector<int>& devices, CommSet** out) {
    std::lock_guard<std::mutex> lock(g_comm_mutex);
    auto it = g_comms.find(devices);
    if (it != g_comms.end()) {
        *out = it->second.get();
        return MFB_OK;
    }
    const NcclApi& api = nccl_api();
    if (!api.ok) return fail(MFB_ENCCL, "libnccl.so.2 could not be opened");
    auto set = std::make_unique<CommSet>();
    set->devices = devices;
    set->comms.resize(devices.size());
    MFB_NCCL_TRY(api.comm_init_all(set->comms.data(), static_cast<int>(devices.size()), devices.data()),
                 "ncclCommInitAll");
    for (int dev : devices) {
        MFB_CUDA_TRY(cudaSetDevice(dev), "cudaSetDevice");
        cudaStream_t s = nullptr;
        MFB_CUDA_TRY(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "collective stream");
        set->streams.push_back(s);
    }
    *out = set.get();
    g_comms[devices] = std::move(set);
    return MFB_OK;
}

// ------------------------------------------------------------------------------ device-local kernels
constexpr int kLocalMaxRanks = 64;

struct RankPtrs {
    float* p[kLocalMaxRanks];
};

// out[i] = op over ranks (in rank order) of in_r[i]; op 2 = max, otherwise sum.
__global__ void local_reduce_kernel(RankPtrs in, int ranks, size_t count, int op, float* __restrict__ out) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        float acc = in.p[0][i];
        for (int r = 1; r < ranks; ++r) acc = op == 2 ? fmaxf(acc, in.p[r][i]) : acc + in.p[r][i];
        out[i] = acc;
    }
}

__global__ void scale_kernel(float* __restrict__ p, size_t count, float factor) {
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        p[i] *= factor;
}

int grid_for(size_t count) { return static_cast<int>(std::min<size_t>((count + 255) / 256, static_cast<size_t>(current_sm_count()) * 8)); }

// ------------------------------------------------------------------------------ common checks
struct Plan {
    int n = 0;
    std::vector<int> devices;
    bool distinct = false;  // one rank per GPU: NCCL
    bool local = false;     // every rank on one GPU: device-local
};

mfb_status_t plan_ranks(const mfb_collective_buffer* ranks, int n, Plan* plan) {
    if (!ranks || n <= 0) return fail(MFB_EINVAL, "collective: no ranks");
    int dev_count = 0;
    MFB_CUDA_TRY(cudaGetDeviceCount(&dev_count), "cudaGetDeviceCount");
    plan->n = n;
    plan->devices.resize(n);
    for (int r = 0; r < n; ++r) {
        if (ranks[r].device < 0 || ranks[r].device >= dev_count)
            return fail(MFB_EINVAL, "collective: CUDA device index out of range");
        if (ranks[r].count > 0 && !ranks[r].data) return fail(MFB_EINVAL, "collective: null buffer");
        plan->devices[r] = ranks[r].device;
        MFB_TRY(select_device(ranks[r].device));
    }
    std::vector<int> sorted = plan->devices;
    std::sort(sorted.begin(), sorted.end());
    plan->distinct = std::adjacent_find(sorted.begin(), sorted.end()) == sorted.end();
    plan->local = sorted.front() == sorted.back();
    if (!plan->distinct && !plan->local)
        return fail(MFB_EUNSUPPORTED, "collective: ranks must sit on distinct GPUs or all on one GPU");
    if (plan->local && n > kLocalMaxRanks) return fail(MFB_EUNSUPPORTED, "collective: too many ranks on one GPU");
    // Blocking semantics: work already queued on the buffers' devices finishes first.
    for (int r = 0; r < n; ++r) {
        MFB_CUDA_TRY(cudaSetDevice(plan->devices[r]), "cudaSetDevice");
        MFB_CUDA_TRY(cudaDeviceSynchronize(), "collective entry sync");
    }
    return MFB_OK;
}

mfb_status_t finish(const Plan& plan, CommSet* set) {
    for (int r = 0; r < plan.n; ++r) {
        MFB_CUDA_TRY(cudaSetDevice(plan.devices[r]), "cudaSetDevice");
        if (set)
            MFB_CUDA_TRY(cudaStreamSynchronize(set->streams[r]), "collective sync");
        else
            MFB_CUDA_TRY(cudaDeviceSynchronize(), "collective sync");
        if (plan.local) break;
    }
    return MFB_OK;
}

// Scratch on a device for the local path / the NCCL staging copies.
mfb_status_t scratch(int device, cudaStream_t stream, size_t floats, float** out) {
    void* p = nullptr;
    MFB_TRY(stream_workspace(device, stream, floats * 4, &p));
    *out = static_cast<float*>(p);
    return MFB_OK;
}

mfb_status_t copy_d2d(float* dst, const float* src, size_t count, cudaStream_t stream) {
    if (count == 0 || dst == src) return MFB_OK;
    MFB_CUDA_TRY(cudaMemcpyAsync(dst, src, count * 4, cudaMemcpyDeviceToDevice, stream), "collective copy");
    return MFB_OK;
}

// Sum / Mean / Max of equal-length buffers into every buffer. Mean = Sum * (1/ranks).
mfb_status_t all_reduce_impl(const mfb_collective_buffer* ranks, int n, int op) {
    if (op < 0 || op > 2) return fail(MFB_EINVAL, "collective: unknown reduce op");
    Plan plan;
    MFB_TRY(plan_ranks(ranks, n, &plan));
    const size_t count = ranks[0].count;
    for (int r = 1; r < n; ++r)
        if (ranks[r].count != count) return fail(MFB_EINVAL, "all_reduce: rank lengths differ");
    if (n == 1 || count == 0) return MFB_OK;
    if (plan.local) {
        MFB_CUDA_TRY(cudaSetDevice(plan.devices[0]), "cudaSetDevice");
        float* tmp = nullptr;
        MFB_TRY(scratch(plan.devices[0], nullptr, count, &tmp));
        RankPtrs in{};
        for (int r = 0; r < n; ++r) in.p[r] = ranks[r].data;
        local_reduce_kernel<<<grid_for(count), 256>>>(in, n, count, op, tmp);
        MFB_CUDA_TRY(cudaGetLastError(), "local reduce launch");
        if (op == 1) scale_kernel<<<grid_for(count), 256>>>(tmp, count, 1.0f / static_cast<float>(n));
        for (int r = 0; r < n; ++r) MFB_TRY(copy_d2d(ranks[r].data, tmp, count, nullptr));
        return finish(plan, nullptr);
    }
    CommSet* set = nullptr;
    MFB_TRY(comm_set(plan.devices, &set));
    const NcclApi& api = nccl_api();
    MFB_NCCL_TRY(api.group_start(), "ncclGroupStart");
    for (int r = 0; r < n; ++r) {
        cudaSetDevice(plan.devices[r]);
        MFB_NCCL_TRY(api.all_reduce(ranks[r].data, ranks[r].data, count, ncclFloat, op == 2 ? ncclMax : ncclSum,
                                    set->comms[r], set->streams[r]),
                     "ncclAllReduce");
    }
    MFB_NCCL_TRY(api.group_end(), "ncclGroupEnd");
    if (op == 1)
        for (int r = 0; r < n; ++r) {
            MFB_CUDA_TRY(cudaSetDevice(plan.devices[r]), "cudaSetDevice");
            scale_kernel<<<grid_for(count), 256, 0, set->streams[r]>>>(ranks[r].data, count,
                                                                       1.0f / static_cast<float>(n));
        }
    return finish(plan, set);
}

}  // namespace

mfb_status_t nccl_streams(const std::vector<int>& devices, std::vector<cudaStream_t>* streams) {
    CommSet* set = nullptr;
    MFB_TRY(comm_set(devices, &set));
    *streams = set->streams;
    return MFB_OK;
}

mfb_status_t nccl_broadcast_group(const std::vector<int>& devices, const std::vector<float*>& bufs, size_t count,
                                  int root) {
    CommSet* set = nullptr;
    MFB_TRY(comm_set(devices, &set));
    if (bufs.size() != devices.size() || root < 0 || root >= static_cast<int>(devices.size()))
        return fail(MFB_EINVAL, "broadcast group: one buffer per device and a root among them");
    const NcclApi& api = nccl_api();
    MFB_NCCL_TRY(api.group_start(), "ncclGroupStart");
    for (size_t r = 0; r < devices.size(); ++r) {
        cudaSetDevice(devices[r]);
        MFB_NCCL_TRY(api.broadcast(bufs[r], bufs[r], count, ncclFloat, root, set->comms[r], set->streams[r]),
                     "ncclBroadcast");
    }
    MFB_NCCL_TRY(api.group_end(), "ncclGroupEnd");
    return MFB_OK;
}

}  // namespace mfb

using namespace mfb;

extern "C" {

MFB_API mfb_status_t mfb_all_reduce(const mfb_collective_buffer* ranks, int rank_count, int op, int algorithm) {
    clear_error();
    if (algorithm != 0 && algorithm != 1) return fail(MFB_EINVAL, "collective: unknown algorithm");
    DeviceGuard guard;
    return all_reduce_impl(ranks, rank_count, op);
}

MFB_API mfb_status_t mfb_broadcast(const mfb_collective_buffer* ranks, int rank_count, int root) {
    clear_error();
    DeviceGuard guard;
    Plan plan;
    MFB_TRY(plan_ranks(ranks, rank_count, &plan));
    if (root < 0 || root >= rank_count) return fail(MFB_EINVAL, "broadcast: root out of range");
    const size_t count = ranks[root].count;
    for (int r = 0; r < rank_count; ++r)
        if (ranks[r].count != count) return fail(MFB_EINVAL, "broadcast: rank lengths differ");
    if (rank_count == 1 || count == 0) return MFB_OK;
    if (plan.local) {
        MFB_CUDA_TRY(cudaSetDevice(plan.devices[0]), "cudaSetDevice");
        for (int r = 0; r < rank_count; ++r)
            if (r != root) MFB_TRY(copy_d2d(ranks[r].data, ranks[root].data, count, nullptr));
        return finish(plan, nullptr);
    }
    CommSet* set = nullptr;
    MFB_TRY(comm_set(plan.devices, &set));
    const NcclApi& api = nccl_api();
    MFB_NCCL_TRY(api.group_start(), "ncclGroupStart");
    for (int r = 0; r < rank_count; ++r) {
        cudaSetDevice(plan.devices[r]);
        MFB_NCCL_TRY(api.broadcast(ranks[r].data, ranks[r].data, count, ncclFloat, root, set->comms[r],
                                   set->streams[r]),
                     "ncclBroadcast");
    }
    MFB_NCCL_TRY(api.group_end(), "ncclGroupEnd");
    return finish(plan, set);
}

MFB_API mfb_status_t mfb_all_gather(const mfb_collective_buffer* ranks, int rank_count, size_t count_per_rank) {
    clear_error();
    DeviceGuard guard;
    Plan plan;
    MFB_TRY(plan_ranks(ranks, rank_count, &plan));
    const size_t full = count_per_rank * static_cast<size_t>(rank_count);
    for (int r = 0; r < rank_count; ++r)
        if (ranks[r].count < full) return fail(MFB_EINVAL, "all_gather: buffer shorter than rank_count * count");
    if (count_per_rank == 0) return MFB_OK;
    if (plan.local) {
        MFB_CUDA_TRY(cudaSetDevice(plan.devices[0]), "cudaSetDevice");
        float* tmp = nullptr;
        MFB_TRY(scratch(plan.devices[0], nullptr, full, &tmp));
        for (int r = 0; r < rank_count; ++r)
            MFB_TRY(copy_d2d(tmp + static_cast<size_t>(r) * count_per_rank, ranks[r].data, count_per_rank, nullptr));
        for (int r = 0; r < rank_count; ++r) MFB_TRY(copy_d2d(ranks[r].data, tmp, full, nullptr));
        return finish(plan, nullptr);
    }
    CommSet* set = nullptr;
    MFB_TRY(comm_set(plan.devices, &set));
    std::vector<float*> send(rank_count);
    for (int r = 0; r < rank_count; ++r) {  // each rank's contribution leaves its buffer before the gather
        MFB_CUDA_TRY(cudaSetDevice(plan.devices[r]), "cudaSetDevice");
        MFB_TRY(scratch(plan.devices[r], set->streams[r], count_per_rank, &send[r]));
        MFB_TRY(copy_d2d(send[r], ranks[r].data, count_per_rank, set->streams[r]));
    }
    const NcclApi& api = nccl_api();
    MFB_NCCL_TRY(api.group_start(), "ncclGroupStart");
    for (int r = 0; r < rank_count; ++r) {
        cudaSetDevice(plan.devices[r]);
        MFB_NCCL_TRY(api.all_gather(send[r], ranks[r].data, count_per_rank, ncclFloat, set->comms[r], set->streams[r]),
                     "ncclAllGather");
    }
    MFB_NCCL_TRY(api.group_end(), "ncclGroupEnd");
    return finish(plan, set);
}

MFB_API mfb_status_t mfb_reduce_scatter(const mfb_collective_buffer* ranks, int rank_count, int op) {
    clear_error();
    if (op < 0 || op > 2) return fail(MFB_EINVAL, "collective: unknown reduce op");
    if (!ranks || rank_count <= 0) return fail(MFB_EINVAL, "collective: no ranks");
    if (ranks[0].count % static_cast<size_t>(rank_count) != 0)
        return fail(MFB_EINVAL, "reduce_scatter: length must be divisible by rank count");
    DeviceGuard guard;
    // All-reduce in place (Sum for Mean), then each rank's chunk to the front of its buffer; Mean
    // scales that chunk only, as the reference does.
    MFB_TRY(all_reduce_impl(ranks, rank_count, op == 1 ? 0 : op));
    const size_t chunk = ranks[0].count / static_cast<size_t>(rank_count);
    for (int r = 0; r < rank_count; ++r) {
        MFB_CUDA_TRY(cudaSetDevice(ranks[r].device), "cudaSetDevice");
        MFB_TRY(copy_d2d(ranks[r].data, ranks[r].data + static_cast<size_t>(r) * chunk, chunk, nullptr));
        if (op == 1 && chunk > 0)
            scale_kernel<<<grid_for(chunk), 256>>>(ranks[r].data, chunk, 1.0f / static_cast<float>(rank_count));
        MFB_CUDA_TRY(cudaDeviceSynchronize(), "reduce_scatter sync");
    }
    return MFB_OK;
}

MFB_API mfb_status_t mfb_scatter(const mfb_collective_buffer* ranks, int rank_count, int root, size_t count_per_rank) {
    clear_error();
    DeviceGuard guard;
    Plan plan;
    MFB_TRY(plan_ranks(ranks, rank_count, &plan));
    if (root < 0 || root >= rank_count) return fail(MFB_EINVAL, "scatter: root out of range");
    const size_t full = count_per_rank * static_cast<size_t>(rank_count);
    if (ranks[root].count < full) return fail(MFB_EINVAL, "scatter: root buffer is too small");
    for (int r = 0; r < rank_count; ++r)
        if (ranks[r].count < count_per_rank) return fail(MFB_EINVAL, "scatter: rank buffer is too small");
    if (count_per_rank == 0) return MFB_OK;
    // The root's chunks are staged first: the root's own buffer is also a destination.
    if (plan.local) {
        MFB_CUDA_TRY(cudaSetDevice(plan.devices[0]), "cudaSetDevice");
        float* tmp = nullptr;
        MFB_TRY(scratch(plan.devices[0], nullptr, full, &tmp));
        MFB_TRY(copy_d2d(tmp, ranks[root].data, full, nullptr));
        for (int r = 0; r < rank_count; ++r)
            MFB_TRY(copy_d2d(ranks[r].data, tmp + static_cast<size_t>(r) * count_per_rank, count_per_rank, nullptr));
        return finish(plan, nullptr);
    }
    CommSet* set = nullptr;
    MFB_TRY(comm_set(plan.devices, &set));
    MFB_CUDA_TRY(cudaSetDevice(plan.devices[root]), "cudaSetDevice");
    float* staged = nullptr;
    MFB_TRY(scratch(plan.devices[root], set->streams[root], full, &staged));
    MFB_TRY(copy_d2d(staged, ranks[root].data, full, set->streams[root]));
    const NcclApi& api = nccl_api();
    MFB_NCCL_TRY(api.group_start(), "ncclGroupStart");
    for (int r = 0; r < rank_count; ++r) {
        if (r == root) continue;
        cudaSetDevice(plan.devices[root]);
        MFB_NCCL_TRY(api.send(staged + static_cast<size_t>(r) * count_per_rank, count_per_rank, ncclFloat, r,
                              set->comms[root], set->streams[root]),
                     "ncclSend");
        cudaSetDevice(plan.devices[r]);
        MFB_NCCL_TRY(api.recv(ranks[r].data, count_per_rank, ncclFloat, root, set->comms[r], set->streams[r]),
                     "ncclRecv");
    }
    MFB_NCCL_TRY(api.group_end(), "ncclGroupEnd");
    MFB_CUDA_TRY(cudaSetDevice(plan.devices[root]), "cudaSetDevice");
    MFB_TRY(copy_d2d(ranks[root].data, staged + static_cast<size_t>(root) * count_per_rank, count_per_rank,
                     set->streams[root]));
    return finish(plan, set);
}

MFB_API mfb_status_t mfb_gather(const mfb_collective_buffer* ranks, int rank_count, int root, size_t count_per_rank) {
    clear_error();
    DeviceGuard guard;
    Plan plan;
    MFB_TRY(plan_ranks(ranks, rank_count, &plan));
    if (root < 0 || root >= rank_count) return fail(MFB_EINVAL, "gather: root out of range");
    const size_t full = count_per_rank * static_cast<size_t>(rank_count);
    if (ranks[root].count < full) return fail(MFB_EINVAL, "gather: root buffer is too small");
    for (int r = 0; r < rank_count; ++r)
        if (ranks[r].count < count_per_rank) return fail(MFB_EINVAL, "gather: rank buffer is too small");
    if (count_per_rank == 0) return MFB_OK;
    if (plan.local) {
        MFB_CUDA_TRY(cudaSetDevice(plan.devices[0]), "cudaSetDevice");
        float* tmp = nullptr;
        MFB_TRY(scratch(plan.devices[0], nullptr, full, &tmp));
        for (int r = 0; r < rank_count; ++r)
            MFB_TRY(copy_d2d(tmp + static_cast<size_t>(r) * count_per_rank, ranks[r].data, count_per_rank, nullptr));
        MFB_TRY(copy_d2d(ranks[root].data, tmp, full, nullptr));
        return finish(plan, nullptr);
    }
    CommSet* set = nullptr;
    MFB_TRY(comm_set(plan.devices, &set));
    // The root's own chunk is saved first: other ranks' chunks may land on top of it.
    MFB_CUDA_TRY(cudaSetDevice(plan.devices[root]), "cudaSetDevice");
    float* own = nullptr;
    MFB_TRY(scratch(plan.devices[root], set->streams[root], count_per_rank, &own));
    MFB_TRY(copy_d2d(own, ranks[root].data, count_per_rank, set->streams[root]));
    const NcclApi& api = nccl_api();
    MFB_NCCL_TRY(api.group_start(), "ncclGroupStart");
    for (int r = 0; r < rank_count; ++r) {
        if (r == root) continue;
        cudaSetDevice(plan.devices[r]);
        MFB_NCCL_TRY(api.send(ranks[r].data, count_per_rank, ncclFloat, root, set->comms[r], set->streams[r]),
                     "ncclSend");
        cudaSetDevice(plan.devices[root]);
        MFB_NCCL_TRY(api.recv(ranks[root].data + static_cast<size_t>(r) * count_per_rank, count_per_rank, ncclFloat,
                              r, set->comms[root], set->streams[root]),
                     "ncclRecv");
    }
    MFB_NCCL_TRY(api.group_end(), "ncclGroupEnd");
    MFB_CUDA_TRY(cudaSetDevice(plan.devices[root]), "cudaSetDevice");
    MFB_TRY(copy_d2d(ranks[root].data + static_cast<size_t>(root) * count_per_rank, own, count_per_rank,
                     set->streams[root]));
    return finish(plan, set);
}

MFB_API mfb_status_t mfb_cuda_nccl_allreduce(float** ptrs, const int* devices, int rank_count, size_t count,
                                             int reduce_op) {
    clear_error();
    if (!ptrs || !devices || rank_count <= 0) return fail(MFB_EINVAL, "collective: no ranks");
    std::vector<mfb_collective_buffer> ranks(static_cast<size_t>(rank_count));
    for (int r = 0; r < rank_count; ++r) ranks[r] = mfb_collective_buffer{ptrs[r], count, devices[r]};
    DeviceGuard guard;
    return all_reduce_impl(ranks.data(), rank_count, reduce_op);
}

}  // extern "C"
