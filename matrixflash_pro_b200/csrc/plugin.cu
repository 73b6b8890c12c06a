// libmfb.so as a MatrixProPluginV1 backend (include/mfb_plugin.h): the table
// CreateMatrixProBackend returns drives devices through the CUDA runtime and runs every
// GEMM on this library's tcgen05 path (mfb_cuda_gemm + mfb_cuda_sync).
#include "mfb_plugin.h"
#include "mfb_internal.h"

#include <cstdio>
#include <mutex>
#include <string>

namespace mfb {
namespace {

void plugin_report(const char* what) { std::fprintf(stderr, "libmfb plugin: %s: %s\n", what, mfb_last_error()); }

void plugin_destroy(void*) {}

int plugin_device_count(void*) {
    int n = 0;
    return mfb_cuda_device_count(&n) == MFB_OK ? n : 0;
}

const char* plugin_device_name(void*, int index) {
    static std::mutex m;
    static std::string names[64];
    if (index < 0 || index >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(m);
    if (names[index].empty()) {
        cudaDeviceProp prop{};
        if (cudaGetDeviceProperties(&prop, index) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        names[index] = prop.name;
    }
    return names[index].c_str();
}

uint64_t plugin_memory_bytes(void*, int index) {
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, index) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return static_cast<uint64_t>(prop.totalGlobalMem);
}

void* plugin_allocate(void*, int index, size_t bytes) {
    clear_error();
    DeviceGuard guard;
    if (select_device(index) != MFB_OK) {
        plugin_report("allocate");
        return nullptr;
    }
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes < 4 ? 4 : bytes);  // the reference allocates at least one float
    if (e != cudaSuccess) {
        cudaGetLastError();
        cuda_fail(e, "plugin cudaMalloc");
        plugin_report("allocate");
        return nullptr;
    }
    return p;
}

void plugin_deallocate(void*, int index, void* pointer) {
    if (!pointer) return;
    DeviceGuard guard;
    if (cudaSetDevice(index) == cudaSuccess) cudaFree(pointer);
    cudaGetLastError();
}

void plugin_copy(void*, int dst_device, void* dst, int src_device, const void* src, size_t bytes) {
    clear_error();
    DeviceGuard guard;
    cudaError_t e = cudaMemcpyPeer(dst, dst_device, src, src_device, bytes);
    if (e == cudaSuccess && cudaSetDevice(dst_device) == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaGetLastError();
        cuda_fail(e, "plugin peer copy");
        plugin_report("copy");
    }
}

void plugin_gemm(void*, const mfb_plugin_gemm_args* a) {
    if (!a) return;
    if (mfb_cuda_gemm(a->device, a->m, a->n, a->k, a->a, a->lda, a->b, a->ldb, a->c, a->ldc, a->alpha, a->beta) !=
            MFB_OK ||
        mfb_cuda_sync(a->device) != MFB_OK)
        plugin_report("gemm");
}

mfb_plugin_v1 g_plugin = {1u,
                          1,  // DeviceType::Cuda
                          "b200-tcgen05",
                          nullptr,
                          plugin_destroy,
                          plugin_device_count,
                          plugin_device_name,
                          plugin_memory_bytes,
                          plugin_allocate,
                          plugin_deallocate,
                          plugin_copy,
                          plugin_gemm};

}  // namespace
}  // namespace mfb

extern "C" MFB_API mfb_plugin_v1* CreateMatrixProBackend(void) { return &mfb::g_plugin; }
