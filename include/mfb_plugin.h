/*
 * mfb_plugin.h — libmfb.so as a plugin of the reference's backend registry.
 *
 * The reference loads accelerator plugins with BackendRegistry::load_plugin(path)
 * (src/hw/backend_registry.cpp:252-266): dlopen, look up CreateMatrixProBackend, take the
 * returned function table (MatrixProPluginV1, include/matrix_pro/core/backend_registry.hpp:
 * 60-94, ABI version 1) and wrap it in a PluginBackend. The two structs below have the
 * reference's member order and types, so the table libmfb.so returns is read as a
 * MatrixProPluginV1 by the unmodified reference. device_type is 1 (DeviceType::Cuda,
 * include/matrix_pro/core/device.hpp:21-23); gemm runs mfb_cuda_gemm then mfb_cuda_sync,
 * the two calls of the reference's own CudaDriver::gemm (src/hw/cuda_backend.cu:274-277),
 * and copy is a peer copy followed by a device sync, as CudaDriver::copy (:269-273).
 * The plugin ABI returns nothing from its calls: a failed call prints the library's last
 * error to stderr and leaves the output untouched.
 */
#ifndef MFB_PLUGIN_H_
#define MFB_PLUGIN_H_

#include <stddef.h>
#include <stdint.h>

#include "mfb.h"

#ifdef __cplusplus
extern "C" {
#endif

/* PluginGemmArgs (backend_registry.hpp:63-76): row-major C = alpha * A * B + beta * C on `device`. */
typedef struct mfb_plugin_gemm_args {
    int device;
    int m, n, k;
    const float* a;
    int lda;
    const float* b;
    int ldb;
    float* c;
    int ldc;
    float alpha, beta;
} mfb_plugin_gemm_args;

/* MatrixProPluginV1 (backend_registry.hpp:79-92). */
typedef struct mfb_plugin_v1 {
    uint32_t abi;
    int device_type;
    const char* name;
    void* user;
    void (*destroy)(void* user);
    int (*device_count)(void* user);
    const char* (*device_name)(void* user, int index);
    uint64_t (*memory_bytes)(void* user, int index);
    void* (*allocate)(void* user, int index, size_t bytes);
    void (*deallocate)(void* user, int index, void* pointer);
    void (*copy)(void* user, int dst_device, void* dst, int src_device, const void* src, size_t bytes);
    void (*gemm)(void* user, const mfb_plugin_gemm_args* args);
} mfb_plugin_v1;

/* The symbol BackendRegistry::load_plugin looks up. Returns a process-wide table. */
MFB_API mfb_plugin_v1* CreateMatrixProBackend(void);

#ifdef __cplusplus
}
#endif

#endif /* MFB_PLUGIN_H_ */
