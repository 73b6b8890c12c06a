// Loads libmfb.so the way the reference's BackendRegistry::load_plugin does
// (src/hw/backend_registry.cpp:252-266: dlopen, CreateMatrixProBackend, ABI check) and drives
// the returned table as PluginBackend would: allocate, gemm, deallocate. Exit code 0 = all
// checks passed. Usage: plugin_host <path to libmfb.so>
#include "mfb_plugin.h"

#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

namespace {
int failures = 0;
void check(bool ok, const char* what) {
    std::printf("%s: %s\n", ok ? "ok  " : "FAIL", what);
    if (!ok) ++failures;
}
}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    void* module = dlopen(argv[1], RTLD_NOW | RTLD_LOCAL);
    check(module != nullptr, "dlopen");
    if (!module) return 1;
    using CreateFn = mfb_plugin_v1* (*)();
    auto create = reinterpret_cast<CreateFn>(dlsym(module, "CreateMatrixProBackend"));
    check(create != nullptr, "CreateMatrixProBackend exported");
    if (!create) return 1;
    mfb_plugin_v1 table = *create();  // PluginBackend copies the table
    check(table.abi == 1 && table.gemm != nullptr && table.device_count != nullptr, "ABI version 1 table");
    check(table.device_type == 1, "device type Cuda");
    const int devices = table.device_count(table.user);
    check(devices >= 1, "at least one device");
    const char* name = table.device_name(table.user, 0);
    check(name != nullptr && std::strlen(name) > 0, "device name");
    check(table.memory_bytes(table.user, 0) > (1ull << 30), "memory size");

    // 300 x 520 x 700, padded rows, alpha 0.5, beta -1 (CudaDriver::gemm's contract)
    const int m = 300, n = 520, k = 700, lda = 704, ldb = 524, ldc = 528;
    std::vector<float> a(static_cast<size_t>(m) * lda), b(static_cast<size_t>(k) * ldb), c(static_cast<size_t>(m) * ldc);
    unsigned s = 12345u;
    auto rnd = [&s]() {
        s = s * 1664525u + 1013904223u;
        return static_cast<float>(static_cast<int>(s >> 8) % 2001 - 1000) / 1000.0f;
    };
    for (auto& v : a) v = rnd();
    for (auto& v : b) v = rnd();
    for (auto& v : c) v = rnd();
    const size_t bytes_a = a.size() * 4, bytes_b = b.size() * 4, bytes_c = c.size() * 4;
    float* da = static_cast<float*>(table.allocate(table.user, 0, bytes_a));
    float* db = static_cast<float*>(table.allocate(table.user, 0, bytes_b));
    float* dc = static_cast<float*>(table.allocate(table.user, 0, bytes_c));
    check(da && db && dc, "allocate");
    if (!da || !db || !dc) return 1;
    cudaMemcpy(da, a.data(), bytes_a, cudaMemcpyHostToDevice);
    cudaMemcpy(db, b.data(), bytes_b, cudaMemcpyHostToDevice);
    cudaMemcpy(dc, c.data(), bytes_c, cudaMemcpyHostToDevice);
    mfb_plugin_gemm_args args;
    std::memset(&args, 0, sizeof(args));
    args.device = 0;
    args.m = m;
    args.n = n;
    args.k = k;
    args.a = da;
    args.lda = lda;
    args.b = db;
    args.ldb = ldb;
    args.c = dc;
    args.ldc = ldc;
    args.alpha = 0.5f;
    args.beta = -1.0f;
    table.gemm(table.user, &args);  // synchronous, as CudaDriver::gemm
    // a device-to-device copy through the table, then back to the host
    float* dcopy = static_cast<float*>(table.allocate(table.user, 0, bytes_c));
    table.copy(table.user, 0, dcopy, 0, dc, bytes_c);
    std::vector<float> got(c.size());
    cudaMemcpy(got.data(), dcopy, bytes_c, cudaMemcpyDeviceToHost);
    double num = 0.0, den = 0.0;
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            double ref = 0.0;
            for (int p = 0; p < k; ++p) ref += static_cast<double>(a[i * lda + p]) * b[p * ldb + j];
            ref = 0.5 * ref - static_cast<double>(c[i * ldc + j]);
            const double d = got[i * ldc + j] - ref;
            num += d * d;
            den += ref * ref;
        }
    const double err = std::sqrt(num / den);
    std::printf("normwise error vs FP64: %.3e\n", err);
    check(err <= 1e-6, "strict FP32 result through the plugin table");
    table.deallocate(table.user, 0, da);
    table.deallocate(table.user, 0, db);
    table.deallocate(table.user, 0, dc);
    table.deallocate(table.user, 0, dcopy);
    table.destroy(table.user);
    std::printf("%d failure(s)\n", failures);
    return failures == 0 ? 0 : 1;
}
