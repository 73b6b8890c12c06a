// The reference-side binding of hw::cuda_gemm, compiled as a stand-alone program:
// matrix_pro::hw::cuda_gemm / cuda_sync (include/matrix_pro/detail/cuda_hooks.hpp:17-18,28)
// implemented over libmfb.so's C ABI, then exercised the way CudaDriver::gemm
// (src/hw/cuda_backend.cu:274-277) uses them. Exit code 0 = all checks passed.
#include "mfb.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

namespace matrix_pro {
// Same name and base as include/matrix_pro/core/errors.hpp:8.
class MatrixProError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};

namespace hw {
namespace {
void check_mfb(mfb_status_t st, const char* what) {
    if (st != MFB_OK) throw MatrixProError(std::string(what) + ": " + mfb_last_error());
}
}  // namespace

void cuda_gemm(int device, int m, int n, int k, const float* a, int lda, const float* b, int ldb, float* c, int ldc,
               float alpha, float beta) {
    check_mfb(mfb_cuda_gemm(device, m, n, k, a, lda, b, ldb, c, ldc, alpha, beta), "cuda_gemm");
}

void cuda_sync(int device) { check_mfb(mfb_cuda_sync(device), "cudaStreamSynchronize"); }
}  // namespace hw
}  // namespace matrix_pro

namespace {
int failures = 0;
void check(bool ok, const char* what) {
    std::printf("%s %s\n", ok ? "[PASS]" : "[FAIL]", what);
    if (!ok) ++failures;
}

float lcg(unsigned& s) {
    s = s * 1664525u + 1013904223u;
    return static_cast<float>((s >> 8) & 0xFFFF) / 32768.0f - 1.0f;
}
}  // namespace

int main() {
    const int m = 300, n = 257, k = 513, lda = 520, ldb = 260, ldc = 264;
    std::vector<float> a(static_cast<size_t>(m) * lda), b(static_cast<size_t>(k) * ldb), c(static_cast<size_t>(m) * ldc);
    unsigned seed = 20261001u;
    for (auto& v : a) v = lcg(seed);
    for (auto& v : b) v = lcg(seed);
    for (auto& v : c) v = lcg(seed);
    float *da = nullptr, *db = nullptr, *dc = nullptr;
    if (cudaMalloc(&da, a.size() * 4) || cudaMalloc(&db, b.size() * 4) || cudaMalloc(&dc, c.size() * 4)) {
        std::printf("cudaMalloc failed\n");
        return 2;
    }
    cudaMemcpy(da, a.data(), a.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(db, b.data(), b.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dc, c.data(), c.size() * 4, cudaMemcpyHostToDevice);
    try {
        matrix_pro::hw::cuda_gemm(0, m, n, k, da, lda, db, ldb, dc, ldc, 0.5f, 1.0f);
        matrix_pro::hw::cuda_sync(0);
    } catch (const std::exception& e) {
        std::printf("unexpected exception: %s\n", e.what());
        return 1;
    }
    std::vector<float> out(c.size());
    cudaMemcpy(out.data(), dc, out.size() * 4, cudaMemcpyDeviceToHost);
    double num = 0, den = 0;
    bool pad_ok = true;
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            double ref = 0;
            for (int p = 0; p < k; ++p) ref += double(a[size_t(i) * lda + p]) * double(b[size_t(p) * ldb + j]);
            ref = 0.5 * ref + double(c[size_t(i) * ldc + j]);
            const double d = double(out[size_t(i) * ldc + j]) - ref;
            num += d * d;
            den += ref * ref;
        }
        for (int j = n; j < ldc; ++j) pad_ok = pad_ok && out[size_t(i) * ldc + j] == c[size_t(i) * ldc + j];
    }
    const double err = std::sqrt(num / den);
    std::printf("normwise error vs FP64: %.3e\n", err);
    check(err <= 1e-6, "cuda_gemm strict FP32 within 1e-6 of FP64");
    check(pad_ok, "cuda_gemm leaves row padding of C untouched");

    bool threw = false;
    try {
        matrix_pro::hw::cuda_gemm(4096, m, n, k, da, lda, db, ldb, dc, ldc, 1.0f, 0.0f);
    } catch (const matrix_pro::MatrixProError& e) {
        threw = std::string(e.what()).find("out of range") != std::string::npos;
    }
    check(threw, "bad device index throws MatrixProError (cuda_backend.cu:40-56)");
    threw = false;
    try {
        matrix_pro::hw::cuda_gemm(0, m, n, k, da, k - 1, db, ldb, dc, ldc, 1.0f, 0.0f);
    } catch (const matrix_pro::MatrixProError&) {
        threw = true;
    }
    check(threw, "lda < k throws MatrixProError");
    cudaFree(da);
    cudaFree(db);
    cudaFree(dc);
    std::printf("%d failure(s)\n", failures);
    return failures == 0 ? 0 : 1;
}
