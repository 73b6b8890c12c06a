// Test infrastructure only (oracle): a C-ABI wrapper around the reference's own
// CPU GEMM, compiled together with the reference's unmodified sources
// (src/hw/gemm.cpp, gemm_avx2.cpp, gemm_scalar.cpp, gemm_avx512.cpp,
// thread_pool.cpp, cpuid.cpp) into oracle/_ref/libmfref_cpu.so by oracle/Makefile.
// Only tests, the smoke check and the CPU-baseline legs of bench.py load it.
//
// Wrapped interfaces:
//   matrix_pro::gemm_f32        include/matrix_pro/cpu/gemm.hpp:23-24 (src/hw/gemm.cpp:73-102)
//   matrix_pro::gemm_reference  include/matrix_pro/cpu/gemm.hpp:20-21 (src/hw/gemm_scalar.cpp:12-33)
//   matrix_pro::gemm_kernel_name include/matrix_pro/cpu/gemm.hpp:28   (src/hw/gemm.cpp:62-71)
//   WorkStealingPool::worker_count include/matrix_pro/core/thread_pool.hpp (src/hw/thread_pool.cpp:187)

#include "matrix_pro/core/thread_pool.hpp"
#include "matrix_pro/cpu/gemm.hpp"

#include <exception>

extern "C" {

int mfref_gemm_f32(int m, int n, int k, const float* a, int lda, const float* b, int ldb, float* c, int ldc,
                   float alpha, float beta) {
    try {
        matrix_pro::gemm_f32(m, n, k, a, lda, b, ldb, c, ldc, alpha, beta);
        return 0;
    } catch (const std::exception&) {
        return 1;
    }
}

int mfref_gemm_reference(int m, int n, int k, const float* a, int lda, const float* b, int ldb, float* c, int ldc,
                         float alpha, float beta) {
    matrix_pro::gemm_reference(m, n, k, a, lda, b, ldb, c, ldc, alpha, beta);
    return 0;
}

const char* mfref_gemm_kernel_name() { return matrix_pro::gemm_kernel_name(); }

int mfref_worker_count() { return matrix_pro::WorkStealingPool::instance().worker_count(); }

}  // extern "C"
