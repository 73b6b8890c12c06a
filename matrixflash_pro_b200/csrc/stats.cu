// Covariance and correlation of the columns of a row-major matrix, on the library's own
// kernels. Replaces matrix_pro::covariance / correlation (src/ops/reductions/covariance.inc:23-60),
// whose centered product runs on cublasSgemm (:38-44).
//
//   mean  = (1/rows) * ones^T X          one m = 1 GEMV (deterministic split-K)
//   cov   = X_c^T X_c / max(rows - 1, 1)  the tcgen05 GEMM with trans_a; the centering
//                                         X_c = X - mean happens inside the operand prepass
//                                         (split_tf32_kernel's column shift), so no centered
//                                         copy of X is written
//   corr  = cov_ij / sqrt(cov_ii cov_jj), 1 on the diagonal, 0 where a variance is not
//           positive (moment_kernels.cuh:51-67)
#include "mfb_internal.h"

namespace mfb {
namespace {

__global__ void fill_kernel(float* __restrict__ p, long long count, float value) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        p[i] = value;
}

__global__ void cov_to_corr_kernel(const float* __restrict__ cov, long long ldcov, float* __restrict__ corr,
                                   long long ldcorr, int dims) {
    const long long total = static_cast<long long>(dims) * dims;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int row = static_cast<int>(idx / dims);
        const int col = static_cast<int>(idx - static_cast<long long>(row) * dims);
        float out = 1.0f;
        if (row != col) {
            const float vr = cov[row * ldcov + row];
            const float vc = cov[col * ldcov + col];
            out = (vr > 0.0f && vc > 0.0f) ? cov[row * ldcov + col] / sqrtf(vr * vc) : 0.0f;
        }
        corr[row * ldcorr + col] = out;
    }
}

size_t align256(size_t bytes) { return (bytes + 255) / 256 * 256; }

// Workspace layout: [ones: rows][mean: cols][GEMV partials][GEMM planes][cov: cols x cols, correlation only]
struct CovPlan {
    mfb_gemm_desc mean_desc{};
    mfb_gemm_desc cov_desc{};
    size_t ones_off = 0, mean_off = 0, gemv_off = 0, tc_off = 0, cov_off = 0, total = 0;
    size_t gemv_bytes = 0, tc_bytes = 0;
};

CovPlan cov_plan(int rows, int cols, long long ldx, int precision, bool with_cov_buffer) {
    CovPlan p;
    mfb_gemm_desc& md = p.mean_desc;
    md.m = 1;
    md.n = cols;
    md.k = rows;
    md.lda = std::max(1, rows);
    md.ldb = static_cast<int>(ldx);
    md.ldc = std::max(1, cols);
    md.alpha = 1.0f / static_cast<float>(rows);
    md.beta = 0.0f;
    md.precision = MFB_PRECISION_FP32;
    mfb_gemm_desc& cd = p.cov_desc;
    cd.m = cols;
    cd.n = cols;
    cd.k = rows;
    cd.lda = static_cast<int>(ldx);  // A = X stored rows x cols, used transposed
    cd.ldb = static_cast<int>(ldx);
    cd.ldc = std::max(1, cols);  // overwritten by the caller's ld
    cd.alpha = 1.0f / static_cast<float>(rows > 1 ? rows - 1 : 1);
    cd.beta = 0.0f;
    cd.precision = precision;
    cd.trans_a = 1;
    p.gemv_bytes = gemv_workspace_bytes(md);
    TcConfig first[1];
    p.tc_bytes = tc_candidates(cd, first, 1) > 0 ? tc_workspace_bytes_for(cd, first[0]) : tc_workspace_bytes(cd);
    p.ones_off = 0;
    p.mean_off = align256(static_cast<size_t>(rows) * 4);
    p.gemv_off = p.mean_off + align256(static_cast<size_t>(cols) * 4);
    p.tc_off = p.gemv_off + align256(p.gemv_bytes);
    p.cov_off = p.tc_off + align256(p.tc_bytes);
    p.total = p.cov_off + (with_cov_buffer ? align256(static_cast<size_t>(cols) * cols * 4) : 0);
    return p;
}

mfb_status_t covariance_run(int device, cudaStream_t stream, int rows, int cols, const float* x, long long ldx,
                            float* cov, long long ldcov, int precision, bool with_cov_buffer, float** cov_tmp) {
    if (rows <= 0 || cols <= 0 || !x || !cov) return fail(MFB_EINVAL, "covariance: bad arguments");
    if (ldx < cols || ldcov < cols) return fail(MFB_EINVAL, "covariance: leading dimension smaller than cols");
    if (ldx > 0x7fffffffLL || ldcov > 0x7fffffffLL) return fail(MFB_EINVAL, "covariance: leading dimension too large");
    if (precision != MFB_PRECISION_FP32 && precision != MFB_PRECISION_TF32)
        return fail(MFB_EINVAL, "Invalid GEMM precision policy");
    CovPlan plan = cov_plan(rows, cols, ldx, precision, with_cov_buffer);
    plan.cov_desc.ldc = static_cast<int>(ldcov);
    void* ws = nullptr;
    MFB_TRY(stream_workspace(device, stream, plan.total, &ws));
    char* base = static_cast<char*>(ws);
    float* ones = reinterpret_cast<float*>(base + plan.ones_off);
    float* mean = reinterpret_cast<float*>(base + plan.mean_off);
    const int fill_blocks = static_cast<int>(std::min<long long>((rows + 255) / 256, static_cast<long long>(current_sm_count()) * 4));
    fill_kernel<<<fill_blocks, 256, 0, stream>>>(ones, rows, 1.0f);
    MFB_CUDA_TRY(cudaGetLastError(), "covariance fill launch");
    MFB_TRY(gemv_launch(plan.mean_desc, stream, ones, x, mean, nullptr, base + plan.gemv_off, plan.gemv_bytes));
    float* target = cov;
    if (with_cov_buffer) {
        target = reinterpret_cast<float*>(base + plan.cov_off);
        plan.cov_desc.ldc = cols;
        *cov_tmp = target;
    }
    TcConfig cfgs[4];
    if (tc_candidates(plan.cov_desc, cfgs, 4) == 0) return fail(MFB_EUNSUPPORTED, "no tcgen05 configuration");
    TcPrologue centering;
    centering.a_col_shift = mean;
    centering.b_col_shift = mean;
    centering.shared_planes = true;  // X^T X: one centered split of X serves both operands
    return tc_gemm(plan.cov_desc, cfgs[0], stream, x, x, target, nullptr, base + plan.tc_off, plan.tc_bytes,
                   kPhaseAll, 0, TcBatch(), centering);
}

}  // namespace
}  // namespace mfb

extern "C" {

MFB_API mfb_status_t mfb_covariance(int device, mfb_stream_t stream_h, int rows, int cols, const float* x,
                                    int ldx, float* cov, int ldcov, int precision) {
    mfb::clear_error();
    if (rows < 0 || cols < 0) return mfb::fail(MFB_EINVAL, "covariance: dimensions must be non-negative");
    if (rows == 0 || cols == 0) return MFB_OK;
    if (cov == x) return mfb::fail(MFB_EINVAL, "covariance output cannot alias its input");
    mfb::DeviceGuard guard;
    MFB_TRY(mfb::select_device(device));
    return mfb::covariance_run(device, reinterpret_cast<cudaStream_t>(stream_h), rows, cols, x, ldx, cov, ldcov,
                               precision, false, nullptr);
}

MFB_API mfb_status_t mfb_correlation(int device, mfb_stream_t stream_h, int rows, int cols, const float* x,
                                     int ldx, float* corr, int ldcorr, int precision) {
    mfb::clear_error();
    if (rows < 0 || cols < 0) return mfb::fail(MFB_EINVAL, "correlation: dimensions must be non-negative");
    if (rows == 0 || cols == 0) return MFB_OK;
    if (corr == x) return mfb::fail(MFB_EINVAL, "correlation output cannot alias its input");
    if (ldcorr < cols) return mfb::fail(MFB_EINVAL, "correlation: leading dimension smaller than cols");
    mfb::DeviceGuard guard;
    MFB_TRY(mfb::select_device(device));
    cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_h);
    float* cov = nullptr;
    MFB_TRY(mfb::covariance_run(device, stream, rows, cols, x, ldx, corr, ldcorr, precision, true, &cov));
    const long long total = static_cast<long long>(cols) * cols;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, static_cast<long long>(current_sm_count()) * 8));
    mfb::cov_to_corr_kernel<<<blocks, 256, 0, stream>>>(cov, cols, corr, ldcorr, cols);
    MFB_CUDA_TRY(cudaGetLastError(), "correlation launch");
    return MFB_OK;
}

}  // extern "C"
