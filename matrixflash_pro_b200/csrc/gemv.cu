// Bandwidth-bound FP32 GEMV / skinny GEMM (strict FP32 FMA arithmetic).
//
// Replaces gemm_gemv (src/ops/gemm/gemm_gemv.cu:86-110): gemv_rows_kernel (:10),
// gemm_skinny_n_kernel (:30) and gemv_cols_kernel (:61), which read A with scalar
// 4-byte loads, handle only contiguous alpha=1/beta=0 operands and n <= 4.
//
// rows kernel (n <= 16): each warp owns R rows; lanes walk K with 128-bit loads of
// A (one 512-byte coalesced segment per row per step). The B columns of the current
// 512-deep K chunk are staged transposed in shared memory (xs[col][k]) so a lane's
// 128-bit shared load of 4 consecutive k is bank-conflict free. Lane partial sums are
// combined with warp shuffles; alpha/beta/bias/activation are fused into the store.
//
// cols kernel (m == 1): y^T = x^T B. Threads own 4 consecutive columns (128-bit loads
// of B rows), blocks split K; per-split partial rows land in scratch and a second
// small kernel reduces them in a fixed order and applies the epilogue, so results are
// deterministic.
#include "gemm_tc.cuh"
#include "mfb_internal.h"

#include <algorithm>

namespace mfb {

namespace {

constexpr int kGemvKChunk = 512;
constexpr int kGemvThreads = 256;

template <int NC, int R>
__global__ void __launch_bounds__(kGemvThreads) gemv_rows_kernel(const float* __restrict__ a, long long lda,
                                                                 const float* __restrict__ x, long long ldx,
                                                                 float* __restrict__ c, long long ldc, int m, int n,
                                                                 int k, float alpha, float beta,
                                                                 const float* __restrict__ bias, int epilogue,
                                                                 int a_vec) {
    __shared__ __align__(16) float xs[NC][kGemvKChunk + 4];  // +4 spreads the transposed stores over banks
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    constexpr int kRowsPerBlock = (kGemvThreads / 32) * R;
    for (long long row0 = static_cast<long long>(blockIdx.x) * kRowsPerBlock; row0 < m;
         row0 += static_cast<long long>(gridDim.x) * kRowsPerBlock) {
        float acc[R][NC];
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int q = 0; q < NC; ++q) acc[r][q] = 0.0f;
        const long long wrow = row0 + warp * R;
        for (int kc = 0; kc < k; kc += kGemvKChunk) {
            const int kn = min(kGemvKChunk, k - kc);
            __syncthreads();
            for (int i = threadIdx.x; i < kGemvKChunk * NC; i += kGemvThreads) {
                const int kk = i / NC;
                const int q = i - kk * NC;
                xs[q][kk] = (kk < kn && q < n) ? __ldg(x + static_cast<long long>(kc + kk) * ldx + q) : 0.0f;
            }
            __syncthreads();
            for (int kk = lane * 4; kk < kn; kk += 128) {
                float4 av[R];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const long long row = wrow + r;
                    av[r] = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (row < m) {
                        const float* src = a + row * lda + kc + kk;
                        if (a_vec && kk + 3 < kn) {
                            av[r] = __ldg(reinterpret_cast<const float4*>(src));
                        } else {
                            av[r].x = (kk + 0 < kn) ? __ldg(src + 0) : 0.0f;
                            av[r].y = (kk + 1 < kn) ? __ldg(src + 1) : 0.0f;
                            av[r].z = (kk + 2 < kn) ? __ldg(src + 2) : 0.0f;
                            av[r].w = (kk + 3 < kn) ? __ldg(src + 3) : 0.0f;
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < NC; ++q) {
                    const float4 xv = *reinterpret_cast<const float4*>(&xs[q][kk]);
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        acc[r][q] = fmaf(av[r].x, xv.x, acc[r][q]);
                        acc[r][q] = fmaf(av[r].y, xv.y, acc[r][q]);
                        acc[r][q] = fmaf(av[r].z, xv.z, acc[r][q]);
                        acc[r][q] = fmaf(av[r].w, xv.w, acc[r][q]);
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int q = 0; q < NC; ++q) {
                float v = acc[r][q];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
                const long long row = wrow + r;
                if (lane == ((r * NC + q) & 31) && row < m && q < n) {
                    float* dst = c + row * ldc + q;
                    float o = alpha * v;
                    if (beta != 0.0f) o = fmaf(beta, *dst, o);
                    *dst = apply_epilogue_op(o, bias, q, epilogue);
                }
            }
        }
    }
}

// Partial sums of y^T = x^T B over K slice blockIdx.y, 4 columns per thread.
__global__ void __launch_bounds__(128) gemv_cols_partial_kernel(const float* __restrict__ x, const float* __restrict__ b,
                                                                long long ldb, int n, int k, int k_per_split,
                                                                float* __restrict__ partial, int b_vec) {
    const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    const int k0 = blockIdx.y * k_per_split;
    const int k1 = min(k, k0 + k_per_split);
    if (col >= n) return;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = k0; p < k1; ++p) {
        const float xv = __ldg(x + p);
        const float* src = b + static_cast<long long>(p) * ldb + col;
        float4 bv;
        if (b_vec && col + 3 < n) {
            bv = __ldg(reinterpret_cast<const float4*>(src));
        } else {
            bv.x = __ldg(src);
            bv.y = (col + 1 < n) ? __ldg(src + 1) : 0.0f;
            bv.z = (col + 2 < n) ? __ldg(src + 2) : 0.0f;
            bv.w = (col + 3 < n) ? __ldg(src + 3) : 0.0f;
        }
        acc.x = fmaf(xv, bv.x, acc.x);
        acc.y = fmaf(xv, bv.y, acc.y);
        acc.z = fmaf(xv, bv.z, acc.z);
        acc.w = fmaf(xv, bv.w, acc.w);
    }
    float* dst = partial + static_cast<long long>(blockIdx.y) * n + col;
    dst[0] = acc.x;
    if (col + 1 < n) dst[1] = acc.y;
    if (col + 2 < n) dst[2] = acc.z;
    if (col + 3 < n) dst[3] = acc.w;
}

__global__ void gemv_cols_finish_kernel(const float* __restrict__ partial, int splits, int n, float* __restrict__ c,
                                        float alpha, float beta, const float* __restrict__ bias, int epilogue) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= n) return;
    float s = 0.0f;
    for (int i = 0; i < splits; ++i) s += partial[static_cast<long long>(i) * n + col];
    float o = alpha * s;
    if (beta != 0.0f) o = fmaf(beta, c[col], o);
    c[col] = apply_epilogue_op(o, bias, col, epilogue);
}

// x^T for m == 1 lives in A's single row (lda irrelevant); it must be contiguous.
int cols_splits(int n, int k) {
    const int col_blocks = (n + 511) / 512;
    int splits = std::max(1, (148 * 4) / std::max(1, col_blocks));
    splits = std::min(splits, std::max(1, k / 64));
    return std::min(splits, 1024);
}

template <int NC, int R>
void launch_rows(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                 const float* bias, int a_vec) {
    constexpr int kRowsPerBlock = (kGemvThreads / 32) * R;
    const long long row_blocks = (static_cast<long long>(d.m) + kRowsPerBlock - 1) / kRowsPerBlock;
    const int grid = static_cast<int>(std::min<long long>(row_blocks, 148LL * 8));
    gemv_rows_kernel<NC, R><<<grid, kGemvThreads, 0, stream>>>(a, d.lda, b, d.ldb, c, d.ldc, d.m, d.n, d.k,
                                                               d.alpha, d.beta, bias, d.epilogue, a_vec);
}

}  // namespace

bool gemv_eligible(const mfb_gemm_desc& d) {
    return d.trans_a == 0 && d.trans_b == 0 && d.k > 0 && (d.n <= 16 || d.m == 1);
}

size_t gemv_workspace_bytes(const mfb_gemm_desc& d) {
    if (d.n <= 16) return 0;
    return static_cast<size_t>(cols_splits(d.n, d.k)) * static_cast<size_t>(d.n) * 4;
}

mfb_status_t gemv_launch(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                         const float* bias, void* workspace, size_t workspace_bytes) {
    if (d.n <= 16) {
        const int a_vec = (aligned16(a) && d.lda % 4 == 0) ? 1 : 0;
        if (d.n == 1)
            launch_rows<1, 4>(d, stream, a, b, c, bias, a_vec);
        else if (d.n <= 2)
            launch_rows<2, 4>(d, stream, a, b, c, bias, a_vec);
        else if (d.n <= 4)
            launch_rows<4, 4>(d, stream, a, b, c, bias, a_vec);
        else if (d.n <= 8)
            launch_rows<8, 4>(d, stream, a, b, c, bias, a_vec);
        else
            launch_rows<16, 2>(d, stream, a, b, c, bias, a_vec);
        MFB_CUDA_TRY(cudaGetLastError(), "GEMV rows launch");
        return MFB_OK;
    }
    // m == 1: x is A's first row (contiguous along k).
    const int splits = cols_splits(d.n, d.k);
    const size_t need = static_cast<size_t>(splits) * static_cast<size_t>(d.n) * 4;
    if (workspace == nullptr || workspace_bytes < need) return fail(MFB_EINVAL, "GEMV workspace too small");
    float* partial = static_cast<float*>(workspace);
    const int k_per_split = (d.k + splits - 1) / splits;
    const int b_vec = (aligned16(b) && d.ldb % 4 == 0) ? 1 : 0;
    dim3 grid((d.n + 511) / 512, splits);
    gemv_cols_partial_kernel<<<grid, 128, 0, stream>>>(a, b, d.ldb, d.n, d.k, k_per_split, partial, b_vec);
    MFB_CUDA_TRY(cudaGetLastError(), "GEMV cols launch");
    gemv_cols_finish_kernel<<<(d.n + 255) / 256, 256, 0, stream>>>(partial, splits, d.n, c, d.alpha, d.beta, bias,
                                                                   d.epilogue);
    MFB_CUDA_TRY(cudaGetLastError(), "GEMV cols finish launch");
    return MFB_OK;
}

// ------------------------------------------------------------------------------------
// Naive device oracle: one thread per output, sequential FMA chain over k
// (the role of the comparison kernel in benchmarks/bench_comparison.cu:76).
// ------------------------------------------------------------------------------------
__global__ void naive_sgemm_kernel(int m, int n, int k, const float* __restrict__ a, long long lda,
                                   const float* __restrict__ b, long long ldb, float* __restrict__ c, long long ldc,
                                   float alpha, float beta, const float* __restrict__ bias, int epilogue) {
    const long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x;
    if (idx >= static_cast<long long>(m) * n) return;
    const int row = static_cast<int>(idx / n);
    const int col = static_cast<int>(idx - static_cast<long long>(row) * n);
    float acc = 0.0f;
    for (int p = 0; p < k; ++p) acc = fmaf(a[row * lda + p], b[p * ldb + col], acc);
    float* dst = c + row * ldc + col;
    float o = alpha * acc;
    if (beta != 0.0f) o = fmaf(beta, *dst, o);
    *dst = apply_epilogue_op(o, bias, col, epilogue);
}

mfb_status_t naive_launch(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                          const float* bias) {
    const long long total = static_cast<long long>(d.m) * d.n;
    if (total == 0) return MFB_OK;
    const long long blocks = (total + 255) / 256;
    if (blocks > 0x7fffffffLL) return fail(MFB_EINVAL, "naive GEMM too large");
    naive_sgemm_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(d.m, d.n, d.k, a, d.lda, b, d.ldb, c, d.ldc,
                                                                          d.alpha, d.beta, bias, d.epilogue);
    MFB_CUDA_TRY(cudaGetLastError(), "naive GEMM launch");
    return MFB_OK;
}

// ------------------------------------------------------------------------------------
// Bounded-wait probe: waits on an mbarrier that nothing arrives on, gives up after
// limit_ns and reports kStatusTimeoutProbe. Exercises the timeout path of the
// device status word without faulting or hanging the GPU.
// ------------------------------------------------------------------------------------
__global__ void probe_wait_kernel(unsigned long long limit_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        if (!mbar_wait_bounded(&bar, 0, limit_ns, &abort_flag)) report_status(kStatusTimeoutProbe, &abort_flag);
    }
    __syncthreads();
}

mfb_status_t probe_wait_launch(cudaStream_t stream, uint64_t limit_ns) {
    probe_wait_kernel<<<1, 32, 0, stream>>>(limit_ns);
    MFB_CUDA_TRY(cudaGetLastError(), "probe launch");
    return MFB_OK;
}

}  // namespace mfb
