/*
 * Oracle — TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU arithmetic for the dense FP32
 * contraction path. Only tests/, __graft_entry__.smoke() and the CPU-baseline
 * legs of bench.py load this library, and only as the checker. Nothing in the
 * product (matrixflash_pro_b200/, include/) links or calls it.
 *
 * Parity is pinned: oracle_gemm_f32 is compared bit-for-bit with the
 * reference's own gemm_f32 built from its sources (oracle/_ref) and with golden
 * fixtures produced by that build (tests/golden/); the conv restatement is
 * pinned by the known answers of tests/unit/test_conv.cpp:31-67,117-121.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#define ORACLE_API __attribute__((visibility("default")))

/*
 * The reference's AVX2 GEMM (src/hw/gemm_avx2.cpp:408-451) computes every
 * C[i][j] as one FP32 chain:
 *   acc = (beta == 0) ? 0 : beta * C[i][j]        (kernel_4x16 :84-103, kernel_edge :202-217)
 *   acc = fma(alpha * A[i][p], B[p][j], acc)       p = 0..k-1 (kernel_4x16 :105-181)
 * alpha is folded into the packed A panel (pack_a :235-287), the chain carries
 * across Kc=512 panels because later panels run with beta = 1 (:444) and C is
 * the carried value. Columns are processed in 16-wide tiles; a tile with fewer
 * than 16 columns goes through kernel_edge (:199-232), where the trailing
 * nr % 8 columns are updated with a separate multiply and add (no FMA: the file
 * is compiled with -ffp-contract=off, cmake/MatrixFlashSources.cmake:93-95).
 * gemm_f32 (src/hw/gemm.cpp:73-102) returns early for m<=0 or n<=0 and uses
 * gemm_reference for k<=0.
 */
static float oracle_element_f32(int i, int j, int n, int k, const float* a, int lda, const float* b, int ldb,
                                float c_in, float alpha, float beta) {
    const int j0 = (j / 16) * 16;
    const int nr = (n - j0) < 16 ? (n - j0) : 16;
    const int fused = (j - j0) < 8 * (nr / 8);
    float acc;
    if (beta == 0.0f) {
        acc = 0.0f;
    } else {
        acc = beta * c_in;
    }
    const float* arow = a + (size_t)i * (size_t)lda;
    for (int p = 0; p < k; ++p) {
        const float coef = alpha * arow[p];
        const float bv = b[(size_t)p * (size_t)ldb + (size_t)j];
        if (fused) {
            acc = fmaf(coef, bv, acc);
        } else {
            const float prod = coef * bv;
            acc = acc + prod;
        }
    }
    return acc;
}

/* gemm_reference (src/hw/gemm_scalar.cpp:12-33): beta-scale the row, then c += (alpha*a)*b, no FMA. */
ORACLE_API void oracle_gemm_reference_f32(int m, int n, int k, const float* a, int lda, const float* b, int ldb,
                                          float* c, int ldc, float alpha, float beta) {
    for (int i = 0; i < m; ++i) {
        float* crow = c + (size_t)i * (size_t)ldc;
        if (beta == 0.0f) {
            for (int j = 0; j < n; ++j) crow[j] = 0.0f;
        } else if (beta != 1.0f) {
            for (int j = 0; j < n; ++j) crow[j] *= beta;
        }
        const float* arow = a + (size_t)i * (size_t)lda;
        for (int p = 0; p < k; ++p) {
            const float coef = alpha * arow[p];
            const float* brow = b + (size_t)p * (size_t)ldb;
            for (int j = 0; j < n; ++j) {
                const float prod = coef * brow[j];
                crow[j] = crow[j] + prod;
            }
        }
    }
}

/* gemm_f32 on an AVX2+FMA host (src/hw/gemm.cpp:73-102 -> gemm_avx2_serial). */
ORACLE_API void oracle_gemm_f32(int m, int n, int k, const float* a, int lda, const float* b, int ldb, float* c,
                                int ldc, float alpha, float beta) {
    if (m <= 0 || n <= 0) return;
    if (k <= 0) {
        oracle_gemm_reference_f32(m, n, 0, a, lda, b, ldb, c, ldc, alpha, beta);
        return;
    }
    for (int i = 0; i < m; ++i) {
        float* crow = c + (size_t)i * (size_t)ldc;
        for (int j = 0; j < n; ++j) {
            crow[j] = oracle_element_f32(i, j, n, k, a, lda, b, ldb, crow[j], alpha, beta);
        }
    }
}

/* Rows [row_begin,row_end) of oracle_gemm_f32, so callers can spread rows over processes. */
ORACLE_API void oracle_gemm_f32_rows(int row_begin, int row_end, int n, int k, const float* a, int lda,
                                     const float* b, int ldb, float* c, int ldc, float alpha, float beta) {
    for (int i = row_begin; i < row_end; ++i) {
        float* crow = c + (size_t)i * (size_t)ldc;
        for (int j = 0; j < n; ++j) {
            crow[j] = oracle_element_f32(i, j, n, k, a, lda, b, ldb, crow[j], alpha, beta);
        }
    }
}

/*
 * Sampled block of oracle_gemm_f32 for the full (m x n x k) product: out[r][s] is
 * element (rows[r], cols[s]) exactly as gemm_f32 computes it on the full problem.
 * c_in (may be NULL when beta == 0) holds C[rows[r]][cols[s]] before the call.
 */
ORACLE_API void oracle_gemm_f32_sampled(int nrows, const int* rows, int ncols, const int* cols, int n, int k,
                                        const float* a, int lda, const float* b, int ldb, const float* c_in,
                                        float alpha, float beta, float* out) {
    for (int r = 0; r < nrows; ++r) {
        for (int s = 0; s < ncols; ++s) {
            const float cv = c_in ? c_in[(size_t)r * (size_t)ncols + (size_t)s] : 0.0f;
            out[(size_t)r * (size_t)ncols + (size_t)s] =
                oracle_element_f32(rows[r], cols[s], n, k, a, lda, b, ldb, cv, alpha, beta);
        }
    }
}

/* FP64 reference: out = alpha * sum_p A[i][p] B[p][j] + beta * C[i][j], all in double. */
ORACLE_API void oracle_gemm_f64(int m, int n, int k, const float* a, int lda, const float* b, int ldb,
                                const float* c_in, int ldc, double alpha, double beta, double* out, int ldo) {
    for (int i = 0; i < m; ++i) {
        double* orow = out + (size_t)i * (size_t)ldo;
        for (int j = 0; j < n; ++j) orow[j] = 0.0;
        const float* arow = a + (size_t)i * (size_t)lda;
        for (int p = 0; p < k; ++p) {
            const double av = (double)arow[p];
            const float* brow = b + (size_t)p * (size_t)ldb;
            for (int j = 0; j < n; ++j) orow[j] += av * (double)brow[j];
        }
        for (int j = 0; j < n; ++j) {
            double v = alpha * orow[j];
            if (beta != 0.0 && c_in) v += beta * (double)c_in[(size_t)i * (size_t)ldc + (size_t)j];
            orow[j] = v;
        }
    }
}

/*
 * conv2d forward, NCHW cross-correlation: a restatement of conv2d_kernel
 * (src/nn/conv.cu:22-49). One output = bias[k], then the taps in the order
 * channel -> kh -> kw, out-of-bounds taps skipped. nvcc contracts the device
 * statement `sum += input * weight` into an FMA (default -fmad=true), so the
 * restatement uses fmaf. Output size follows src/nn/conv.cu:118-119.
 */
ORACLE_API void oracle_conv2d_f32(int batch, int channels, int height, int width, int filters, int kh_size,
                                  int kw_size, int stride, int padding, const float* input, const float* weights,
                                  const float* bias, float* output) {
    const int oh_size = (height + 2 * padding - kh_size) / stride + 1;
    const int ow_size = (width + 2 * padding - kw_size) / stride + 1;
    for (int n = 0; n < batch; ++n) {
        for (int f = 0; f < filters; ++f) {
            for (int oh = 0; oh < oh_size; ++oh) {
                for (int ow = 0; ow < ow_size; ++ow) {
                    float sum = bias[f];
                    for (int c = 0; c < channels; ++c) {
                        for (int kh = 0; kh < kh_size; ++kh) {
                            const long row = (long)oh * stride + kh - padding;
                            if (row < 0 || row >= height) continue;
                            for (int kw = 0; kw < kw_size; ++kw) {
                                const long col = (long)ow * stride + kw - padding;
                                if (col < 0 || col >= width) continue;
                                const size_t xi = (((size_t)n * channels + c) * height + (size_t)row) * width +
                                                  (size_t)col;
                                const size_t wi = (((size_t)f * channels + c) * kh_size + kh) * kw_size + kw;
                                sum = fmaf(input[xi], weights[wi], sum);
                            }
                        }
                    }
                    output[(((size_t)n * filters + f) * oh_size + oh) * ow_size + ow] = sum;
                }
            }
        }
    }
}

/* FP64 variant of the conv restatement (same loop order, double accumulation). */
ORACLE_API void oracle_conv2d_f64(int batch, int channels, int height, int width, int filters, int kh_size,
                                  int kw_size, int stride, int padding, const float* input, const float* weights,
                                  const float* bias, double* output) {
    const int oh_size = (height + 2 * padding - kh_size) / stride + 1;
    const int ow_size = (width + 2 * padding - kw_size) / stride + 1;
    for (int n = 0; n < batch; ++n) {
        for (int f = 0; f < filters; ++f) {
            for (int oh = 0; oh < oh_size; ++oh) {
                for (int ow = 0; ow < ow_size; ++ow) {
                    double sum = (double)bias[f];
                    for (int c = 0; c < channels; ++c) {
                        for (int kh = 0; kh < kh_size; ++kh) {
                            const long row = (long)oh * stride + kh - padding;
                            if (row < 0 || row >= height) continue;
                            for (int kw = 0; kw < kw_size; ++kw) {
                                const long col = (long)ow * stride + kw - padding;
                                if (col < 0 || col >= width) continue;
                                const size_t xi = (((size_t)n * channels + c) * height + (size_t)row) * width +
                                                  (size_t)col;
                                const size_t wi = (((size_t)f * channels + c) * kh_size + kh) * kw_size + kw;
                                sum += (double)input[xi] * (double)weights[wi];
                            }
                        }
                    }
                    output[(((size_t)n * filters + f) * oh_size + oh) * ow_size + ow] = sum;
                }
            }
        }
    }
}

/*
 * conv2d backward, restated from the reference's kernels (src/nn/backward/convolution_kernels.cuh):
 * conv2d_input_backward_kernel (:9-47), conv2d_weight_backward_kernel (:50-82) and
 * conv2d_bias_backward_kernel (:85-95), same loop orders and skip rules. The products accumulate
 * as `acc += a * b`, which nvcc contracts to one FMA; the bias sum is a plain add.
 * ACC is float (FMA) or double (exact products) below.
 */
#define ORACLE_CONV_BWD(NAME, ACC, MAC)                                                                        \
    ORACLE_API void oracle_conv2d_input_backward_##NAME(                                                      \
        int batch, int channels, int height, int width, int filters, int kh_size, int kw_size, int stride,    \
        int padding, const float* grad, const float* weights, ACC* input_grad) {                              \
        const long out_h = (height + 2 * padding - kh_size) / stride + 1;                                    \
        const long out_w = (width + 2 * padding - kw_size) / stride + 1;                                     \
        for (int n = 0; n < batch; ++n)                                                                        \
            for (int c = 0; c < channels; ++c)                                                                 \
                for (int ih = 0; ih < height; ++ih)                                                            \
                    for (int iw = 0; iw < width; ++iw) {                                                       \
                        ACC acc = 0;                                                                           \
                        for (int f = 0; f < filters; ++f)                                                      \
                            for (int kh = 0; kh < kh_size; ++kh) {                                             \
                                const long ohl = (long)ih + padding - kh;                                      \
                                if (ohl < 0 || ohl % stride != 0) continue;                                    \
                                const long oh = ohl / stride;                                                  \
                                if (oh >= out_h) continue;                                                     \
                                for (int kw = 0; kw < kw_size; ++kw) {                                         \
                                    const long owl = (long)iw + padding - kw;                                  \
                                    if (owl < 0 || owl % stride != 0) continue;                                \
                                    const long ow = owl / stride;                                              \
                                    if (ow >= out_w) continue;                                                 \
                                    const float g = grad[(((size_t)n * filters + f) * out_h + oh) * out_w + ow]; \
                                    const float w = weights[(((size_t)f * channels + c) * kh_size + kh) * kw_size + kw]; \
                                    acc = MAC(g, w, acc);                                                      \
                                }                                                                              \
                            }                                                                                  \
                        input_grad[(((size_t)n * channels + c) * height + ih) * width + iw] = acc;             \
                    }                                                                                          \
    }                                                                                                          \
    ORACLE_API void oracle_conv2d_weight_backward_##NAME(                                                     \
        int batch, int channels, int height, int width, int filters, int kh_size, int kw_size, int stride,    \
        int padding, const float* grad, const float* input, ACC* weight_grad) {                               \
        const long out_h = (height + 2 * padding - kh_size) / stride + 1;                                    \
        const long out_w = (width + 2 * padding - kw_size) / stride + 1;                                     \
        for (int f = 0; f < filters; ++f)                                                                      \
            for (int c = 0; c < channels; ++c)                                                                 \
                for (int kh = 0; kh < kh_size; ++kh)                                                           \
                    for (int kw = 0; kw < kw_size; ++kw) {                                                     \
                        ACC acc = 0;                                                                           \
                        for (int n = 0; n < batch; ++n)                                                        \
                            for (long oh = 0; oh < out_h; ++oh) {                                              \
                                const long ih = oh * stride + kh - padding;                                    \
                                if (ih < 0 || ih >= height) continue;                                          \
                                for (long ow = 0; ow < out_w; ++ow) {                                          \
                                    const long iw = ow * stride + kw - padding;                                \
                                    if (iw < 0 || iw >= width) continue;                                       \
                                    const float g = grad[(((size_t)n * filters + f) * out_h + oh) * out_w + ow]; \
                                    const float x = input[(((size_t)n * channels + c) * height + ih) * width + iw]; \
                                    acc = MAC(g, x, acc);                                                      \
                                }                                                                              \
                            }                                                                                  \
                        weight_grad[(((size_t)f * channels + c) * kh_size + kh) * kw_size + kw] = acc;         \
                    }                                                                                          \
    }                                                                                                          \
    ORACLE_API void oracle_conv2d_bias_backward_##NAME(int batch, int filters, int out_h, int out_w,          \
                                                       const float* grad, ACC* bias_grad) {                    \
        for (int f = 0; f < filters; ++f) {                                                                    \
            ACC acc = 0;                                                                                       \
            for (int n = 0; n < batch; ++n)                                                                    \
                for (int oh = 0; oh < out_h; ++oh)                                                             \
                    for (int ow = 0; ow < out_w; ++ow)                                                         \
                        acc += grad[(((size_t)n * filters + f) * out_h + oh) * out_w + ow];                    \
            bias_grad[f] = acc;                                                                                \
        }                                                                                                      \
    }

#define ORACLE_FMA_F32(a, b, acc) fmaf((a), (b), (acc))
#define ORACLE_MAC_F64(a, b, acc) ((acc) + (double)(a) * (double)(b))
ORACLE_CONV_BWD(f32, float, ORACLE_FMA_F32)
ORACLE_CONV_BWD(f64, double, ORACLE_MAC_F64)

/*
 * Column-bias epilogue: a restatement of epilogue_col_bias_kernel
 * (src/ops/gemm/gemm_fused.cu:23-40): v = c + bias[col]; mode 1 ReLU, mode 2 tanh-GELU.
 */
ORACLE_API void oracle_epilogue_f32(float* c, int ldc, const float* bias, int m, int n, int mode) {
    for (int i = 0; i < m; ++i) {
        for (int j = 0; j < n; ++j) {
            float v = c[(size_t)i * (size_t)ldc + (size_t)j] + bias[j];
            if (mode == 1) {
                v = v > 0.0f ? v : 0.0f;
            } else if (mode == 2) {
                const float x3 = v * v * v;
                v = 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * x3)));
            }
            c[(size_t)i * (size_t)ldc + (size_t)j] = v;
        }
    }
}
