// conv2d forward (NCHW cross-correlation), replacing conv2d / conv2d_kernel of the
// reference (src/nn/conv.cu:22-49,110-163).
//
// Direct kernel: one thread per output pixel and a block-shared copy of the
// filter's weights; taps in the reference's order (channel -> kh -> kw, bias
// first, FMA), so results match the reference kernel's arithmetic exactly.
#include "mfb_internal.h"

#include <algorithm>

namespace mfb {

namespace {

constexpr int kConvThreads = 256;

// grid: (ceil(P*Q / 256), K, N). Weights of filter blockIdx.y are staged in shared memory.
__global__ void __launch_bounds__(kConvThreads) conv2d_direct_kernel(const float* __restrict__ x,
                                                                     const float* __restrict__ w,
                                                                     const float* __restrict__ bias,
                                                                     float* __restrict__ y, int C, int H, int W,
                                                                     int K, int R, int S, int P, int Q, int stride,
                                                                     int pad) {
    extern __shared__ float ws[];
    const int f = blockIdx.y;
    const int nimg = blockIdx.z;
    const int taps = C * R * S;
    for (int i = threadIdx.x; i < taps; i += blockDim.x) ws[i] = w[static_cast<long long>(f) * taps + i];
    __syncthreads();
    const int pix = blockIdx.x * blockDim.x + threadIdx.x;
    if (pix >= P * Q) return;
    const int oh = pix / Q;
    const int ow = pix - oh * Q;
    float sum = bias[f];
    const float* xn = x + static_cast<long long>(nimg) * C * H * W;
    for (int c = 0; c < C; ++c) {
        const float* xc = xn + static_cast<long long>(c) * H * W;
        for (int kh = 0; kh < R; ++kh) {
            const int row = oh * stride + kh - pad;
            if (row < 0 || row >= H) continue;
            for (int kw = 0; kw < S; ++kw) {
                const int col = ow * stride + kw - pad;
                if (col < 0 || col >= W) continue;
                sum = fmaf(__ldg(xc + static_cast<long long>(row) * W + col), ws[(c * R + kh) * S + kw], sum);
            }
        }
    }
    y[(static_cast<long long>(nimg) * K + f) * P * Q + pix] = sum;
}

}  // namespace

mfb_status_t conv2d_launch(int device, cudaStream_t stream, int n, int c, int h, int w, int k, int r, int s,
                           int stride, int pad, const float* x, const float* wgt, const float* bias, float* y,
                           int precision) {
    (void)device;
    (void)precision;
    const int P = (h + 2 * pad - r) / stride + 1;
    const int Q = (w + 2 * pad - s) / stride + 1;
    if (n == 0 || P <= 0 || Q <= 0) return MFB_OK;
    const long long taps = static_cast<long long>(c) * r * s;
    const size_t smem = static_cast<size_t>(taps) * 4;
    if (smem > 200 * 1024) return fail(MFB_EUNSUPPORTED, "conv2d filter too large for the direct kernel");
    if (k > 65535 || n > 65535) return fail(MFB_EUNSUPPORTED, "conv2d batch or filter count too large");
    if (smem > 48 * 1024)
        MFB_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(&conv2d_direct_kernel),
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
                     "conv smem attribute");
    dim3 grid((P * Q + kConvThreads - 1) / kConvThreads, k, n);
    conv2d_direct_kernel<<<grid, kConvThreads, smem, stream>>>(x, wgt, bias, y, c, h, w, k, r, s, P, Q, stride, pad);
    MFB_CUDA_TRY(cudaGetLastError(), "conv2d launch");
    return MFB_OK;
}

}  // namespace mfb
