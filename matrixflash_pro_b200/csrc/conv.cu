// conv2d forward (NCHW cross-correlation), replacing conv2d / conv2d_kernel of the
// reference (src/nn/conv.cu:22-49,110-163).
//
// Stride 1 (the reference's bench shapes): implicit GEMM on tcgen05 (conv_tc.cuh)
// after a prepass that writes the zero-padded input with channels innermost, and the
// per-tap weights, as TF32 planes (hi/lo for strict FP32, one rounded plane for TF32).
// Other strides: a direct kernel, one thread per output with the filter staged in
// shared memory and the reference's tap order (channel -> kh -> kw, FMA).
#include "conv_tc.cuh"
#include "mfb_internal.h"

#include <algorithm>
#include <cstdlib>
#include <string>
#include <mutex>

namespace mfb {

namespace {

constexpr int kConvThreads = 256;
// Stride-1 convs below these sizes run the direct kernel (measured with CUDA-graph replay on
// B200, 32 x 32 images, 3 x 3 filters): the tensor path pays three launches and a pipeline
// fill (~12 us), and pads channels to 32-channel slabs, so with C <= 4 it does 8x or more
// of useless K work. C = 3, K = 16: 8 images 6.4 us direct vs 15.3 us tcgen05, 64 images
// 28.6 vs 52.3 us (57 MFLOP); 8 x 3 x 64 x 64 with 64 filters (113 MFLOP): 54.2 vs 43.6 us.
// C = 8 at 19 MFLOP: 14.1 vs 13.4 us; C >= 16 at 19 MFLOP and above: the tensor path wins.
constexpr double kConvDirectMaxFlops = 1e7;
constexpr double kConvDirectMaxFlopsNarrowC = 8e7;  // C <= 4
constexpr int kConvNarrowC = 4;

// Algorithm override for measurements: MFB_CONV_ALGO = direct | implicit_gemm (anything
// else, or unset: the size rule above). implicit_gemm applies to stride 1 only; other
// strides always run the direct kernel. Read once per process.
int conv_algo_override() {
    static const int algo = [] {
        const char* v = std::getenv("MFB_CONV_ALGO");
        if (!v) return 0;
        const std::string s(v);
        return s == "direct" ? 1 : s == "implicit_gemm" ? 2 : 0;
    }();
    return algo;
}

bool conv_use_direct(int stride, double flops, int c) {
    if (stride != 1) return true;
    const int algo = conv_algo_override();
    if (algo != 0) return algo == 1;
    return flops < (c <= kConvNarrowC ? kConvDirectMaxFlopsNarrowC : kConvDirectMaxFlops);
}

__device__ __forceinline__ float conv_round_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Writes 4 consecutive floats as TF32 planes: hi = tf32(v), lo = tf32(v - hi) (lo may be null).
__device__ __forceinline__ void write_planes4(float* hi, float* lo, long long off, float v0, float v1, float v2,
                                              float v3) {
    const float v[4] = {v0, v1, v2, v3};
    float h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        h[i] = conv_round_tf32(v[i]);
        l[i] = conv_round_tf32(v[i] - h[i]);
    }
    *reinterpret_cast<float4*>(hi + off) = make_float4(h[0], h[1], h[2], h[3]);
    if (lo) *reinterpret_cast<float4*>(lo + off) = make_float4(l[0], l[1], l[2], l[3]);
}

// x (N,C,H,W) -> X [N][Hp*Wp][Cp]: zero border of `pad`, zero channels in [C, Cp).
// grid (ceil(Hp / kPackRows), ceil(Cp / 32), N): a block takes kPackRows padded rows of
// 32 channels. Phase 1: each warp reads whole input rows of one channel (64-bit loads when
// W is even and the image is 8-byte aligned) and stores them transposed, [row][iw][33];
// the odd position stride keeps the channel reads of phase 2 conflict-free. Phase 2 writes
// one float4 of 4 channels per (padded position, group) as 128-byte channel rows; border
// positions and channels >= C become zeros there, so the tile is never zero-filled. The
// kernel is issue-bound unless its index arithmetic stays out of the inner loops: no
// division, 32-bit offsets from a per-block base, guards hoisted.
constexpr int kPackRows = 2;
constexpr int kPackStride = 33;
constexpr int kPackMaxWp = 512;  // padded width the shared tile holds; wider images use the generic kernel

size_t pack_rows_smem_bytes(int w) { return static_cast<size_t>(kPackRows) * w * kPackStride * 4; }

__global__ void __launch_bounds__(256) conv_pack_rows_kernel(const float* __restrict__ x, int c, int h, int w,
                                                             int pad_h, int pad_w, int cp, int hp, int wp, int vec,
                                                             float* __restrict__ hi, float* __restrict__ lo);

// The pack kernel's shared tile grows with the image width (up to kPackMaxWp): its dynamic
// shared-memory limit is raised to the largest tile once per device, under a lock, so host
// threads packing images of different widths never race on the attribute.
mfb_status_t allow_pack_rows_smem() {
    static std::mutex mutex;
    static std::vector<char> done;
    int dev = 0;
    MFB_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mutex);
    if (static_cast<int>(done.size()) <= dev) done.resize(dev + 1, 0);
    if (!done[dev]) {
        MFB_CUDA_TRY(cudaFuncSetAttribute(reinterpret_cast<const void*>(&conv_pack_rows_kernel),
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(pack_rows_smem_bytes(kPackMaxWp))),
                     "conv prepass smem attribute");
        done[dev] = 1;
    }
    return MFB_OK;
}

__global__ void __launch_bounds__(256) conv_pack_rows_kernel(const float* __restrict__ x, int c, int h, int w,
                                                             int pad_h, int pad_w, int cp, int hp, int wp, int vec2,
                                                             float* __restrict__ hi, float* __restrict__ lo) {
    extern __shared__ float tile[];  // [kPackRows][w][kPackStride]
    const int pr0 = blockIdx.x * kPackRows;
    const int c0 = blockIdx.y * 32;
    const int img = blockIdx.z;
    const int rows = min(kPackRows, hp - pr0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // Phase 1: input rows -> transposed tile (rows outside the image and channels >= C are skipped).
    // Warp w owns the channel rows (task) w, w + 8, ..., w + 56 (task = rr * 32 + channel); all
    // eight loads of a lane are issued before any shared-memory store, so each SM keeps
    // ~128 KB of loads in flight.
    const int ntask = 32 * rows;
    const int units = vec2 ? w / 2 : w;  // float2 or float units per channel row
    for (int jc = 0; jc < units; jc += 32) {
        const int j = jc + lane;
        float2 v[8];
        bool ok[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int task = warp + 8 * u;
            const int cc = task & 31, rr = task >> 5;
            const int ih = pr0 + rr - pad_h, ch = c0 + cc;
            ok[u] = task < ntask && j < units && ih >= 0 && ih < h && ch < c;
            v[u] = make_float2(0.0f, 0.0f);
            if (ok[u]) {
                const float* src = x + ((static_cast<long long>(img) * c + ch) * h + ih) * w;
                if (vec2) v[u] = __ldg(reinterpret_cast<const float2*>(src) + j);
                else v[u].x = __ldg(src + j);
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            if (!ok[u]) continue;
            const int task = warp + 8 * u;
            const int cc = task & 31, rr = task >> 5;
            if (vec2) {
                float* dst = tile + (rr * w + 2 * j) * kPackStride + cc;
                dst[0] = v[u].x;
                dst[kPackStride] = v[u].y;
            } else {
                tile[(rr * w + j) * kPackStride + cc] = v[u].x;
            }
        }
    }
    __syncthreads();
    // Phase 2: thread t writes channel group q = t % 8 (4 channels) of positions t / 8, +32, ...
    // Offsets are 32-bit from a per-block base; every guard is hoisted out of the loop.
    const int q = threadIdx.x & 7;
    if (q >= min(8, (cp - c0) / 4)) return;
    const long long base = (static_cast<long long>(img) * hp + pr0) * wp * cp + c0 + 4 * q;
    const int nch = min(4, c - (c0 + 4 * q));  // real channels of this group (<= 0: all zero)
    for (int rr = 0; rr < rows; ++rr) {
        const int ih = pr0 + rr - pad_h;
        const bool row_in = ih >= 0 && ih < h && nch > 0;
        const float* trow = tile + rr * w * kPackStride + 4 * q;
        float* hrow = hi + base + static_cast<long long>(rr) * wp * cp;
        float* lrow = lo ? lo + base + static_cast<long long>(rr) * wp * cp : nullptr;
        for (int pw = threadIdx.x >> 3; pw < wp; pw += 32) {
            const int iw = pw - pad_w;
            float v0 = 0.0f, v1 = 0.0f, v2 = 0.0f, v3 = 0.0f;
            if (row_in && static_cast<unsigned>(iw) < static_cast<unsigned>(w)) {
                const float* t = trow + iw * kPackStride;
                v0 = t[0];
                v1 = nch > 1 ? t[1] : 0.0f;
                v2 = nch > 2 ? t[2] : 0.0f;
                v3 = nch > 3 ? t[3] : 0.0f;
            }
            write_planes4(hrow, lrow, static_cast<long long>(pw) * cp, v0, v1, v2, v3);
        }
    }
}

// Generic version of the same layout change (any padded width): 32 channels x 64 positions per block.
// grid (ceil(Hp*Wp / 64), ceil(Cp / 32), N): a 32-channel x 64-position tile is read
// along positions (coalesced in W) and written as 128-byte channel rows.
__global__ void __launch_bounds__(256) conv_pack_input_kernel(const float* __restrict__ x, int c, int h, int w,
                                                              int pad_h, int pad_w, int cp, int hp, int wp,
                                                              float* __restrict__ hi, float* __restrict__ lo) {
    __shared__ float tile[32][65];
    const int npos = hp * wp;
    const int pos0 = blockIdx.x * 64;
    const int c0 = blockIdx.y * 32;
    const int img = blockIdx.z;
    for (int i = threadIdx.x; i < 32 * 64; i += blockDim.x) {
        const int cc = i / 64, pp = i % 64;
        const int pos = pos0 + pp, ch = c0 + cc;
        float v = 0.0f;
        if (pos < npos && ch < c) {
            const int ih = pos / wp - pad_h, iw = pos % wp - pad_w;
            if (ih >= 0 && ih < h && iw >= 0 && iw < w)
                v = __ldg(x + ((static_cast<long long>(img) * c + ch) * h + ih) * w + iw);
        }
        tile[cc][pp] = v;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
        const int pp = i / 8, q = i % 8;
        const int pos = pos0 + pp, ch = c0 + 4 * q;
        if (pos < npos && ch < cp) {
            const long long off = (static_cast<long long>(img) * npos + pos) * cp + ch;
            write_planes4(hi, lo, off, tile[4 * q][pp], tile[4 * q + 1][pp], tile[4 * q + 2][pp], tile[4 * q + 3][pp]);
        }
    }
}

// w (K,C,R,S) -> W [R*S][K][Cp]. flip != 0: `wt` is the (C,K,R,S) filter bank of the forward
// conv whose input gradient is being formed; filter f, channel ch, tap (rr, ss) of the
// packed bank is wt[ch][f][R-1-rr][S-1-ss] (the transposed, spatially flipped filters).
__global__ void conv_pack_weights_kernel(const float* __restrict__ wt, int kf, int c, int r, int s, int cp, int flip,
                                         float* __restrict__ hi, float* __restrict__ lo) {
    const int groups = cp / 4;
    const long long total = static_cast<long long>(r) * s * kf * groups;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int g = static_cast<int>(idx % groups);
        const long long r1 = idx / groups;
        const int f = static_cast<int>(r1 % kf);
        const int tap = static_cast<int>(r1 / kf);
        const int rr = tap / s, ss = tap % s;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int ch = 4 * g + i;
            if (ch >= c)
                v[i] = 0.0f;
            else if (flip)
                v[i] = __ldg(wt + ((static_cast<long long>(ch) * kf + f) * r + (r - 1 - rr)) * s + (s - 1 - ss));
            else
                v[i] = __ldg(wt + ((static_cast<long long>(f) * c + ch) * r + rr) * s + ss);
        }
        write_planes4(hi, lo, idx * 4, v[0], v[1], v[2], v[3]);
    }
}

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

mfb_status_t conv2d_direct(cudaStream_t stream, int n, int c, int h, int w, int k, int r, int s, int stride, int pad,
                           int P, int Q, const float* x, const float* wgt, const float* bias, float* y) {
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

// ------------------------------------------------------------------------------------ backward kernels

// dy (N,K,P,Q) -> G [N][K][ldy]: output positions j = p*Wp + q of X's padded width, zeros for
// q >= Q and j >= P*Wp. grid (ceil(ldy / 4 / 128), up to 16 row slots per SM): a thread writes 4
// positions of every grid.y-th (image, filter) row; one multiply-shift division locates its first
// position, the others follow by wrapping q (no per-element integer division: the kernel was
// issue-bound).
__global__ void __launch_bounds__(128) conv_pack_grad_kernel(const float* __restrict__ dy, int P, int Q, int wp,
                                                             int ldy, long long rows, FastDiv div_wp,
                                                             float* __restrict__ hi, float* __restrict__ lo) {
    const int j0 = 4 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (j0 >= ldy) return;
    const int pr0 = static_cast<int>(fastdiv(static_cast<uint32_t>(j0), div_wp));
    const int q0 = j0 - pr0 * wp;
#pragma unroll 4
    for (long long row = blockIdx.y; row < rows; row += gridDim.y) {
        const float* src = dy + row * P * Q;
        int pr = pr0, q = q0;
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            v[e] = (pr < P && q < Q) ? __ldg(src + static_cast<long long>(pr) * Q + q) : 0.0f;
            if (++q == wp) {
                q = 0;
                ++pr;
            }
        }
        write_planes4(hi, lo, row * ldy + j0, v[0], v[1], v[2], v[3]);
    }
}

// dW[f][c][r][s] = sum over splits, in split order, of the partial tiles of the weight-gradient GEMM.
// Threads walk the partial rows (m = tap * cg + channel) with the filter index fastest, so a warp
// reads 128 contiguous bytes per split; the loads of 16 splits are issued before their adds,
// which stay in split order.
__global__ void conv_wgrad_reduce_kernel(const float* __restrict__ partial, int splits, long long rows_alloc,
                                         int ld_partial, int kf, int c, int taps, int cg, float* __restrict__ dw) {
    const long long total = static_cast<long long>(taps) * cg * kf;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int f = static_cast<int>(idx % kf);
        const long long m = idx / kf;
        const int tap = static_cast<int>(m / cg);
        const int ch = static_cast<int>(m - static_cast<long long>(tap) * cg);
        if (ch >= c) continue;
        const float* src = partial + m * ld_partial + f;
        const long long step = rows_alloc * ld_partial;
        float sum = 0.0f;
        int sp = 0;
        for (; sp + 16 <= splits; sp += 16) {
            float v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = src[(sp + u) * step];
#pragma unroll
            for (int u = 0; u < 16; ++u) sum += v[u];
        }
        for (; sp < splits; ++sp) sum += src[sp * step];
        dw[(static_cast<long long>(f) * c + ch) * taps + tap] = sum;
    }
}

// Direct restatements of the reference's backward kernels (src/nn/backward/convolution_kernels.cuh:9-82),
// one thread per output, FP32 FMA: other strides and problems too small for the tensor path.
__global__ void conv_bwd_data_direct_kernel(const float* __restrict__ grad, const float* __restrict__ wt,
                                            float* __restrict__ dx, int n, int c, int h, int w, int kf, int r, int s,
                                            int P, int Q, int stride, int pad) {
    const long long total = static_cast<long long>(n) * c * h * w;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int iw = static_cast<int>(idx % w);
        const int ih = static_cast<int>((idx / w) % h);
        const int ch = static_cast<int>((idx / (static_cast<long long>(w) * h)) % c);
        const long long img = idx / (static_cast<long long>(c) * h * w);
        float acc = 0.0f;
        for (int f = 0; f < kf; ++f)
            for (int kh = 0; kh < r; ++kh) {
                const int ohl = ih + pad - kh;
                if (ohl < 0 || ohl % stride != 0) continue;
                const int oh = ohl / stride;
                if (oh >= P) continue;
                for (int kw = 0; kw < s; ++kw) {
                    const int owl = iw + pad - kw;
                    if (owl < 0 || owl % stride != 0) continue;
                    const int ow = owl / stride;
                    if (ow >= Q) continue;
                    acc = fmaf(__ldg(grad + ((img * kf + f) * P + oh) * Q + ow),
                               __ldg(wt + ((static_cast<long long>(f) * c + ch) * r + kh) * s + kw), acc);
                }
            }
        dx[idx] = acc;
    }
}

__global__ void conv_bwd_filter_direct_kernel(const float* __restrict__ grad, const float* __restrict__ x,
                                              float* __restrict__ dw, int n, int c, int h, int w, int kf, int r,
                                              int s, int P, int Q, int stride, int pad) {
    const long long total = static_cast<long long>(kf) * c * r * s;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const int kw = static_cast<int>(idx % s);
        const int kh = static_cast<int>((idx / s) % r);
        const int ch = static_cast<int>((idx / (static_cast<long long>(s) * r)) % c);
        const int f = static_cast<int>(idx / (static_cast<long long>(c) * r * s));
        float acc = 0.0f;
        for (int img = 0; img < n; ++img)
            for (int oh = 0; oh < P; ++oh) {
                const int ih = oh * stride + kh - pad;
                if (ih < 0 || ih >= h) continue;
                for (int ow = 0; ow < Q; ++ow) {
                    const int iw = ow * stride + kw - pad;
                    if (iw < 0 || iw >= w) continue;
                    acc = fmaf(__ldg(grad + ((static_cast<long long>(img) * kf + f) * P + oh) * Q + ow),
                               __ldg(x + ((static_cast<long long>(img) * c + ch) * h + ih) * w + iw), acc);
                }
            }
        dw[idx] = acc;
    }
}

// dB[f] = sum over images, in image order, of the per-(image, filter) row sums. The loads of
// 16 images are issued before their adds, which stay in image order (one dependent load per
// image made the kernel L2-latency-bound).
__global__ void conv_bias_images_kernel(const float* __restrict__ row_sums, int n, int kf, float* __restrict__ db) {
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= kf) return;
    float acc = 0.0f;
    int img = 0;
    for (; img + 16 <= n; img += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = row_sums[static_cast<long long>(img + u) * kf + f];
#pragma unroll
        for (int u = 0; u < 16; ++u) acc += v[u];
    }
    for (; img < n; ++img) acc += row_sums[static_cast<long long>(img) * kf + f];
    db[f] = acc;
}

__global__ void conv_fill_kernel(float* __restrict__ p, long long count, float value) {
    for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<long long>(gridDim.x) * blockDim.x)
        p[i] = value;
}

// ------------------------------------------------------------------------------------ tcgen05 conv table
struct ConvEntry {
    int bn, planes;
    const void* fn;
    int smem, threads;
    int kslabs;  // 32-channel slabs per K block
};

template <int BN, int PLANES, int KS = 1>
ConvEntry make_conv_entry() {
    using P = ConvProblem<BN, PLANES, KS>;
    using L = TcLayout<P>;
    return ConvEntry{BN, PLANES, reinterpret_cast<const void*>(&tc_persistent_kernel<P>), L::kBytes, L::kThreads,
                     KS};
}

const ConvEntry* conv_table(int* count) {
    static const ConvEntry table[] = {
        // narrow tiles: 2 (strict) or 4 (TF32) 32-channel slabs per K block; wide tiles: 1
        make_conv_entry<16, 2, 2>(), make_conv_entry<32, 2, 2>(), make_conv_entry<64, 2, 2>(), make_conv_entry<128, 2>(),
        make_conv_entry<256, 2>(), make_conv_entry<16, 1, 4>(), make_conv_entry<32, 1, 4>(), make_conv_entry<64, 1, 4>(),
        make_conv_entry<128, 1>(), make_conv_entry<256, 1>(),
    };
    *count = static_cast<int>(sizeof(table) / sizeof(table[0]));
    return table;
}

// Narrowest filter tile that covers K (one filter tile per position tile when K <= 256).
const ConvEntry* pick_conv(int kf, int planes) {
    int count = 0;
    const ConvEntry* t = conv_table(&count);
    const ConvEntry* best = nullptr;
    for (int i = 0; i < count; ++i) {
        if (t[i].planes != planes) continue;
        if (t[i].bn >= kf && (!best || t[i].bn < best->bn)) best = &t[i];
    }
    if (!best)
        for (int i = 0; i < count; ++i)
            if (t[i].planes == planes && (!best || t[i].bn > best->bn)) best = &t[i];
    return best;
}

template <int BN, int PLANES, int KS = 1>
ConvEntry make_wgrad_entry() {
    using P = ConvWgradProblem<BN, PLANES, KS>;
    using L = TcLayout<P>;
    return ConvEntry{BN, PLANES, reinterpret_cast<const void*>(&tc_persistent_kernel<P>), L::kBytes, L::kThreads,
                     KS};
}

const ConvEntry* wgrad_table(int* count) {
    static const ConvEntry table[] = {
        make_wgrad_entry<64, 2, 2>(), make_wgrad_entry<128, 2>(), make_wgrad_entry<256, 2>(),
        make_wgrad_entry<64, 1, 2>(), make_wgrad_entry<128, 1>(), make_wgrad_entry<256, 1>(),
    };
    *count = static_cast<int>(sizeof(table) / sizeof(table[0]));
    return table;
}

// Narrowest filter tile covering K (64, 128 or 256 filters), else 256-filter tiles.
const ConvEntry* pick_wgrad(int kf, int planes) {
    int count = 0;
    const ConvEntry* t = wgrad_table(&count);
    const ConvEntry* best = nullptr;
    for (int i = 0; i < count; ++i)
        if (t[i].planes == planes && t[i].bn >= kf && (!best || t[i].bn < best->bn)) best = &t[i];
    if (!best)
        for (int i = 0; i < count; ++i)
            if (t[i].planes == planes && (!best || t[i].bn > best->bn)) best = &t[i];
    return best;
}

long long round_up64(long long v) { return (v + 63) / 64 * 64; }

}  // namespace

struct ConvGeom {
    int n, c, h, w, k, r, s, pad_h, pad_w;
};

size_t conv_tc_workspace_bytes(const ConvGeom& g, int precision) {
    const long long planes = precision == MFB_PRECISION_FP32 ? 2 : 1;
    const long long cp = (g.c + 3) / 4 * 4;
    const long long a = round_up64(static_cast<long long>(g.n) * (g.h + 2 * g.pad_h) * (g.w + 2 * g.pad_w) * cp);
    const long long b = round_up64(static_cast<long long>(g.r) * g.s * g.k * cp);
    return static_cast<size_t>(planes * (a + b) * 4);
}

// Stride-1 implicit GEMM on tcgen05: y (N,K,P,Q) = bias + x (N,C,H,W) correlated with the filter
// bank, P = H + 2 pad_h - R + 1, Q = W + 2 pad_w - S + 1. flip selects the packing of `wgt`
// (conv_pack_weights_kernel); bias may be null.
mfb_status_t conv_tc_forward(int device, cudaStream_t stream, const ConvGeom& g, const float* x, const float* wgt,
                             int flip, const float* bias, float* y, int precision) {
    const int n = g.n, c = g.c, h = g.h, w = g.w, k = g.k, r = g.r, s = g.s;
    const int P = h + 2 * g.pad_h - r + 1;
    const int Q = w + 2 * g.pad_w - s + 1;
    const int planes = precision == MFB_PRECISION_FP32 ? 2 : 1;
    const int cp = (c + 3) / 4 * 4;
    const int hp = h + 2 * g.pad_h, wp = w + 2 * g.pad_w;
    const long long npos = static_cast<long long>(hp) * wp;
    if (n > 65535 || npos > 0x7fffffffLL) return fail(MFB_EUNSUPPORTED, "conv2d input too large");
    const ConvEntry* e = pick_conv(k, planes);
    if (!e) return fail(MFB_EUNSUPPORTED, "no tcgen05 conv configuration");

    const size_t need = conv_tc_workspace_bytes(g, precision);
    void* ws = nullptr;
    MFB_TRY(stream_workspace(device, stream, need, &ws));
    const long long a_plane = round_up64(static_cast<long long>(n) * npos * cp);
    const long long b_plane = round_up64(static_cast<long long>(r) * s * k * cp);
    float* a_hi = static_cast<float*>(ws);
    float* a_lo = planes == 2 ? a_hi + a_plane : nullptr;
    float* b_hi = a_hi + planes * a_plane;
    float* b_lo = planes == 2 ? b_hi + b_plane : nullptr;
    if (wp <= kPackMaxWp) {
        const size_t tile_bytes = pack_rows_smem_bytes(w);
        MFB_TRY(allow_pack_rows_smem());
        const int vec = (w % 2 == 0 && (reinterpret_cast<uintptr_t>(x) & 7u) == 0) ? 1 : 0;
        dim3 pgrid(static_cast<unsigned>((hp + kPackRows - 1) / kPackRows), static_cast<unsigned>((cp + 31) / 32), n);
        conv_pack_rows_kernel<<<pgrid, 256, tile_bytes, stream>>>(x, c, h, w, g.pad_h, g.pad_w, cp, hp, wp, vec,
                                                                 a_hi, a_lo);
    } else {
        dim3 pgrid(static_cast<unsigned>((npos + 63) / 64), static_cast<unsigned>((cp + 31) / 32), n);
        conv_pack_input_kernel<<<pgrid, 256, 0, stream>>>(x, c, h, w, g.pad_h, g.pad_w, cp, hp, wp, a_hi, a_lo);
    }
    MFB_CUDA_TRY(cudaGetLastError(), "conv input prepass launch");
    const long long wgroups = static_cast<long long>(r) * s * k * (cp / 4);
    conv_pack_weights_kernel<<<static_cast<int>(std::min<long long>((wgroups + 255) / 256, static_cast<long long>(current_sm_count()) * 4)), 256, 0,
                               stream>>>(wgt, k, c, r, s, cp, flip, b_hi, b_lo);
    MFB_CUDA_TRY(cudaGetLastError(), "conv weight prepass launch");

    // X: dims (Cp, Hp*Wp, N, planes); W: dims (Cp, K, R*S, planes); boxes of 32 channels.
    CUtensorMap map_a, map_b;
    {
        const uint64_t dims[4] = {static_cast<uint64_t>(cp), static_cast<uint64_t>(npos), static_cast<uint64_t>(n),
                                  static_cast<uint64_t>(planes)};
        const uint64_t strides[3] = {static_cast<uint64_t>(cp) * 4, static_cast<uint64_t>(npos) * cp * 4,
                                     static_cast<uint64_t>(a_plane) * 4};
        const uint32_t box[4] = {32, static_cast<uint32_t>(kTcBM), 1, static_cast<uint32_t>(planes)};
        MFB_TRY(encode_tensor_map(&map_a, a_hi, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B));
    }
    {
        const uint64_t dims[4] = {static_cast<uint64_t>(cp), static_cast<uint64_t>(k), static_cast<uint64_t>(r) * s,
                                  static_cast<uint64_t>(planes)};
        const uint64_t strides[3] = {static_cast<uint64_t>(cp) * 4, static_cast<uint64_t>(k) * cp * 4,
                                     static_cast<uint64_t>(b_plane) * 4};
        const uint32_t box[4] = {32, static_cast<uint32_t>(e->bn), 1, static_cast<uint32_t>(planes)};
        MFB_TRY(encode_tensor_map(&map_b, b_hi, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B));
    }

    ConvTcParams p{};
    p.n_img = n;
    p.c = c;
    p.h = h;
    p.w = w;
    p.kf = k;
    p.r = r;
    p.s = s;
    p.pad = g.pad_h;
    p.hp = hp;
    p.wp = wp;
    p.p_out = P;
    p.q_out = Q;
    p.ncb = (cp + 31) / 32;  // 32-channel slabs per tap
    p.num_kb = (r * s * p.ncb + e->kslabs - 1) / e->kslabs;
    p.div_ncb = make_fastdiv(static_cast<uint32_t>(p.ncb));
    p.div_s = make_fastdiv(static_cast<uint32_t>(s));
    p.tiles_pos = static_cast<int>((static_cast<long long>(P) * wp + kTcBM - 1) / kTcBM);
    p.tiles_f = (k + e->bn - 1) / e->bn;
    p.y = y;
    p.bias = bias;
    p.wait_limit_ns = wait_limit_ns();
    const long long tiles = static_cast<long long>(n) * p.tiles_pos * p.tiles_f;
    if (tiles > 0x7fffffffLL) return fail(MFB_EINVAL, "conv2d has too many output tiles");
    const int grid = static_cast<int>(std::min<long long>(tiles, sm_count(device)));
    static std::mutex attr_mutex;
    {
        std::lock_guard<std::mutex> lock(attr_mutex);
        MFB_CUDA_TRY(cudaFuncSetAttribute(e->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, e->smem),
                     "conv smem attribute");
    }
    void* args[] = {&map_a, &map_b, &p};
    MFB_CUDA_TRY(cudaLaunchKernel(e->fn, dim3(grid), dim3(e->threads), args, static_cast<size_t>(e->smem), stream),
                 "tcgen05 conv launch");
    return MFB_OK;
}


size_t conv2d_workspace_bytes(int n, int c, int h, int w, int k, int r, int s, int stride, int pad, int precision) {
    if (stride != 1) return 0;
    return conv_tc_workspace_bytes(ConvGeom{n, c, h, w, k, r, s, pad, pad}, precision);
}

mfb_status_t conv2d_launch(int device, cudaStream_t stream, int n, int c, int h, int w, int k, int r, int s,
                           int stride, int pad, const float* x, const float* wgt, const float* bias, float* y,
                           int precision) {
    const int P = (h + 2 * pad - r) / stride + 1;
    const int Q = (w + 2 * pad - s) / stride + 1;
    if (n == 0 || P <= 0 || Q <= 0) return MFB_OK;
    // Other strides, and problems too small to amortize the tensor path (conv_use_direct):
    // the direct kernel, one launch, FP32 FMA chains in the reference's order (at least as
    // accurate as either precision policy asks).
    const double flops = 2.0 * n * k * P * Q * static_cast<double>(c) * r * s;
    if (conv_use_direct(stride, flops, c))
        return conv2d_direct(stream, n, c, h, w, k, r, s, stride, pad, P, Q, x, wgt, bias, y);
    return conv_tc_forward(device, stream, ConvGeom{n, c, h, w, k, r, s, pad, pad}, x, wgt, 0, bias, y, precision);
}

mfb_status_t conv2d_bwd_data_launch(int device, cudaStream_t stream, int n, int c, int h, int w, int k, int r, int s,
                                    int stride, int pad, const float* dy, const float* wgt, float* dx,
                                    int precision) {
    const int P = (h + 2 * pad - r) / stride + 1;
    const int Q = (w + 2 * pad - s) / stride + 1;
    if (n == 0) return MFB_OK;
    const double flops = 2.0 * n * k * P * Q * static_cast<double>(c) * r * s;
    // Stride 1: dX is the forward correlation of dY (K channels, P x Q) with the transposed,
    // flipped filters and padding (R-1-pad, S-1-pad): P + R - 1 - 2 pad = H rows out.
    if (stride == 1 && pad <= r - 1 && pad <= s - 1 && flops >= kConvDirectMaxFlops)
        return conv_tc_forward(device, stream, ConvGeom{n, k, P, Q, c, r, s, r - 1 - pad, s - 1 - pad}, dy, wgt, 1,
                               nullptr, dx, precision);
    const long long total = static_cast<long long>(n) * c * h * w;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, static_cast<long long>(current_sm_count()) * 16));
    conv_bwd_data_direct_kernel<<<blocks, 256, 0, stream>>>(dy, wgt, dx, n, c, h, w, k, r, s, P, Q, stride, pad);
    MFB_CUDA_TRY(cudaGetLastError(), "conv2d input-gradient launch");
    return MFB_OK;
}

mfb_status_t conv2d_bwd_filter_launch(int device, cudaStream_t stream, int n, int c, int h, int w, int k, int r,
                                      int s, int stride, int pad, const float* x, const float* dy, float* dw,
                                      int precision) {
    const int P = (h + 2 * pad - r) / stride + 1;
    const int Q = (w + 2 * pad - s) / stride + 1;
    const long long wtotal = static_cast<long long>(k) * c * r * s;
    const double flops = 2.0 * n * k * P * Q * static_cast<double>(c) * r * s;
    if (n == 0) {  // an empty batch contributes nothing: dW = 0
        MFB_CUDA_TRY(cudaMemsetAsync(dw, 0, static_cast<size_t>(wtotal) * 4, stream), "dW clear");
        return MFB_OK;
    }
    const int planes = precision == MFB_PRECISION_FP32 ? 2 : 1;
    const int hp = h + 2 * pad, wp = w + 2 * pad;
    const long long npos = static_cast<long long>(hp) * wp;
    const long long gpos = static_cast<long long>(P) * wp;
    const ConvEntry* e = pick_wgrad(k, planes);
    // The producer indexes K blocks within a split as 32-bit values: n * P * Wp / 32 < 2^30 keeps
    // them below 2^31 (the planes of any problem that fits in device memory are far smaller).
    const bool tensor = stride == 1 && flops >= kConvDirectMaxFlops && e != nullptr && n <= 65535 &&
                        npos <= 0x7fffffffLL && gpos <= 0x7fffffffLL && n * ((gpos + 31) / 32) < (1LL << 30);
    if (!tensor) {
        const int blocks = static_cast<int>(std::min<long long>((wtotal + 127) / 128, static_cast<long long>(current_sm_count()) * 16));
        conv_bwd_filter_direct_kernel<<<blocks, 128, 0, stream>>>(dy, x, dw, n, c, h, w, k, r, s, P, Q, stride, pad);
        MFB_CUDA_TRY(cudaGetLastError(), "conv2d weight-gradient launch");
        return MFB_OK;
    }
    const int cp = (c + 3) / 4 * 4;
    const int cg = (c + 31) / 32 * 32;
    const int ldy = static_cast<int>((gpos + 3) / 4 * 4);
    ConvWgradParams p{};
    p.n_img = n;
    p.c = c;
    p.kf = k;
    p.r = r;
    p.s = s;
    p.cg = cg;
    p.wp = wp;
    p.kb_per_img = static_cast<int>((gpos + 32 * e->kslabs - 1) / (32 * e->kslabs));
    p.div_kb_per_img = make_fastdiv(static_cast<uint32_t>(p.kb_per_img));
    p.rows_total = r * s * cg;
    p.tiles_m = (p.rows_total + kTcBM - 1) / kTcBM;
    p.tiles_f = (k + e->bn - 1) / e->bn;
    p.ld_partial = p.tiles_f * e->bn;
    const long long total_kb = static_cast<long long>(n) * p.kb_per_img;
    // Equal-length work units filling whole waves of the persistent grid: splits * tiles just
    // under a multiple of the SM count (4 waves), each split at least 16 K blocks long.
    const int sms = sm_count(device);
    const long long out_tiles = static_cast<long long>(p.tiles_m) * p.tiles_f;
    long long splits = std::max(1LL, (4LL * sms) / out_tiles);
    splits = std::max(1LL, std::min(splits, total_kb / 16));
    const long long kbs = (total_kb + splits - 1) / splits;
    splits = (total_kb + kbs - 1) / kbs;
    p.kb_per_split = static_cast<int>(kbs);
    p.splits = static_cast<int>(splits);
    p.wait_limit_ns = wait_limit_ns();
    const long long rows_alloc = static_cast<long long>(p.tiles_m) * kTcBM;

    const long long a_plane = round_up64(static_cast<long long>(n) * npos * cp);
    const long long g_plane = round_up64(static_cast<long long>(n) * k * ldy);
    const long long part = round_up64(splits * rows_alloc * p.ld_partial);
    const size_t need = static_cast<size_t>((planes * (a_plane + g_plane) + part) * 4);
    void* ws = nullptr;
    MFB_TRY(stream_workspace(device, stream, need, &ws));
    float* a_hi = static_cast<float*>(ws);
    float* a_lo = planes == 2 ? a_hi + a_plane : nullptr;
    float* g_hi = a_hi + planes * a_plane;
    float* g_lo = planes == 2 ? g_hi + g_plane : nullptr;
    p.partial = g_hi + planes * g_plane;

    // X planes (as the forward), dY planes in X's padded width.
    if (wp <= kPackMaxWp) {
        const size_t tile_bytes = pack_rows_smem_bytes(w);
        MFB_TRY(allow_pack_rows_smem());
        const int vec = (w % 2 == 0 && (reinterpret_cast<uintptr_t>(x) & 7u) == 0) ? 1 : 0;
        dim3 pgrid(static_cast<unsigned>((hp + kPackRows - 1) / kPackRows), static_cast<unsigned>((cp + 31) / 32), n);
        conv_pack_rows_kernel<<<pgrid, 256, tile_bytes, stream>>>(x, c, h, w, pad, pad, cp, hp, wp, vec, a_hi, a_lo);
    } else {
        dim3 pgrid(static_cast<unsigned>((npos + 63) / 64), static_cast<unsigned>((cp + 31) / 32), n);
        conv_pack_input_kernel<<<pgrid, 256, 0, stream>>>(x, c, h, w, pad, pad, cp, hp, wp, a_hi, a_lo);
    }
    MFB_CUDA_TRY(cudaGetLastError(), "wgrad input prepass launch");
    const long long grad_rows = static_cast<long long>(n) * k;
    dim3 ggrid(static_cast<unsigned>((ldy / 4 + 127) / 128), static_cast<unsigned>(std::min(grad_rows, static_cast<long long>(current_sm_count()) * 16)));
    conv_pack_grad_kernel<<<ggrid, 128, 0, stream>>>(dy, P, Q, wp, ldy, grad_rows,
                                                     make_fastdiv(static_cast<uint32_t>(wp)), g_hi, g_lo);
    MFB_CUDA_TRY(cudaGetLastError(), "wgrad gradient prepass launch");

    CUtensorMap map_a, map_b;
    {
        // X planes read MN-major: channels innermost, 32-channel x 32-position boxes.
        const uint64_t dims[4] = {static_cast<uint64_t>(cp), static_cast<uint64_t>(npos), static_cast<uint64_t>(n),
                                  static_cast<uint64_t>(planes)};
        const uint64_t strides[3] = {static_cast<uint64_t>(cp) * 4, static_cast<uint64_t>(npos) * cp * 4,
                                     static_cast<uint64_t>(a_plane) * 4};
        const uint32_t box[4] = {32, 32, 1, static_cast<uint32_t>(planes)};
        MFB_TRY(encode_tensor_map(&map_a, a_hi, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B));
    }
    {
        const uint64_t dims[4] = {static_cast<uint64_t>(gpos), static_cast<uint64_t>(k), static_cast<uint64_t>(n),
                                  static_cast<uint64_t>(planes)};
        const uint64_t strides[3] = {static_cast<uint64_t>(ldy) * 4, static_cast<uint64_t>(k) * ldy * 4,
                                     static_cast<uint64_t>(g_plane) * 4};
        const uint32_t box[4] = {32, static_cast<uint32_t>(e->bn), 1, static_cast<uint32_t>(planes)};
        MFB_TRY(encode_tensor_map(&map_b, g_hi, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B));
    }
    const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_f * p.splits;
    if (tiles > 0x7fffffffLL) return fail(MFB_EINVAL, "weight gradient has too many work units");
    static std::mutex attr_mutex;
    {
        std::lock_guard<std::mutex> lock(attr_mutex);
        MFB_CUDA_TRY(cudaFuncSetAttribute(e->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, e->smem),
                     "wgrad smem attribute");
    }
    void* args[] = {&map_a, &map_b, &p};
    const int grid = static_cast<int>(std::min<long long>(tiles, sms));
    MFB_CUDA_TRY(cudaLaunchKernel(e->fn, dim3(grid), dim3(e->threads), args, static_cast<size_t>(e->smem), stream),
                 "tcgen05 weight-gradient launch");
    const int rblocks = static_cast<int>(std::min<long long>((wtotal + 255) / 256, static_cast<long long>(current_sm_count()) * 8));
    conv_wgrad_reduce_kernel<<<rblocks, 256, 0, stream>>>(p.partial, p.splits, rows_alloc, p.ld_partial, k, c, r * s,
                                                          cg, dw);
    MFB_CUDA_TRY(cudaGetLastError(), "wgrad reduce launch");
    return MFB_OK;
}

// dB: the (N*K) x (P*Q) matrix dY times a ones vector on the GEMV path (row sums at the HBM
// rate), then the images summed per filter in image order. Deterministic.
mfb_status_t conv2d_bwd_bias_launch(int device, cudaStream_t stream, int n, int k, int P, int Q, const float* dy,
                                    float* db) {
    if (k == 0) return MFB_OK;
    const long long plane = static_cast<long long>(P) * Q;
    const long long rows = static_cast<long long>(n) * k;
    if (rows == 0 || plane == 0) {
        MFB_CUDA_TRY(cudaMemsetAsync(db, 0, static_cast<size_t>(k) * 4, stream), "dB clear");
        return MFB_OK;
    }
    if (rows > 0x7fffffffLL || plane > 0x7fffffffLL) return fail(MFB_EUNSUPPORTED, "conv2d bias gradient too large");
    mfb_gemm_desc d{};
    d.m = static_cast<int>(rows);
    d.n = 1;
    d.k = static_cast<int>(plane);
    d.lda = d.k;
    d.ldb = 1;
    d.ldc = 1;
    d.alpha = 1.0f;
    d.beta = 0.0f;
    d.precision = MFB_PRECISION_FP32;
    const size_t ones_bytes = static_cast<size_t>((plane + 63) / 64 * 64) * 4;
    const size_t sums_bytes = static_cast<size_t>((rows + 63) / 64 * 64) * 4;
    const size_t gemv_bytes = gemv_workspace_bytes(d);
    void* ws = nullptr;
    MFB_TRY(stream_workspace(device, stream, ones_bytes + sums_bytes + gemv_bytes, &ws));
    float* ones = static_cast<float*>(ws);
    float* sums = ones + ones_bytes / 4;
    void* gemv_ws = gemv_bytes ? static_cast<void*>(sums + sums_bytes / 4) : nullptr;
    conv_fill_kernel<<<static_cast<int>(std::min<long long>((plane + 255) / 256, static_cast<long long>(current_sm_count()) * 4)), 256, 0, stream>>>(
        ones, plane, 1.0f);
    MFB_CUDA_TRY(cudaGetLastError(), "dB ones launch");
    MFB_TRY(gemv_launch(d, stream, dy, ones, sums, nullptr, gemv_ws, gemv_bytes));
    conv_bias_images_kernel<<<(k + 255) / 256, 256, 0, stream>>>(sums, n, k, db);
    MFB_CUDA_TRY(cudaGetLastError(), "dB image-sum launch");
    return MFB_OK;
}

}  // namespace mfb
