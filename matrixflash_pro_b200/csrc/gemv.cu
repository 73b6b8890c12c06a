// Bandwidth-bound FP32 GEMV / skinny GEMM (strict FP32 FMA arithmetic).
//
// Replaces gemm_gemv (src/ops/gemm/gemm_gemv.cu:86-110): gemv_rows_kernel (:10),
// gemm_skinny_n_kernel (:30) and gemv_cols_kernel (:61), which read A with scalar
// 4-byte loads, handle only contiguous alpha=1/beta=0 operands and n <= 4.
//
// tile kernel (n <= 16, 16-byte aligned operands): described at gemv_tile_kernel below;
// it streams A at 86-98% of the measured HBM rate on the 16384 x 16384 GEMV.
//
// rows kernel (other n <= 16 operands): each warp owns R rows; lanes walk K with 128-bit loads of
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
#include <mutex>

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

// ------------------------------------------------------------------------------------
// Tile kernel for 4 < n <= 16 (A and B 16-byte aligned, lda and ldb multiples of 4).
//
// At n = 16 every element of A feeds 16 FMAs, so the rows kernel above (which re-stages
// all of x per 16-row block and reads it lane-strided) runs out of shared-memory and
// L2 bandwidth long before HBM. Here each CTA owns one tile of about m / #SMs rows for
// the whole of K. A producer warp streams A[tile][32 KB k] (TMA, KB boxes of 128-byte
// rows, 128-byte swizzle) and x[32 KB k][NC] (TMA, zero fill beyond n and k) through an
// S-stage ring. All W consumer warps work on the same stage, each on 32 KB / W of its k,
// so a stage is held only for 1/W of its compute time and nearly the whole ring is in
// flight to HBM. The lanes form CH groups of 32 / CH; lane l of group h owns rows
// l + (32 / CH) i (i < R) and columns [h NC / CH, (h + 1) NC / CH): an x value is a
// broadcast read within the group, reused for R rows. FMAs are packed pairs
// (fma.rn.f32x2, the same rounding as fmaf). The W per-warp partial sums are reduced in
// shared memory in warp order (deterministic) and alpha/beta/bias/activation are
// applied on the way out.
// ------------------------------------------------------------------------------------
constexpr int kGtBoxK = 32;  // K per TMA box of A: 128-byte rows, one SWIZZLE_128B span

struct GemvTileParams {
    float* c;
    const float* bias;
    long long ldc;
    int m, n, k;
    int tile_rows;
    float alpha, beta;
    int epilogue;
    uint64_t wait_limit_ns;
};

template <int NC, int CH, int R, int W, int S, int KB>
struct GemvTileLayout {
    static constexpr int kKc = kGtBoxK * KB;  // K per stage
    static constexpr int kGroup = 32 / CH;    // lanes per column group
    static constexpr int kCols = NC / CH;     // columns per lane
    static constexpr int kRows = kGroup * R;  // rows one tile can hold
    static constexpr int kChunks = kKc / 4 / W;  // 16-byte k chunks per warp and stage
    static constexpr int kABox = kRows * kGtBoxK * 4;
    static constexpr int kAStage = KB * kABox;
    static constexpr int kXStage = kKc * NC * 4;
    static constexpr int kRedStride = NC + 1;  // odd row stride: lane-strided writes hit distinct banks
    static constexpr int kRedBytes = W * kRows * kRedStride * 4;
    static constexpr int kAOff = 0;
    static constexpr int kXOff = kAOff + S * kAStage;
    static constexpr int kRedOff = kXOff + S * kXStage;
    static constexpr int kBarOff = kRedOff + kRedBytes;  // full[S], empty[S]
    static constexpr int kAbortOff = kBarOff + 2 * S * 8;
    static constexpr int kSmem = kAbortOff + 16 + 1024;  // + slack to align the base to 1024 bytes
    static constexpr int kThreads = (W + 1) * 32;
    static_assert(kABox % 1024 == 0, "SWIZZLE_128B boxes must stay 1024-byte aligned");
    static_assert((NC == 1 || kCols % 4 == 0) && kGroup % 8 == 0, "float4 column groups, 8-row swizzle period");
    static_assert(kChunks >= 1 && kChunks * W * 4 == kKc, "the warps split a stage's k evenly");
    static_assert(kBarOff % 8 == 0, "mbarriers need 8-byte alignment");
    static_assert(kSmem <= 232448, "shared memory per CTA");
};

__device__ __forceinline__ void consumer_bar_sync(int threads) {
    asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// c0 += a * x0 and c1 += a * x1 as one packed f32x2 FMA (round to nearest, like fmaf).
__device__ __forceinline__ void fma_pair(float& c0, float& c1, float a, float x0, float x1) {
    asm("{\n\t.reg .b64 ra, rx, rc;\n\t"
        "mov.b64 ra, {%2, %2};\n\t"
        "mov.b64 rx, {%3, %4};\n\t"
        "mov.b64 rc, {%0, %1};\n\t"
        "fma.rn.f32x2 rc, ra, rx, rc;\n\t"
        "mov.b64 {%0, %1}, rc;\n\t}"
        : "+f"(c0), "+f"(c1)
        : "f"(a), "f"(x0), "f"(x1));
}

template <int NC, int CH, int R, int W, int S, int KB>
__global__ void __launch_bounds__((W + 1) * 32, 1)
    gemv_tile_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_x,
                     GemvTileParams p) {
    using L = GemvTileLayout<NC, CH, R, W, S, KB>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
    uint64_t* empty = full + S;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kAbortOff);
    float* red = reinterpret_cast<float*>(smem + L::kRedOff);
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int nk = (p.k + L::kKc - 1) / L::kKc;
    const int tiles = (p.m + p.tile_rows - 1) / p.tile_rows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == W) {  // TMA producer
        if (lane == 0) {
            tma_prefetch_desc(&tmap_a);
            tma_prefetch_desc(&tmap_x);
            const uint32_t bytes = static_cast<uint32_t>(KB * p.tile_rows * kGtBoxK * 4 + L::kXStage);
            long long g = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                for (int j = 0; j < nk; ++j, ++g) {
                    const int s = static_cast<int>(g % S);
                    if (!mbar_wait_bounded(&empty[s], static_cast<uint32_t>((g / S) & 1) ^ 1u, p.wait_limit_ns,
                                           abort_flag)) {
                        report_status(kStatusTimeoutProducer, abort_flag);
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], bytes);
#pragma unroll
                    for (int b = 0; b < KB; ++b)
                        tma_load_2d(smem + L::kAOff + s * L::kAStage + b * L::kABox, &tmap_a, &full[s],
                                    j * L::kKc + b * kGtBoxK, t * p.tile_rows);
                    if constexpr (NC == 1)  // x as one row of k values
                        tma_load_2d(smem + L::kXOff + s * L::kXStage, &tmap_x, &full[s], j * L::kKc, 0);
                    else
                        tma_load_2d(smem + L::kXOff + s * L::kXStage, &tmap_x, &full[s], 0, j * L::kKc);
                }
            }
            // Teardown: no copy may land after the CTA has exited.
            for (long long q = g > S ? g - S : 0; q < g; ++q) {
                if (!mbar_wait_drain(&full[q % S], static_cast<uint32_t>((q / S) & 1), p.wait_limit_ns)) {
                    report_status(kStatusTimeoutDrain, abort_flag);
                    break;
                }
            }
        }
        return;
    }

    // Consumers. SWIZZLE_128B moves 16-byte chunk j of a 128-byte row r to chunk j ^ (r & 7);
    // rows rl + kGroup i share rl & 7 (kGroup is a multiple of 8).
    const int rl = lane % L::kGroup;
    const int col0 = (lane / L::kGroup) * L::kCols;
    const int sw = rl & 7;
    bool ok = true;
    long long g = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        float acc[R][L::kCols];
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
            for (int q = 0; q < L::kCols; ++q) acc[i][q] = 0.0f;

        for (int j = 0; j < nk && ok; ++j, ++g) {
            const int s = static_cast<int>(g % S);
            const bool got = mbar_wait_bounded(&full[s], static_cast<uint32_t>((g / S) & 1), p.wait_limit_ns,
                                               abort_flag);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) report_status(kStatusTimeoutMma, abort_flag);
                ok = false;
                break;
            }
            const float* a_st = reinterpret_cast<const float*>(smem + L::kAOff + s * L::kAStage);
            const float* x_st = reinterpret_cast<const float*>(smem + L::kXOff + s * L::kXStage);
#pragma unroll
            for (int cq = 0; cq < L::kChunks; ++cq) {
                const int kq = warp * L::kChunks + cq;  // this warp's 16-byte chunk of the stage
                const float* a_box = a_st + (kq / 8) * (L::kABox / 4);
                float4 av[R];
#pragma unroll
                for (int i = 0; i < R; ++i)
                    av[i] = *reinterpret_cast<const float4*>(a_box + (rl + L::kGroup * i) * kGtBoxK +
                                                             (((kq % 8) ^ sw) << 2));
                if constexpr (NC == 1) {
                    // x is one contiguous column: the chunk's 4 k values in one broadcast read.
                    const float4 xv = *reinterpret_cast<const float4*>(x_st + kq * 4);
#pragma unroll
                    for (int i = 0; i < R; ++i) {
                        acc[i][0] = fmaf(av[i].x, xv.x, acc[i][0]);
                        acc[i][0] = fmaf(av[i].y, xv.y, acc[i][0]);
                        acc[i][0] = fmaf(av[i].z, xv.z, acc[i][0]);
                        acc[i][0] = fmaf(av[i].w, xv.w, acc[i][0]);
                    }
                } else {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
                        for (int c4 = 0; c4 < L::kCols / 4; ++c4) {
                            const float4 xv =
                                *reinterpret_cast<const float4*>(x_st + (kq * 4 + kk) * NC + col0 + c4 * 4);
#pragma unroll
                            for (int i = 0; i < R; ++i) {
                                const float a = kk == 0 ? av[i].x : kk == 1 ? av[i].y : kk == 2 ? av[i].z : av[i].w;
                                float* c = &acc[i][c4 * 4];
                                fma_pair(c[0], c[1], a, xv.x, xv.y);
                                fma_pair(c[2], c[3], a, xv.z, xv.w);
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }

        // Cross-warp reduction in warp order, then the fused epilogue. Every consumer warp
        // passes both barriers of every tile, also after a timeout.
        float* rw = red + warp * L::kRows * L::kRedStride;
#pragma unroll
        for (int i = 0; i < R; ++i)
#pragma unroll
            for (int q = 0; q < L::kCols; ++q) rw[(rl + L::kGroup * i) * L::kRedStride + col0 + q] = acc[i][q];
        consumer_bar_sync(W * 32);
        const int row0 = t * p.tile_rows;
        const int rows = min(p.tile_rows, p.m - row0);
        if (ok) {
            for (int o = threadIdx.x; o < rows * p.n; o += W * 32) {
                const int r = o / p.n;
                const int q = o - r * p.n;
                float v = 0.0f;
#pragma unroll
                for (int w = 0; w < W; ++w) v += red[(w * L::kRows + r) * L::kRedStride + q];
                float* dst = p.c + static_cast<long long>(row0 + r) * p.ldc + q;
                float out = p.alpha * v;
                if (p.beta != 0.0f) out = fmaf(p.beta, *dst, out);
                *dst = apply_epilogue_op(out, p.bias, q, p.epilogue);
            }
        }
        consumer_bar_sync(W * 32);
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
#pragma unroll 8
    for (int p = k0; p < k1; ++p) {  // unrolled: eight row loads in flight per thread
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
    // Split order; the loads of 16 splits are issued before their adds (one dependent load per
    // split left this kernel L2-latency-bound).
    float s = 0.0f;
    int i = 0;
    for (; i + 16 <= splits; i += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = partial[static_cast<long long>(i + u) * n + col];
#pragma unroll
        for (int u = 0; u < 16; ++u) s += v[u];
    }
    for (; i < splits; ++i) s += partial[static_cast<long long>(i) * n + col];
    float o = alpha * s;
    if (beta != 0.0f) o = fmaf(beta, c[col], o);
    c[col] = apply_epilogue_op(o, bias, col, epilogue);
}

// x^T for m == 1 lives in A's single row (lda irrelevant); it must be contiguous.
int cols_splits(int n, int k) {
    const int col_blocks = (n + 511) / 512;
    int splits = std::max(1, (current_sm_count() * 8) / std::max(1, col_blocks));  // ~8 blocks of 4 warps per SM
    splits = std::min(splits, std::max(1, k / 32));
    return std::min(splits, 1024);
}

template <int NC, int R>
void launch_rows(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                 const float* bias, int a_vec) {
    constexpr int kRowsPerBlock = (kGemvThreads / 32) * R;
    const long long row_blocks = (static_cast<long long>(d.m) + kRowsPerBlock - 1) / kRowsPerBlock;
    const int grid = static_cast<int>(std::min<long long>(row_blocks, static_cast<long long>(current_sm_count()) * 8));
    gemv_rows_kernel<NC, R><<<grid, kGemvThreads, 0, stream>>>(a, d.lda, b, d.ldb, c, d.ldc, d.m, d.n, d.k,
                                                               d.alpha, d.beta, bias, d.epilogue, a_vec);
}

// Rows per tile: balanced over the SMs (every CTA gets the same number of tiles), a
// multiple of 8, at most 128 (4 rows per lane).
int gemv_tile_rows(int m, int sms) {
    const long long cap = 128;
    const long long per_cta = (static_cast<long long>(m) + sms - 1) / sms;
    const long long tiles_per_cta = (per_cta + cap - 1) / cap;
    long long rows = (static_cast<long long>(m) + sms * tiles_per_cta - 1) / (sms * tiles_per_cta);
    rows = (rows + 7) / 8 * 8;
    return static_cast<int>(std::min(cap, std::max(8LL, rows)));
}

template <int NC, int CH, int R, int W, int S, int KB>
mfb_status_t launch_tile(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                         const float* bias, int tile_rows, int sms) {
    using L = GemvTileLayout<NC, CH, R, W, S, KB>;
    CUtensorMap map_a, map_x;
    {
        const uint64_t dims[2] = {static_cast<uint64_t>(d.k), static_cast<uint64_t>(d.m)};
        const uint64_t strides[1] = {static_cast<uint64_t>(d.lda) * 4};
        const uint32_t box[2] = {static_cast<uint32_t>(kGtBoxK), static_cast<uint32_t>(tile_rows)};
        MFB_TRY(encode_tensor_map(&map_a, a, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B));
    }
    if constexpr (NC == 1) {  // contiguous x (ldb == 1): a 1 x k tensor
        const uint64_t dims[2] = {static_cast<uint64_t>(d.k), 1};
        const uint64_t strides[1] = {(static_cast<uint64_t>(d.k) * 4 + 15) / 16 * 16};
        const uint32_t box[2] = {static_cast<uint32_t>(L::kKc), 1};
        MFB_TRY(encode_tensor_map(&map_x, b, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE));
    } else {
        const uint64_t dims[2] = {static_cast<uint64_t>(d.n), static_cast<uint64_t>(d.k)};
        const uint64_t strides[1] = {static_cast<uint64_t>(d.ldb) * 4};
        const uint32_t box[2] = {static_cast<uint32_t>(NC), static_cast<uint32_t>(L::kKc)};
        MFB_TRY(encode_tensor_map(&map_x, b, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE));
    }
    GemvTileParams p;
    p.c = c;
    p.bias = bias;
    p.ldc = d.ldc;
    p.m = d.m;
    p.n = d.n;
    p.k = d.k;
    p.tile_rows = tile_rows;
    p.alpha = d.alpha;
    p.beta = d.beta;
    p.epilogue = d.epilogue;
    p.wait_limit_ns = wait_limit_ns();
    auto fn = gemv_tile_kernel<NC, CH, R, W, S, KB>;
    static std::mutex attr_mutex;
    {
        std::lock_guard<std::mutex> lock(attr_mutex);
        MFB_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmem),
                     "cudaFuncSetAttribute(GEMV tile smem)");
    }
    const int tiles = (d.m + tile_rows - 1) / tile_rows;
    const int grid = std::min(tiles, sms);
    fn<<<grid, L::kThreads, L::kSmem, stream>>>(map_a, map_x, p);
    MFB_CUDA_TRY(cudaGetLastError(), "GEMV tile launch");
    return MFB_OK;
}

constexpr int kGtWarps = 8;
constexpr int kGtBoxes = 4;  // 32-k boxes of A per stage: 512 contiguous bytes of each row

// Stage count: measured on the 16384 x 16384 GEMV, a ring of two (n > 8) or three
// 128-k stages beats deeper rings of smaller stages; never more than fit beside the
// reduction buffer.
template <int NC, int CH, int R>
constexpr int gemv_tile_stages() {
    using L = GemvTileLayout<NC, CH, R, kGtWarps, 1, kGtBoxes>;
    constexpr int fit = (232448 - 1024 - 1024 - L::kRedBytes) / (L::kAStage + L::kXStage);
    constexpr int want = NC > 8 ? 2 : 3;
    return fit < want ? fit : want;
}

template <int NC, int CH, int R>
mfb_status_t launch_tile_r(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                           const float* bias, int rows, int sms) {
    static_assert(gemv_tile_stages<NC, CH, R>() >= 2, "the GEMV tile ring needs two stages");
    return launch_tile<NC, CH, R, kGtWarps, gemv_tile_stages<NC, CH, R>(), kGtBoxes>(d, stream, a, b, c, bias, rows,
                                                                                     sms);
}

// n > 4: the lanes split the columns in two groups of 16 lanes; a lane holds R rows of
// 16-row strides, R chosen so that R * 16 covers the tile's rows. n <= 4: one group,
// R rows of 32-row strides.
template <int NC>
mfb_status_t launch_tile_nc(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                            const float* bias, int sms) {
    const int rows = gemv_tile_rows(d.m, sms);
    if constexpr (NC > 4) {
        if (rows > 112) return launch_tile_r<NC, 2, 8>(d, stream, a, b, c, bias, rows, sms);
        if (rows > 64) return launch_tile_r<NC, 2, 7>(d, stream, a, b, c, bias, rows, sms);
        if (rows > 32) return launch_tile_r<NC, 2, 4>(d, stream, a, b, c, bias, rows, sms);
        return launch_tile_r<NC, 2, 2>(d, stream, a, b, c, bias, rows, sms);
    } else {
        if (rows > 64) return launch_tile_r<NC, 1, 4>(d, stream, a, b, c, bias, rows, sms);
        if (rows > 32) return launch_tile_r<NC, 1, 2>(d, stream, a, b, c, bias, rows, sms);
        return launch_tile_r<NC, 1, 1>(d, stream, a, b, c, bias, rows, sms);
    }
}

// The TMA tile kernel needs 16-byte aligned A and B with row strides in whole 16 bytes;
// for n == 1 a contiguous x (ldb == 1) also qualifies.
bool gemv_tile_eligible(const mfb_gemm_desc& d, const float* a, const float* b) {
    if (d.n < 1 || d.n > 16 || !aligned16(a) || !aligned16(b) || d.lda % 4 != 0) return false;
    return d.ldb % 4 == 0 || (d.n == 1 && d.ldb == 1);
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
    if (gemv_tile_eligible(d, a, b)) {
        int dev = 0;
        MFB_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
        const int sms = sm_count(dev);
        if (d.n == 1 && d.ldb == 1) return launch_tile_nc<1>(d, stream, a, b, c, bias, sms);
        if (d.n <= 4) return launch_tile_nc<4>(d, stream, a, b, c, bias, sms);
        if (d.n <= 8) return launch_tile_nc<8>(d, stream, a, b, c, bias, sms);
        return launch_tile_nc<16>(d, stream, a, b, c, bias, sms);
    }
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
