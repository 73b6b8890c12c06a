// tcgen05 FP32 GEMM for sm_100a: C = epilogue(alpha * op(A) * op(B) + beta * C), row-major.
//
// Persistent kernel, one CTA per SM, 128 x BN output tiles handed out round-robin:
//   warp 0      TMA producer: one elected lane streams 32-deep K slabs of A and B
//               into a STAGES-deep ring of swizzled shared-memory tiles, running
//               ahead across tile boundaries.
//   warp 1      allocates 2 x BN TMEM columns; one elected lane issues
//               tcgen05.mma kind::tf32 and releases each stage with tcgen05.commit.
//   warps 2..   epilogue: tcgen05.ld of the FP32 accumulator, fused
//               alpha/beta/bias/activation, strided stores to C.
//
// PLANES = 1 (GemmPrecision::tf32): one TF32 pass per K step into a 128 x BN FP32
// accumulator; two accumulators alternate between tiles so the epilogue of tile i
// overlaps the MMAs of tile i+1 (4 epilogue warps, one per TMEM sub-partition).
//
// PLANES = 2 (strict FP32): each operand arrives as a (hi, lo) pair of TF32 planes
// written by split_tf32_kernel (x = hi + lo + O(2^-22 |x|)); every K step issues
// lo*hi, hi*lo, then hi*hi. The tensor core folds each MMA into its FP32 accumulator
// with a truncating (round-toward-zero) add, so one accumulator over all of K drifts
// by ~K/8 ulps (1.4e-5 normwise at K=2048, measured). The accumulator is therefore
// restarted every kChunkKb K blocks (64 of K) and the epilogue warps fold each
// finished chunk into FP32 registers with round-to-nearest adds; two chunk buffers
// alternate so the MMAs never wait for the fold. 8 epilogue warps: two per TMEM
// sub-partition, each owning BN/2 columns of its 32 rows in registers.
//
// Operand majors: A is K-major (row-major A) or MN-major (A stored transposed);
// B is MN-major (row-major B) or K-major (B stored transposed). K-major tiles are one
// TMA box of 32 K x rows with 128B swizzle (16-byte atoms). MN-major tiles are
// 32-element-wide column groups with the 128B/32-byte-atom swizzle that tcgen05
// requires for MN-major TF32 operands.
//
// Every mbarrier wait is bounded by params.wait_limit_ns of %globaltimer; a wait
// that runs out records a bit in mfb::g_status, asks the other roles to stop,
// drains in-flight TMA copies and MMAs (again bounded) and frees TMEM before the
// CTA exits.
#pragma once

#include "mfb_device.cuh"

#include <cuda.h>

namespace mfb {

struct GemmTcParams {
    int m, n, k;
    int num_kb;          // ceil(k / 32)
    int tiles_m, tiles_n;
    int group_m;         // tile raster: group_m tile-rows walk N together
    float* c;
    long long ldc;
    float alpha, beta;
    const float* bias;   // length n, or nullptr
    int epilogue;        // 0 none, 1 bias, 2 bias+relu, 3 bias+gelu
    int c_vec4;          // C base 16B aligned and ldc % 4 == 0
    unsigned long long wait_limit_ns;
};

constexpr int kBM = 128;
constexpr int kBK = 32;        // 32 fp32 = 128 bytes: one swizzle row
constexpr int kChunkKb = 2;    // strict mode: accumulator restarts every 2 K blocks (64 of K)

template <int BN, int STAGES, int PLANES>
struct GemmTcSmem {
    static constexpr int kATileBytes = PLANES * kBM * kBK * 4;
    static constexpr int kBTileBytes = PLANES * BN * kBK * 4;
    static constexpr int kStageBytes = kATileBytes + kBTileBytes;
    static constexpr int kBarrierOffset = STAGES * kStageBytes;
    static constexpr int kBytes = kBarrierOffset + 256 + 1024;  // barriers + 1 KiB alignment slack
    static constexpr int kTmemCols = 2 * BN;                    // two accumulator buffers
    static constexpr int kEpiWarps = PLANES == 2 ? 8 : 4;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
};

__device__ __forceinline__ float apply_epilogue_op(float v, const float* bias, int col, int epilogue) {
    if (epilogue != 0) {
        v += bias[col];
        if (epilogue == 2) {
            v = v > 0.0f ? v : 0.0f;
        } else if (epilogue == 3) {
            const float x3 = v * v * v;
            v = 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * x3)));
        }
    }
    return v;
}

__device__ __forceinline__ void tile_coords(int t, const GemmTcParams& p, int bn, int* m0, int* n0) {
    const int per_group = p.group_m * p.tiles_n;
    const int group = t / per_group;
    const int first_m = group * p.group_m;
    const int gsize = min(p.group_m, p.tiles_m - first_m);
    const int in_group = t - group * per_group;
    *m0 = (first_m + in_group % gsize) * kBM;
    *n0 = (in_group / gsize) * bn;
}

// Shared-memory descriptor of plane `pl`, K step `ks` of an operand tile at `addr`.
template <int MN_MAJOR, int ROWS, int PLANES>
__device__ __forceinline__ uint64_t operand_desc(uint32_t addr, int pl, int ks) {
    if (MN_MAJOR) {
        // [group of 32 MN][plane][32 K rows][32 MN]: MN groups PLANES*4 KiB apart (LBO),
        // 4-row K groups 512 B apart (SBO); a K step of 8 rows is 1 KiB.
        return umma_smem_desc(addr + pl * 4096 + ks * 1024, PLANES * 4096, 512, kLayoutSwizzle128B_Base32B);
    }
    // [plane][ROWS][32 K]: 8-row groups 1 KiB apart (SBO); a K step of 8 is 32 B.
    return umma_smem_desc(addr + pl * ROWS * 128 + ks * 32, 16, 1024, kLayoutSwizzle128B);
}

// Writes 32 consecutive outputs of one row: o = epilogue(alpha * acc + beta * C).
__device__ __forceinline__ void store_row_chunk(float* crow, int col0, const float* v, const GemmTcParams& p) {
    if (p.c_vec4 && col0 + 32 <= p.n) {
        // Two halves of 16: the C loads of a half are issued together, then combined and stored.
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float4 cin[4];
            if (p.beta != 0.0f) {
#pragma unroll
                for (int j = 0; j < 4; ++j) cin[j] = *reinterpret_cast<const float4*>(crow + col0 + 16 * h + 4 * j);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int c = 16 * h + 4 * j;
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = p.alpha * v[c + e];
                if (p.beta != 0.0f) {
                    o[0] = fmaf(p.beta, cin[j].x, o[0]);
                    o[1] = fmaf(p.beta, cin[j].y, o[1]);
                    o[2] = fmaf(p.beta, cin[j].z, o[2]);
                    o[3] = fmaf(p.beta, cin[j].w, o[3]);
                }
                if (p.epilogue) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[e] = apply_epilogue_op(o[e], p.bias, col0 + c + e, p.epilogue);
                }
                *reinterpret_cast<float4*>(crow + col0 + c) = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int col = col0 + j;
            if (col < p.n) {
                float o = p.alpha * v[j];
                if (p.beta != 0.0f) o = fmaf(p.beta, crow[col], o);
                crow[col] = apply_epilogue_op(o, p.bias, col, p.epilogue);
            }
        }
    }
}

template <int BN, int STAGES, int PLANES, int A_MN, int B_MN>
__global__ void __launch_bounds__(GemmTcSmem<BN, STAGES, PLANES>::kThreads, 1)
    gemm_tf32_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const GemmTcParams p) {
    using L = GemmTcSmem<BN, STAGES, PLANES>;
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
    uint64_t* empty_bar = full_bar + STAGES;
    uint64_t* acc_full_bar = empty_bar + STAGES;  // [2] tile (tf32) or K-chunk (strict) buffers
    uint64_t* acc_empty_bar = acc_full_bar + 2;   // [2]
    uint64_t* drain_bar = acc_empty_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int num_tiles = p.tiles_m * p.tiles_n;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full_bar[b], 1);
            mbar_init(&acc_empty_bar[b], L::kEpiWarps);  // one arrival per epilogue warp
        }
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmap_a);
        tma_prefetch_desc(&tmap_b);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, L::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint64_t limit = p.wait_limit_ns;

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            int m0, n0;
            tile_coords(t, p, BN, &m0, &n0);
            for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&empty_bar[s], ((it / STAGES) & 1) ^ 1, limit, abort_flag)) {
                    report_status(kStatusTimeoutProducer, abort_flag);
                    ok = false;
                    break;
                }
                uint8_t* a_tile = smem + s * L::kStageBytes;
                uint8_t* b_tile = a_tile + L::kATileBytes;
                mbar_arrive_expect_tx(&full_bar[s], L::kStageBytes);
                const int k0 = kb * kBK;
                if (A_MN) {
#pragma unroll
                    for (int g = 0; g < kBM / 32; ++g)
                        tma_load_3d(a_tile + g * PLANES * 4096, &tmap_a, &full_bar[s], m0 + 32 * g, k0, 0);
                } else {
                    tma_load_3d(a_tile, &tmap_a, &full_bar[s], k0, m0, 0);
                }
                if (B_MN) {
#pragma unroll
                    for (int g = 0; g < BN / 32; ++g)
                        tma_load_3d(b_tile + g * PLANES * 4096, &tmap_b, &full_bar[s], n0 + 32 * g, k0, 0);
                } else {
                    tma_load_3d(b_tile, &tmap_b, &full_bar[s], k0, n0, 0);
                }
            }
        }
        // Drain: every issued copy must land before this CTA's shared memory goes away.
        for (int j = it - STAGES < 0 ? 0 : it - STAGES; j < it; ++j) {
            if (!mbar_wait_drain(&full_bar[j % STAGES], (j / STAGES) & 1, limit)) {
                report_status(kStatusTimeoutDrain, nullptr);
                break;
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ------------------------------------------------------------ MMA issuer
        constexpr uint32_t idesc = umma_idesc_tf32(kBM, BN, A_MN, B_MN);
        // Accumulator buffers are handed out per tile (tf32) or per K chunk (strict).
        const int kb_per_buf = PLANES == 2 ? kChunkKb : 0x7fffffff;
        int it = 0;    // K blocks consumed (stage ring position)
        int buf = 0;   // accumulator buffers used so far
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            uint32_t d_tmem = 0;
            uint32_t acc = 0;
            for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
                if (kb % kb_per_buf == 0) {
                    const int b = buf & 1;
                    if (!mbar_wait_bounded(&acc_empty_bar[b], ((buf >> 1) & 1) ^ 1, limit, abort_flag)) {
                        report_status(kStatusTimeoutMma, abort_flag);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    d_tmem = tmem_base + b * BN;
                    acc = 0;
                }
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&full_bar[s], (it / STAGES) & 1, limit, abort_flag)) {
                    report_status(kStatusTimeoutMma, abort_flag);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes);
                const uint32_t b_addr = a_addr + L::kATileBytes;
#pragma unroll
                for (int ks = 0; ks < kBK / 8; ++ks) {
                    const uint64_t a_hi = operand_desc<A_MN, kBM, PLANES>(a_addr, 0, ks);
                    const uint64_t b_hi = operand_desc<B_MN, BN, PLANES>(b_addr, 0, ks);
                    if (PLANES == 2) {
                        const uint64_t a_lo = operand_desc<A_MN, kBM, PLANES>(a_addr, 1, ks);
                        const uint64_t b_lo = operand_desc<B_MN, BN, PLANES>(b_addr, 1, ks);
                        umma_tf32(d_tmem, a_lo, b_hi, idesc, acc);
                        acc = 1;
                        umma_tf32(d_tmem, a_hi, b_lo, idesc, 1);
                    }
                    umma_tf32(d_tmem, a_hi, b_hi, idesc, acc);
                    acc = 1;
                }
                umma_commit(&empty_bar[s]);
                if (kb % kb_per_buf == kb_per_buf - 1 || kb == p.num_kb - 1) {
                    umma_commit(&acc_full_bar[buf & 1]);
                    ++buf;
                }
            }
        }
        // Drain: every MMA this thread issued must retire before TMEM is freed.
        umma_commit(drain_bar);
        if (!mbar_wait_drain(drain_bar, 0, limit)) report_status(kStatusTimeoutDrain, nullptr);
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 belong to this warp
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        int buf = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
            int m0, n0;
            tile_coords(t, p, BN, &m0, &n0);
            const int row = m0 + quarter * 32 + lane;
            const bool row_ok = row < p.m;
            float* crow = p.c + static_cast<long long>(row) * p.ldc;
            if constexpr (PLANES == 2) {
                // Round-to-nearest FP32 sum of the K chunks, in registers: this warp owns
                // columns [half * BN/2, (half + 1) * BN/2) of the tile.
                constexpr int kCols = BN / 2;
                const int half = (warp - 2) >> 2;
                float sum[kCols];
#pragma unroll
                for (int j = 0; j < kCols; ++j) sum[j] = 0.0f;
                const int n_chunks = (p.num_kb + kChunkKb - 1) / kChunkKb;
                for (int c = 0; c < n_chunks; ++c, ++buf) {
                    const int b = buf & 1;
                    if (!mbar_wait_bounded(&acc_full_bar[b], (buf >> 1) & 1, limit, abort_flag)) {
                        report_status(kStatusTimeoutEpilogue, abort_flag);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int q = 0; q < kCols / 16; ++q) {
                        uint32_t r[16];
                        tmem_ld_32x32b_x16(tmem_base + lane_base + b * BN + half * kCols + q * 16, r);
                        tmem_ld_wait();
#pragma unroll
                        for (int j = 0; j < 16; ++j) sum[q * 16 + j] += __uint_as_float(r[j]);
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty_bar[b]);
                }
                if (!ok) break;
                if (row_ok) {
#pragma unroll
                    for (int q = 0; q < kCols / 32; ++q) {
                        const int col0 = n0 + half * kCols + q * 32;
                        if (col0 < p.n) store_row_chunk(crow, col0, &sum[q * 32], p);
                    }
                }
            } else {
                const int b = buf & 1;
                if (!mbar_wait_bounded(&acc_full_bar[b], (buf >> 1) & 1, limit, abort_flag)) {
                    report_status(kStatusTimeoutEpilogue, abort_flag);
                    break;
                }
                tc_fence_after();
                const int nchunks = min(BN / 32, (p.n - n0 + 31) / 32);
                for (int q = 0; q < nchunks; ++q) {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(tmem_base + lane_base + b * BN + q * 32, r);
                    tmem_ld_wait();
                    if (q == nchunks - 1) {
                        // Accumulator fully read: hand it back to the MMA issuer.
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&acc_empty_bar[b]);
                    }
                    if (row_ok) {
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
                        store_row_chunk(crow, n0 + q * 32, v, p);
                    }
                }
                ++buf;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

}  // namespace mfb
