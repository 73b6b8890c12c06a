// Persistent tcgen05 mainloop shared by the GEMM and the implicit-GEMM conv2d.
//
// One CTA per SM walks 128 x BN output tiles round-robin:
//   warp 0      TMA producer: one elected lane fills a STAGES-deep ring of
//               shared-memory stages (Prob::load), running ahead across tiles.
//   warp 1      allocates 2 x BN TMEM columns; one elected lane issues
//               tcgen05.mma kind::tf32 (Prob::a_desc / b_desc) and releases each stage
//               with tcgen05.commit.
//   warps 2..   epilogue: tcgen05.ld of the FP32 accumulator and Prob::store.
//
// PLANES = 1 (TF32): one TF32 pass per K step into a 128 x BN FP32 accumulator; two
// accumulators alternate between tiles so the epilogue of tile i overlaps the MMAs of
// tile i+1 (4 epilogue warps, one per TMEM sub-partition).
//
// PLANES = 2 (strict FP32): each operand arrives as a (hi, lo) pair of TF32 planes
// (x = hi + lo + O(2^-22 |x|)); every K step issues lo*hi, hi*lo, then hi*hi. The
// tensor core folds each MMA into its FP32 accumulator with a truncating
// (round-toward-zero) add, so one accumulator over all of K drifts by ~K/8 ulps
// (1.4e-5 normwise at K=2048, measured). The accumulator is therefore restarted every
// kChunkKb K blocks (64 of K) and the epilogue warps fold each finished chunk into FP32
// registers with round-to-nearest adds; two chunk buffers alternate so the MMAs never
// wait for the fold. 8 epilogue warps: two per TMEM sub-partition, each owning BN/2
// columns of its 32 rows in registers.
//
// Every mbarrier wait is bounded by p.wait_limit_ns of %globaltimer; a wait that runs
// out records a bit in mfb::g_status, asks the other roles to stop, drains in-flight
// TMA copies and MMAs (again bounded) and frees TMEM before the CTA exits.
#pragma once

#include "mfb_device.cuh"

#include <cuda.h>
#include <type_traits>

namespace mfb {

constexpr int kTcBM = 128;
constexpr int kChunkKb = 2;  // strict mode: the accumulator restarts every 2 K blocks

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

// Strict mode with stacked B (Prob::kStackB, K-major B tiles of at most 64 rows): the hi
// and lo planes of a B tile lie back to back in shared memory, so they form one N = 2*BN
// operand. Each K step then issues two MMAs, A_hi x [B_hi | B_lo] and A_lo x [B_hi | B_lo],
// instead of three N = BN ones (lo*lo is a harmless extra term): a tcgen05 TF32 MMA with
// M = 128 costs about the same for N = 32, 64 or 128 (measured ~38 ns), so narrow tiles
// are issue-bound and stacking cuts their MMA time by a third. The accumulator is 2*BN
// columns wide and the epilogue adds its two halves.
template <class Prob>
constexpr int tc_acc_cols() {
    return Prob::kStackB ? 2 * Prob::BN : Prob::BN;
}

// K blocks per strict accumulator chunk: kChunkKb, or Prob::kChunkKbOverride for policies
// whose K blocks are deeper than 32 (the chunk stays 64 deep).
template <class P, class = void>
struct TcChunk : std::integral_constant<int, kChunkKb> {};
template <class P>
struct TcChunk<P, std::void_t<decltype(P::kChunkKbOverride)>> : std::integral_constant<int, P::kChunkKbOverride> {};

// ------------------------------------------------------------------------------------
// Work schedule: data-parallel tiles, then a stream-K share of the K blocks.
//
// Policies that declare kStreamK (the GEMM) may set p.sk_tiles > 0: the last sk_tiles
// tiles (in the policy's raster order) are not dealt out whole; their K blocks, flattened
// tile-major into I = sk_tiles * KB iterations, are cut into one contiguous range per
// worker (worker w: [floor(w I / G), floor((w+1) I / G)), G workers). A tile whose K blocks
// all fall in one worker's range is written as usual. A tile shared by several workers is
// not: each worker stores the FP32 sum of its part in a partial slot (slot 2w for the
// first tile of w's range, 2w + 1 for its last), and a separate reduce kernel adds a
// tile's slots in K order and applies the epilogue, so results do not depend on timing
// and no CTA ever waits for another. The first tiles (all but the last one or two waves)
// stay data parallel: worker w takes tiles w, w + G, ...
// Every role of a CTA walks the same sequence of work units.
// ------------------------------------------------------------------------------------
struct TcWork {
    int tile;      // tile index in the policy's raster
    int kb0, kb1;  // K blocks [kb0, kb1) of that tile
    int slot;      // -1: the unit covers the whole tile (normal store); else its partial slot
};

template <class P, class = void>
struct TcStreamK : std::false_type {};
template <class P>
struct TcStreamK<P, std::void_t<decltype(P::kStreamK)>> : std::integral_constant<bool, P::kStreamK> {};

template <class Prob>
__device__ __forceinline__ int tc_sk_tiles(const typename Prob::Params& p) {
    if constexpr (TcStreamK<Prob>::value) return p.sk_tiles;
    return 0;
}

// Worker owning flattened stream-K iteration i (the largest w with floor(w I / G) <= i).
__host__ __device__ __forceinline__ int tc_sk_owner(long long i, long long iters, int workers) {
    return static_cast<int>(((i + 1) * workers - 1) / iters);
}

template <class Prob>
struct TcWorkIter {
    int w, G, kb, dp_tiles, next_dp;
    long long iters, i, e, first_rel;

    __device__ TcWorkIter(const typename Prob::Params& p, int worker, int workers) {
        w = worker;
        G = workers;
        kb = Prob::num_kb(p);
        const int sk = tc_sk_tiles<Prob>(p);
        dp_tiles = Prob::num_tiles(p) - sk;
        next_dp = worker;
        iters = static_cast<long long>(sk) * kb;
        i = iters * worker / workers;
        e = iters * (worker + 1) / workers;
        first_rel = kb > 0 ? i / kb : 0;
    }

    __device__ bool next(TcWork& u) {
        if (next_dp < dp_tiles) {
            u = TcWork{next_dp, 0, kb, -1};
            next_dp += G;
            return true;
        }
        if (i >= e) return false;
        const long long rel = i / kb;
        const long long base = rel * kb;
        const int kb0 = static_cast<int>(i - base);
        const int kb1 = static_cast<int>(e - base < kb ? e - base : kb);
        const bool whole = kb0 == 0 && kb1 == kb;
        u = TcWork{dp_tiles + static_cast<int>(rel), kb0, kb1, whole ? -1 : (rel == first_rel ? 2 * w : 2 * w + 1)};
        i = base + kb;
        return true;
    }
};

template <class Prob>
struct TcLayout {
    static constexpr int kStageBytes = Prob::kATileBytes + Prob::kBTileBytes;
    static constexpr int kBarrierOffset = Prob::STAGES * kStageBytes;
    static constexpr int kBytes = kBarrierOffset + 256 + 1024;  // barriers + 1 KiB alignment slack
    static constexpr int kTmemCols = 2 * tc_acc_cols<Prob>() < 32 ? 32 : 2 * tc_acc_cols<Prob>();
    // tcgen05.alloc takes a power of two of at most 512 columns
    static_assert(kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation");
    static constexpr int kEpiWarps = Prob::PLANES == 2 ? 8 : 4;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
};

// Loads `count` (8 or 16) accumulator columns of this warp's 32 lanes.
template <int COUNT>
__device__ __forceinline__ void tmem_load_cols(uint32_t taddr, float* out) {
    if constexpr (COUNT == 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(taddr, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) out[j] = __uint_as_float(r[j]);
    } else {
        uint32_t r[8];
        tmem_ld_32x32b_x8(taddr, r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 8; ++j) out[j] = __uint_as_float(r[j]);
    }
}

// Writes COUNT consecutive accumulator columns of one row of a work unit: through the
// policy's epilogue for a whole tile (slot < 0), raw into the unit's partial slot for a
// stream-K share (rank: the CTA's rank within an SM pair; 0 for single-CTA tiles).
template <class Prob, int COUNT>
__device__ __forceinline__ void tc_store(const typename Prob::Params& p, const typename Prob::Tile& tile, int slot,
                                         int rank, int row_in_tile, int col0_in_tile, const float* v) {
    if constexpr (TcStreamK<Prob>::value) {
        if (slot >= 0) {
            Prob::template store_partial<COUNT>(p, slot, rank, row_in_tile, col0_in_tile, v);
            return;
        }
    }
    Prob::template store<COUNT>(p, tile, row_in_tile, col0_in_tile, v);
}

// Epilogue role (warps 2..) shared by the persistent tcgen05 kernels: waits for each
// finished accumulator (a tile in TF32 mode, a 64-deep K chunk in strict mode, summed in
// registers with round-to-nearest adds), hands the TMEM buffer back to the MMA issuer and
// writes the tile through Prob::store.
template <class Prob>
__device__ __forceinline__ void tc_epilogue_role(const typename Prob::Params& p, uint32_t tmem_base,
                                                 uint64_t* acc_full_bar, uint64_t* acc_empty_bar,
                                                 volatile int* abort_flag, uint64_t limit, int warp, int lane) {
    constexpr int BN = Prob::BN;
    constexpr int PLANES = Prob::PLANES;
    constexpr int ACC = tc_acc_cols<Prob>();  // accumulator columns per buffer
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 belong to this warp
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int row = quarter * 32 + lane;  // row within the tile
    int buf = 0;
    bool ok = true;
    TcWorkIter<Prob> work(p, blockIdx.x, gridDim.x);
    TcWork u;
    while (ok && work.next(u)) {
        const typename Prob::Tile tile = Prob::tile(p, u.tile);
        const int valid = Prob::valid_cols(p, tile);
        if constexpr (PLANES == 2) {
            // Round-to-nearest FP32 sum of the K chunks, in registers: this warp owns
            // columns [half * BN/2, (half + 1) * BN/2) of the tile.
            constexpr int kCols = BN / 2;
            constexpr int kStep = kCols % 16 == 0 ? 16 : 8;
            const int half = (warp - 2) >> 2;
            float sum[kCols];
#pragma unroll
            for (int j = 0; j < kCols; ++j) sum[j] = 0.0f;
            const int n_chunks = (u.kb1 - u.kb0 + TcChunk<Prob>::value - 1) / TcChunk<Prob>::value;
            for (int c = 0; c < n_chunks; ++c, ++buf) {
                const int b = buf & 1;
                if (!mbar_wait_bounded(&acc_full_bar[b], (buf >> 1) & 1, limit, abort_flag)) {
                    report_status(kStatusTimeoutEpilogue, abort_flag);
                    ok = false;
                    break;
                }
                tc_fence_after();
                if constexpr (Prob::kStackB && kStep == 16 && kCols <= 32) {
                    // Narrow stacked tiles: all loads of the chunk (both halves) in flight at
                    // once, one wait. The chunk's MMAs are short here, so the epilogue has to
                    // drain a chunk faster than one TMEM load round trip per 16 columns allows.
                    uint32_t rh[kCols / 16][16], rl[kCols / 16][16];
#pragma unroll
                    for (int q = 0; q < kCols / 16; ++q) {
                        tmem_ld_32x32b_x16(tmem_base + lane_base + b * ACC + half * kCols + q * 16, rh[q]);
                        tmem_ld_32x32b_x16(tmem_base + lane_base + b * ACC + BN + half * kCols + q * 16, rl[q]);
                    }
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < kCols / 16; ++q) {
                        tmem_regs_ready(rh[q]);
                        tmem_regs_ready(rl[q]);
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            sum[q * 16 + j] += __uint_as_float(rh[q][j]) + __uint_as_float(rl[q][j]);
                    }
                } else
#pragma unroll
                for (int q = 0; q < kCols / kStep; ++q) {
                    float v[kStep];
                    tmem_load_cols<kStep>(tmem_base + lane_base + b * ACC + half * kCols + q * kStep, v);
                    if constexpr (Prob::kStackB) {
                        // second half: the products with B_lo
                        float w[kStep];
                        tmem_load_cols<kStep>(tmem_base + lane_base + b * ACC + BN + half * kCols + q * kStep, w);
#pragma unroll
                        for (int j = 0; j < kStep; ++j) v[j] += w[j];
                    }
#pragma unroll
                    for (int j = 0; j < kStep; ++j) sum[q * kStep + j] += v[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty_bar[b]);
            }
            if (!ok) break;
#pragma unroll
            for (int q = 0; q < kCols / kStep; ++q) {
                const int col0 = half * kCols + q * kStep;
                if (col0 < valid) tc_store<Prob, kStep>(p, tile, u.slot, 0, row, col0, &sum[q * kStep]);
            }
        } else {
            const int b = buf & 1;
            if (!mbar_wait_bounded(&acc_full_bar[b], (buf >> 1) & 1, limit, abort_flag)) {
                report_status(kStatusTimeoutEpilogue, abort_flag);
                break;
            }
            tc_fence_after();
            const int nq = (min(valid, BN) + 15) / 16;
            for (int q = 0; q < nq; ++q) {
                float v[16];
                tmem_load_cols<16>(tmem_base + lane_base + b * BN + q * 16, v);
                if (q == nq - 1) {
                    // Accumulator fully read: hand it back to the MMA issuer.
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acc_empty_bar[b]);
                }
                tc_store<Prob, 16>(p, tile, u.slot, 0, row, q * 16, v);
            }
            ++buf;
        }
    }
}

template <class Prob>
__global__ void __launch_bounds__(TcLayout<Prob>::kThreads, 1)
    tc_persistent_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                         const typename Prob::Params p) {
    using L = TcLayout<Prob>;
    constexpr int BN = Prob::BN;
    constexpr int STAGES = Prob::STAGES;
    constexpr int PLANES = Prob::PLANES;
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN");
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
    grid_dependency_wait();  // operands written by the preceding prepass (programmatic launch)

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer
        int it = 0;
        bool ok = true;
        TcWorkIter<Prob> work(p, blockIdx.x, gridDim.x);
        TcWork u;
        while (ok && work.next(u)) {
            const typename Prob::Tile tile = Prob::tile(p, u.tile);
            for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&empty_bar[s], ((it / STAGES) & 1) ^ 1, limit, abort_flag)) {
                    report_status(kStatusTimeoutProducer, abort_flag);
                    ok = false;
                    break;
                }
                uint8_t* a_tile = smem + s * L::kStageBytes;
                mbar_arrive_expect_tx(&full_bar[s], L::kStageBytes);
                Prob::load(p, &tmap_a, &tmap_b, a_tile, a_tile + Prob::kATileBytes, &full_bar[s], tile, kb);
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
        constexpr uint32_t idesc = umma_idesc_tf32(kTcBM, BN, Prob::A_MN, Prob::B_MN);
        constexpr uint32_t idesc_stacked = umma_idesc_tf32(kTcBM, 2 * BN, Prob::A_MN, Prob::B_MN);
        // Accumulator buffers are handed out per tile (tf32) or per K chunk (strict).
        const int kb_per_buf = PLANES == 2 ? TcChunk<Prob>::value : 0x7fffffff;
        int it = 0;   // K blocks consumed (stage ring position)
        int buf = 0;  // accumulator buffers used so far
        bool ok = true;
        TcWorkIter<Prob> work(p, blockIdx.x, gridDim.x);
        TcWork u;
        while (ok && work.next(u)) {
            uint32_t d_tmem = 0;
            uint32_t acc = 0;
            for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
                const int kr = kb - u.kb0;  // K blocks into this unit
                if (kr % kb_per_buf == 0) {
                    const int b = buf & 1;
                    if (!mbar_wait_bounded(&acc_empty_bar[b], ((buf >> 1) & 1) ^ 1, limit, abort_flag)) {
                        report_status(kStatusTimeoutMma, abort_flag);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    d_tmem = tmem_base + b * tc_acc_cols<Prob>();
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
                const uint32_t b_addr = a_addr + Prob::kATileBytes;
#pragma unroll
                for (int ks = 0; ks < Prob::kKSteps; ++ks) {
                    const uint64_t a_hi = Prob::a_desc(a_addr, 0, ks);
                    const uint64_t b_hi = Prob::b_desc(b_addr, 0, ks);
                    if constexpr (Prob::kStackB) {
                        // b_hi spans both planes: 2*BN rows [B_hi; B_lo]
                        umma_tf32(d_tmem, a_hi, b_hi, idesc_stacked, acc);
                        umma_tf32(d_tmem, Prob::a_desc(a_addr, 1, ks), b_hi, idesc_stacked, 1);
                        acc = 1;
                        continue;
                    }
                    if (PLANES == 2) {
                        umma_tf32(d_tmem, Prob::a_desc(a_addr, 1, ks), b_hi, idesc, acc);
                        acc = 1;
                        umma_tf32(d_tmem, a_hi, Prob::b_desc(b_addr, 1, ks), idesc, 1);
                    }
                    umma_tf32(d_tmem, a_hi, b_hi, idesc, acc);
                    acc = 1;
                }
                umma_commit(&empty_bar[s]);
                if (kr % kb_per_buf == kb_per_buf - 1 || kb == u.kb1 - 1) {
                    umma_commit(&acc_full_bar[buf & 1]);
                    ++buf;
                }
            }
        }
        // Drain: every MMA this thread issued must retire before TMEM is freed.
        umma_commit(drain_bar);
        if (!mbar_wait_drain(drain_bar, 0, limit)) report_status(kStatusTimeoutDrain, nullptr);
    } else if (warp >= 2) {
        tc_epilogue_role<Prob>(p, tmem_base, acc_full_bar, acc_empty_bar, abort_flag, limit, warp, lane);
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

}  // namespace mfb
