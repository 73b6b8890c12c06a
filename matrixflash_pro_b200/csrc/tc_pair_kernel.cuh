// tcgen05 GEMM on SM pairs (cluster of 2 CTAs, tcgen05.mma.cta_group::2): 256 x BN tiles.
//
// Each CTA of a pair holds half of the tile's operands in its shared memory: A rows
// [m0 + 128*rank, +128) and B columns [n0 + (BN/2)*rank, +BN/2). The leader CTA
// (cluster rank 0) issues one M=256 x N=BN MMA per K step for the pair; each SM's tensor
// core reads its own A half and both B halves, so per SM the shared-memory operand traffic
// per FLOP is that of a 128 x BN tile with half the B bytes loaded, and each CTA's TMEM
// holds the 128 x BN accumulator rows of its half.
//
// Roles per CTA (same as tc_persistent_kernel, plus the pair protocol):
//   warp 0 (both)   TMA producer for this CTA's halves; waits on its own "empty" barriers;
//                   completions are counted on the leader's "full" barriers (cta_group::2
//                   loads); only the leader posts the expected byte count (both halves).
//   warp 1 (both)   allocates TMEM with cta_group::2; on the leader one lane issues the
//                   MMAs and tcgen05.commit multicasts to both CTAs' empty / accumulator
//                   barriers.
//   warps 2.. (both) epilogue of this CTA's 128 rows; releases accumulator buffers on the
//                   leader's barrier (a remote arrive from the peer).
// Accumulation (TF32 one pass per tile; strict FP32 chunked every 64 of K with
// round-to-nearest register sums) is the same as tc_persistent_kernel's.
//
// Every wait is bounded by p.wait_limit_ns; a role that gives up sets the abort flag of
// both CTAs and records a status bit. The CTAs meet at cluster barriers after set-up and
// before TMEM is freed, so neither frees shared memory the other may still signal.
#pragma once

#include "gemm_tc.cuh"

namespace mfb {

// KS = 32-deep K slabs per stage (a K block is 32 * KS deep; strict accumulator chunks stay
// 64 deep whatever KS is).
template <int BN_, int STAGES_, int PLANES_, int A_MN_, int B_MN_, int KS_ = 1>
struct GemmPairProblem {
    using Params = GemmTcParams;
    static constexpr int BN = BN_, STAGES = STAGES_, PLANES = PLANES_, A_MN = A_MN_, B_MN = B_MN_;
    static constexpr int KS = KS_;
    static constexpr int kChunkKbOverride = KS == 1 ? kChunkKb : 1;  // strict chunks stay 64 deep
    static constexpr int kBH = BN / 2;  // B columns per CTA
    static constexpr int kASlabBytes = PLANES * kTcBM * kBK * 4;
    static constexpr int kBSlabBytes = PLANES * kBH * kBK * 4;
    static constexpr int kATileBytes = KS * kASlabBytes;
    static constexpr int kBTileBytes = KS * kBSlabBytes;
    static constexpr int kKSteps = KS * kBK / 8;
    static constexpr int kPairBM = 2 * kTcBM;
    static constexpr bool kStreamK = true;  // p.sk_tiles / p.partials: stream-K share of the last tiles
    static_assert(kBH % 32 == 0 || !B_MN, "MN-major B halves are 32-column groups");

    struct Tile {
        int m0, n0;  // pair tile origin (256 x BN)
        int b;       // batch entry
    };

    __device__ static int num_tiles(const Params& p) { return p.batch * p.tiles_m * p.tiles_n; }
    __device__ static int num_kb(const Params& p) { return p.num_kb; }

    __device__ static Tile tile(const Params& p, int t) {
        const int per_batch = p.tiles_m * p.tiles_n;
        const int b = t / per_batch;
        t -= b * per_batch;
        const int per_group = p.group_m * p.tiles_n;
        const int group = t / per_group;
        const int first_m = group * p.group_m;
        const int gsize = min(p.group_m, p.tiles_m - first_m);
        const int in_group = t - group * per_group;
        return Tile{(first_m + in_group % gsize) * kPairBM, p.n_base + (in_group / gsize) * BN, b};
    }

    __device__ static void load(const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* a_tile, uint8_t* b_tile,
                                uint32_t full_bar_leader, const Tile& t, int kb, int rank) {
        const int ma = t.m0 + kTcBM * rank;
        const int nb = t.n0 + kBH * rank;
        // maps are 4-D: (cols, rows, batch entry, plane); slab j of the stage holds K [k0, k0 + 32)
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            const int k0 = (kb * KS + j) * kBK;
            uint8_t* as = a_tile + j * kASlabBytes;
            uint8_t* bs = b_tile + j * kBSlabBytes;
            if (A_MN) {
#pragma unroll
                for (int g = 0; g < kTcBM / 32; ++g)
                    tma_load_4d_pair(as + g * PLANES * 4096, ta, full_bar_leader, ma + 32 * g, k0, t.b, 0);
            } else {
                tma_load_4d_pair(as, ta, full_bar_leader, k0, ma, t.b, 0);
            }
            if (B_MN) {
#pragma unroll
                for (int g = 0; g < kBH / 32; ++g)
                    tma_load_4d_pair(bs + g * PLANES * 4096, tb, full_bar_leader, nb + 32 * g, k0, t.b, 0);
            } else {
                tma_load_4d_pair(bs, tb, full_bar_leader, k0, nb, t.b, 0);
            }
        }
    }

    __device__ static uint64_t a_desc(uint32_t addr, int pl, int ks) {
        return GemmProblem<BN, STAGES, PLANES, A_MN, B_MN>::template desc<A_MN, kTcBM>(
            addr + (ks / 4) * kASlabBytes, pl, ks % 4);
    }
    __device__ static uint64_t b_desc(uint32_t addr, int pl, int ks) {
        return GemmProblem<BN, STAGES, PLANES, A_MN, B_MN>::template desc<B_MN, kBH>(
            addr + (ks / 4) * kBSlabBytes, pl, ks % 4);
    }

    template <int COUNT>
    __device__ static void store_partial(const Params& p, int slot, int rank, int row_in_tile, int col0_in_tile,
                                         const float* v) {
        store_partial_rows<kPairBM, BN, COUNT>(p, slot, rank, row_in_tile, col0_in_tile, v);
    }

    // Whole tile (slot < 0): the epilogue; stream-K share: the raw sum into the partial slot.
    template <int COUNT>
    __device__ static void store_unit(const Params& p, const Tile& t, int slot, int rank, int row_in_tile,
                                      int col0_in_tile, const float* v) {
        if (slot >= 0)
            store_partial<COUNT>(p, slot, rank, row_in_tile, col0_in_tile, v);
        else
            store<COUNT>(p, t, rank, row_in_tile, col0_in_tile, v);
    }

    template <int COUNT>
    __device__ static void store(const Params& p, const Tile& t, int rank, int row_in_tile, int col0_in_tile,
                                 const float* v) {
        using One = GemmProblem<BN, STAGES, PLANES, A_MN, B_MN>;
        typename One::Tile ot{t.m0 + kTcBM * rank, t.n0, t.b};
        One::template store<COUNT>(p, ot, row_in_tile, col0_in_tile, v);
    }
};

template <class Prob>
struct TcPairLayout {
    static constexpr int kStageBytes = Prob::kATileBytes + Prob::kBTileBytes;
    static constexpr int kBarrierOffset = Prob::STAGES * kStageBytes;
    static constexpr int kBytes = kBarrierOffset + 256 + 1024;
    // tcgen05.alloc takes a power of two >= 32 columns: two BN-wide accumulator buffers, rounded up.
    static constexpr int kTmemCols = 2 * Prob::BN <= 32 ? 32 : 2 * Prob::BN <= 64 ? 64 : 2 * Prob::BN <= 128 ? 128
                                     : 2 * Prob::BN <= 256 ? 256 : 512;
    static_assert(2 * Prob::BN <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation");
    static constexpr int kEpiWarps = Prob::PLANES == 2 ? 8 : 4;
    static constexpr int kThreads = 64 + 32 * kEpiWarps;
};

template <class Prob>
__global__ void __launch_bounds__(TcPairLayout<Prob>::kThreads, 1)
    tc_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                   const GemmTcParams p) {
    using L = TcPairLayout<Prob>;
    constexpr int BN = Prob::BN;
    constexpr int STAGES = Prob::STAGES;
    constexpr int PLANES = Prob::PLANES;
    static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256 && 2 * BN <= 512, "BN");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);  // used in the leader
    uint64_t* empty_bar = full_bar + STAGES;                                       // both CTAs
    uint64_t* acc_full_bar = empty_bar + STAGES;                                   // [2] both CTAs
    uint64_t* acc_empty_bar = acc_full_bar + 2;                                    // [2] used in the leader
    uint64_t* drain_bar = acc_empty_bar + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int rank = static_cast<int>(cluster_ctarank());
    const bool leader = rank == 0;
    const int pair = blockIdx.x / 2;
    const int npairs = gridDim.x / 2;
    const uint32_t abort_peer = map_to_cta(smem_u32(const_cast<int*>(abort_flag)), rank ^ 1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full_bar[b], 1);
            mbar_init(&acc_empty_bar[b], 2 * L::kEpiWarps);  // epilogue warps of both CTAs
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
        tmem_alloc_pair(tmem_slot, L::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // barriers of both CTAs initialised, TMEM of both allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const uint64_t limit = p.wait_limit_ns;
    grid_dependency_wait();  // operands written by the preceding prepass (programmatic launch)

    auto give_up = [&](uint32_t bits) {
        report_status(bits, abort_flag);
        st_cluster_u32(abort_peer, 1);
    };

    if (warp == 0 && lane == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        int it = 0;
        bool ok = true;
        TcWorkIter<Prob> work(p, pair, npairs);
        TcWork u;
        while (ok && work.next(u)) {
            const typename Prob::Tile tile = Prob::tile(p, u.tile);
            for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&empty_bar[s], ((it / STAGES) & 1) ^ 1, limit, abort_flag)) {
                    give_up(kStatusTimeoutProducer);
                    ok = false;
                    break;
                }
                uint8_t* a_tile = smem + s * L::kStageBytes;
                if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * L::kStageBytes);
                Prob::load(&tmap_a, &tmap_b, a_tile, a_tile + Prob::kATileBytes,
                           map_to_cta(smem_u32(&full_bar[s]), 0), tile, kb, rank);
            }
        }
        // Drain: wait until the MMAs consumed (hence the copies landed in) the last stages.
        for (int j = it - STAGES < 0 ? 0 : it - STAGES; j < it; ++j) {
            if (!mbar_wait_drain(&empty_bar[j % STAGES], (j / STAGES) & 1, limit)) {
                report_status(kStatusTimeoutDrain, nullptr);
                break;
            }
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ------------------------------------------------------------ MMA issuer (leader)
        constexpr uint32_t idesc = umma_idesc_tf32(2 * kTcBM, BN, Prob::A_MN, Prob::B_MN);
        const int kb_per_buf = PLANES == 2 ? TcChunk<Prob>::value : 0x7fffffff;
        int it = 0;
        int buf = 0;
        bool ok = true;
        TcWorkIter<Prob> work(p, pair, npairs);
        TcWork u;
        while (ok && work.next(u)) {
            uint32_t d_tmem = 0;
            uint32_t acc = 0;
            for (int kb = u.kb0; kb < u.kb1; ++kb, ++it) {
                const int kr = kb - u.kb0;  // K blocks into this unit
                if (kr % kb_per_buf == 0) {
                    const int b = buf & 1;
                    if (!mbar_wait_bounded(&acc_empty_bar[b], ((buf >> 1) & 1) ^ 1, limit, abort_flag)) {
                        give_up(kStatusTimeoutMma);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    d_tmem = tmem_base + b * BN;
                    acc = 0;
                }
                const int s = it % STAGES;
                if (!mbar_wait_bounded(&full_bar[s], (it / STAGES) & 1, limit, abort_flag)) {
                    give_up(kStatusTimeoutMma);
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
                    if (PLANES == 2) {
                        umma_tf32_pair(d_tmem, Prob::a_desc(a_addr, 1, ks), b_hi, idesc, acc);
                        acc = 1;
                        umma_tf32_pair(d_tmem, a_hi, Prob::b_desc(b_addr, 1, ks), idesc, 1);
                    }
                    umma_tf32_pair(d_tmem, a_hi, b_hi, idesc, acc);
                    acc = 1;
                }
                umma_commit_pair(&empty_bar[s], 0x3);
                if (kr % kb_per_buf == kb_per_buf - 1 || kb == u.kb1 - 1) {
                    umma_commit_pair(&acc_full_bar[buf & 1], 0x3);
                    ++buf;
                }
            }
        }
        umma_commit_pair(drain_bar, 0x1);
        if (!mbar_wait_drain(drain_bar, 0, limit)) report_status(kStatusTimeoutDrain, nullptr);
    } else if (warp >= 2) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int quarter = warp & 3;
        const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
        const int row = quarter * 32 + lane;
        int buf = 0;
        bool ok = true;
        TcWorkIter<Prob> work(p, pair, npairs);
        TcWork u;
        while (ok && work.next(u)) {
            const typename Prob::Tile tile = Prob::tile(p, u.tile);
            const int valid = min(BN, p.n - tile.n0);
            if constexpr (PLANES == 2) {
                constexpr int kCols = BN / 2;
                const int half = (warp - 2) >> 2;
                float sum[kCols];
#pragma unroll
                for (int j = 0; j < kCols; ++j) sum[j] = 0.0f;
                const int n_chunks = (u.kb1 - u.kb0 + TcChunk<Prob>::value - 1) / TcChunk<Prob>::value;
                for (int c = 0; c < n_chunks; ++c, ++buf) {
                    const int b = buf & 1;
                    if (!mbar_wait_bounded(&acc_full_bar[b], (buf >> 1) & 1, limit, abort_flag)) {
                        give_up(kStatusTimeoutEpilogue);
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int q = 0; q < kCols / 16; ++q) {
                        float v[16];
                        tmem_load_cols<16>(tmem_base + lane_base + b * BN + half * kCols + q * 16, v);
#pragma unroll
                        for (int j = 0; j < 16; ++j) sum[q * 16 + j] += v[j];
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&acc_empty_bar[b]), 0));
                }
                if (!ok) break;
#pragma unroll
                for (int q = 0; q < kCols / 16; ++q) {
                    const int col0 = half * kCols + q * 16;
                    if (col0 < valid) Prob::template store_unit<16>(p, tile, u.slot, rank, row, col0, &sum[q * 16]);
                }
            } else {
                const int b = buf & 1;
                if (!mbar_wait_bounded(&acc_full_bar[b], (buf >> 1) & 1, limit, abort_flag)) {
                    give_up(kStatusTimeoutEpilogue);
                    break;
                }
                tc_fence_after();
                const int nq = (valid + 15) / 16;
                for (int q = 0; q < nq; ++q) {
                    float v[16];
                    tmem_load_cols<16>(tmem_base + lane_base + b * BN + q * 16, v);
                    if (q == nq - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cluster(map_to_cta(smem_u32(&acc_empty_bar[b]), 0));
                    }
                    Prob::template store_unit<16>(p, tile, u.slot, rank, row, q * 16, v);
                }
                ++buf;
            }
        }
    }

    tc_fence_before();
    __syncwarp();
    cluster_sync_all();  // both CTAs done with each other's shared memory and TMEM
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, L::kTmemCols);
    }
}

}  // namespace mfb
