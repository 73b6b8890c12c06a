// tcgen05 FP32 GEMM policy for tc_persistent_kernel:
// C = epilogue(alpha * op(A) * op(B) + beta * C), row-major, 128 x BN tiles.
//
// Operand majors: A is K-major (row-major A) or MN-major (A stored transposed);
// B is MN-major (row-major B) or K-major (B stored transposed). K-major tiles are one
// TMA box of 32 K x rows with 128B swizzle (16-byte atoms). MN-major tiles are
// 32-element-wide column groups with the 128B/32-byte-atom swizzle that tcgen05
// requires for MN-major TF32 operands. Each operand tensor map is 4-D: (cols, rows,
// batch, plane), so one TMA box brings both planes (hi/lo in strict mode) of a slab of
// one batch entry. Unbatched problems have batch = 1.
#pragma once

#include "tc_kernel.cuh"

namespace mfb {

struct GemmTcParams {
    int m, n, k;
    int num_kb;          // ceil(k / 32)
    int tiles_m, tiles_n;
    int n_base;          // first output column of the launch (column-range multiplies), else 0
    int batch;           // strided-batched GEMMs: tiles of batch entry b follow those of b - 1
    long long c_batch_stride;  // floats between consecutive C matrices
    int group_m;         // tile raster: group_m tile-rows walk N together
    float* c;
    long long ldc;
    float alpha, beta;
    const float* bias;   // length n, or nullptr
    int epilogue;        // 0 none, 1 bias, 2 bias+relu, 3 bias+gelu
    int c_vec4;          // C base 16B aligned and ldc % 4 == 0
    unsigned long long wait_limit_ns;
    int sk_tiles;        // the last sk_tiles tiles share their K blocks among the workers (stream-K)
    float* partials;     // 2 slots per worker of (tile rows x BN) floats for shared tiles
};

// FP32 sums of a stream-K share: slot `slot` holds one tile of ROWS x BN floats, row-major;
// CTA `rank` of an SM pair writes rows [128 rank, 128 rank + 128). Slots start 256-byte
// aligned and COUNT-column groups start at multiples of COUNT, so 8-column groups take
// whole-sector stores.
template <int ROWS, int BN, int COUNT>
__device__ __forceinline__ void store_partial_rows(const GemmTcParams& p, int slot, int rank, int row_in_tile,
                                                   int col0_in_tile, const float* v) {
    float* dst = p.partials + static_cast<long long>(slot) * (ROWS * BN) +
                 static_cast<long long>(rank * kTcBM + row_in_tile) * BN + col0_in_tile;
    if constexpr (COUNT % 8 == 0) {
#pragma unroll
        for (int j = 0; j < COUNT / 8; ++j) st_global_v8(dst + 8 * j, v + 8 * j);
    } else {
#pragma unroll
        for (int j = 0; j < COUNT / 4; ++j)
            reinterpret_cast<float4*>(dst)[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
}

constexpr int kBK = 32;  // 32 fp32 = 128 bytes of K per stage: one swizzle row

// KS = 32-deep K slabs per stage: a K block is 32 * KS deep. Two slabs halve the fixed cost
// the MMA issuer pays per K block (barrier wait, fences, commit), which matters when a block
// holds few MMAs (TF32, narrow tiles). Strict accumulator chunks stay 64 deep.
template <int BN_, int STAGES_, int PLANES_, int A_MN_, int B_MN_, int KS_ = 1>
struct GemmProblem {
    using Params = GemmTcParams;
    static constexpr int BN = BN_, STAGES = STAGES_, PLANES = PLANES_, A_MN = A_MN_, B_MN = B_MN_;
    static constexpr int KS = KS_;
    static constexpr bool kStackB = false;  // row-major B is MN-major: its planes interleave per 32 columns
    static constexpr bool kStreamK = true;  // p.sk_tiles / p.partials: stream-K share of the last tiles
    static constexpr int kASlabBytes = PLANES * kTcBM * kBK * 4;
    static constexpr int kBSlabBytes = PLANES * BN * kBK * 4;
    static constexpr int kATileBytes = KS * kASlabBytes;
    static constexpr int kBTileBytes = KS * kBSlabBytes;
    static constexpr int kKSteps = KS * kBK / 8;
    static constexpr int kChunkKbOverride = KS == 1 ? kChunkKb : 1;

    struct Tile {
        int m0, n0, b;
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
        return Tile{(first_m + in_group % gsize) * kTcBM, p.n_base + (in_group / gsize) * BN, b};
    }

    __device__ static int valid_cols(const Params& p, const Tile& t) { return min(BN, p.n - t.n0); }

    __device__ static void load(const Params&, const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* a_tile,
                                uint8_t* b_tile, uint64_t* bar, const Tile& t, int kb) {
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            const int k0 = (kb * KS + j) * kBK;
            uint8_t* as = a_tile + j * kASlabBytes;
            uint8_t* bs = b_tile + j * kBSlabBytes;
            if (A_MN) {
#pragma unroll
                for (int g = 0; g < kTcBM / 32; ++g)
                    tma_load_4d(as + g * PLANES * 4096, ta, bar, t.m0 + 32 * g, k0, t.b, 0);
            } else {
                tma_load_4d(as, ta, bar, k0, t.m0, t.b, 0);
            }
            if (B_MN) {
#pragma unroll
                for (int g = 0; g < BN / 32; ++g)
                    tma_load_4d(bs + g * PLANES * 4096, tb, bar, t.n0 + 32 * g, k0, t.b, 0);
            } else {
                tma_load_4d(bs, tb, bar, k0, t.n0, t.b, 0);
            }
        }
    }

    // Shared-memory descriptor of plane `pl`, K step `ks` of an operand tile at `addr`.
    template <int MN_MAJOR, int ROWS>
    __device__ static uint64_t desc(uint32_t addr, int pl, int ks) {
        if (MN_MAJOR) {
            // [group of 32 MN][plane][32 K rows][32 MN]: MN groups PLANES*4 KiB apart (LBO),
            // 4-row K groups 512 B apart (SBO); a K step of 8 rows is 1 KiB.
            return umma_smem_desc(addr + pl * 4096 + ks * 1024, PLANES * 4096, 512, kLayoutSwizzle128B_Base32B);
        }
        // [plane][ROWS][32 K]: 8-row groups 1 KiB apart (SBO); a K step of 8 is 32 B.
        return umma_smem_desc(addr + pl * ROWS * 128 + ks * 32, 16, 1024, kLayoutSwizzle128B);
    }
    __device__ static uint64_t a_desc(uint32_t addr, int pl, int ks) {
        return desc<A_MN, kTcBM>(addr + (ks / 4) * kASlabBytes, pl, ks % 4);
    }
    __device__ static uint64_t b_desc(uint32_t addr, int pl, int ks) {
        return desc<B_MN, BN>(addr + (ks / 4) * kBSlabBytes, pl, ks % 4);
    }

    template <int COUNT>
    __device__ static void store_partial(const Params& p, int slot, int rank, int row_in_tile, int col0_in_tile,
                                         const float* v) {
        store_partial_rows<kTcBM, BN, COUNT>(p, slot, rank, row_in_tile, col0_in_tile, v);
    }

    // Writes COUNT consecutive outputs of one row: o = epilogue(alpha * acc + beta * C). Each
    // thread writes its own row. Where the row segment is 32-byte aligned it goes out in
    // whole-sector (256-bit) stores: 2048^3 GEMM 86.0 -> 84.0 us against 128-bit stores.
    // (Staging 32 x 32 blocks through shared memory for 4-row x 128-byte stores was slower
    // inside the GEMM: 87 -> 102 us.)
    template <int COUNT>
    __device__ static void store(const Params& p, const Tile& t, int row_in_tile, int col0_in_tile, const float* v) {
        const int row = t.m0 + row_in_tile;
        if (row >= p.m) return;
        const int col0 = t.n0 + col0_in_tile;
        float* crow = p.c + t.b * p.c_batch_stride + static_cast<long long>(row) * p.ldc;
        if (p.c_vec4 && col0 + COUNT <= p.n) {
            float4 cin[COUNT / 4];
            if (p.beta != 0.0f) {
#pragma unroll
                for (int j = 0; j < COUNT / 4; ++j) cin[j] = *reinterpret_cast<const float4*>(crow + col0 + 4 * j);
            }
            float o[COUNT];
#pragma unroll
            for (int j = 0; j < COUNT / 4; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) o[4 * j + e] = p.alpha * v[4 * j + e];
                if (p.beta != 0.0f) {
                    o[4 * j + 0] = fmaf(p.beta, cin[j].x, o[4 * j + 0]);
                    o[4 * j + 1] = fmaf(p.beta, cin[j].y, o[4 * j + 1]);
                    o[4 * j + 2] = fmaf(p.beta, cin[j].z, o[4 * j + 2]);
                    o[4 * j + 3] = fmaf(p.beta, cin[j].w, o[4 * j + 3]);
                }
                if (p.epilogue) {
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        o[4 * j + e] = apply_epilogue_op(o[4 * j + e], p.bias, col0 + 4 * j + e, p.epilogue);
                }
            }
            if (COUNT % 8 == 0 && (reinterpret_cast<uintptr_t>(crow + col0) & 31) == 0) {
#pragma unroll
                for (int j = 0; j < COUNT / 8; ++j) st_global_v8(crow + col0 + 8 * j, o + 8 * j);
            } else {
#pragma unroll
                for (int j = 0; j < COUNT / 4; ++j)
                    *reinterpret_cast<float4*>(crow + col0 + 4 * j) =
                        make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < COUNT; ++j) {
                const int col = col0 + j;
                if (col < p.n) {
                    float o = p.alpha * v[j];
                    if (p.beta != 0.0f) o = fmaf(p.beta, crow[col], o);
                    crow[col] = apply_epilogue_op(o, p.bias, col, p.epilogue);
                }
            }
        }
    }
};

}  // namespace mfb
