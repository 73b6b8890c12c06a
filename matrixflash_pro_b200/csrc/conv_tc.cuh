// Implicit-GEMM conv2d forward policy for tc_persistent_kernel (stride 1).
//
// Reference operation: conv2d_kernel (src/nn/conv.cu:22-49), NCHW cross-correlation
// y[n][f][p][q] = bias[f] + sum_{c,r,s} x[n][c][p+r-pad][q+s-pad] * w[f][c][r][s].
//
// Layout (written by the conv prepass, as TF32 planes):
//   X [plane][n][Hp*Wp][Cp]    input zero-padded to Hp = H+2pad, Wp = W+2pad, channels
//                              innermost, Cp = C rounded up to 4 (zeros beyond C)
//   W [plane][R*S][K][Cp]      weights per tap, channels innermost
// GEMM view per image: M = output positions j = p*Wp + q in padded-width space (the
// Wp-Q columns q >= Q of each row are computed and dropped), N = filters, K = (tap, c).
// With stride 1, tap (r, s) of output position j reads padded input position
// j + r*Wp + s, so each K block (one tap, 32 channels) is one TMA box of
// 32 channels x 128 consecutive positions: 128-byte rows, K-major, 128B swizzle —
// the same shared-memory tile as the GEMM's row-major A operand. The position
// coordinate is free of alignment rules; the channel coordinate (innermost) is a
// multiple of 32. Channels beyond Cp and positions beyond the image read as zeros.
#pragma once

#include "fastdiv.h"
#include "tc_kernel.cuh"

namespace mfb {

struct ConvTcParams {
    int n_img, c, h, w, kf, r, s, pad;
    int hp, wp;         // padded input height / width
    int p_out, q_out;   // output height / width
    int ncb;            // 32-channel slabs per tap (K blocks span KS consecutive slabs)
    FastDiv div_ncb;    // division by ncb
    FastDiv div_s;      // division by s
    int num_kb;         // r * s * ncb
    int tiles_pos;      // ceil(p_out * wp / 128) position tiles per image
    int tiles_f;        // filter tiles
    float* y;
    const float* bias;
    unsigned long long wait_limit_ns;
};

template <int BN, int PLANES, int KS>
constexpr int conv_stages() {
    return (196608 / (KS * PLANES * (kTcBM + BN) * 128)) > 8 ? 8
                                                              : (196608 / (KS * PLANES * (kTcBM + BN) * 128));
}

// KS = 32-channel slabs per stage: a K block is (one tap, 32 * KS channels). Two slabs halve
// the K blocks per tile and with them the fixed per-block cost of the MMA issuer (barrier wait,
// fences, commit), which the narrow N <= 128 MMAs of a conv cannot hide.
template <int BN_, int PLANES_, int KS_ = 1>
struct ConvProblem {
    using Params = ConvTcParams;
    static constexpr int BN = BN_, PLANES = PLANES_, A_MN = 0, B_MN = 0;
    static constexpr int KS = KS_;
    static constexpr bool kStackB = PLANES_ == 2 && BN_ <= 64;  // K-major weight tiles: hi, lo rows adjacent
    static constexpr int STAGES = conv_stages<BN_, PLANES_, KS_>();
    static constexpr int kASlabBytes = PLANES * kTcBM * 128;
    static constexpr int kBSlabBytes = PLANES * BN * 128;
    static constexpr int kATileBytes = KS * kASlabBytes;
    static constexpr int kBTileBytes = KS * kBSlabBytes;
    static constexpr int kKSteps = 4 * KS;  // 32 channels = 4 K steps of 8 per slab
    static_assert(KS == 1 || KS == 2 || (KS == 4 && PLANES_ == 1), "slabs per K block");
    static constexpr int kChunkKbOverride = KS == 1 ? 2 : 1;  // strict chunks stay 64 channels deep
    static_assert(STAGES >= 2, "conv tile configuration");

    struct Tile {
        int img, j0, f0;
    };

    __device__ static int num_tiles(const Params& p) { return p.n_img * p.tiles_pos * p.tiles_f; }
    __device__ static int num_kb(const Params& p) { return p.num_kb; }

    __device__ static Tile tile(const Params& p, int t) {
        const int f_tile = t % p.tiles_f;
        const int rest = t / p.tiles_f;
        return Tile{rest / p.tiles_pos, (rest % p.tiles_pos) * kTcBM, f_tile * BN};
    }

    __device__ static int valid_cols(const Params& p, const Tile& t) { return min(BN, p.kf - t.f0); }

    // The tile's K runs over (tap, 32-channel slab) pairs, tap-major, p.ncb slabs per tap; K block
    // kb holds slabs kb*KS .. kb*KS+KS-1, so a block may span two taps and no slab is wasted when
    // the channel count fills an odd number of slabs. Channels past Cp and the slabs after the
    // last tap (the tail of the last block) read the maps' zero fill.
    __device__ static void load(const Params& p, const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* a_tile,
                                uint8_t* b_tile, uint64_t* bar, const Tile& t, int kb) {
        const int taps = p.r * p.s;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            const int g = kb * KS + j;
            int tap = static_cast<int>(fastdiv(static_cast<uint32_t>(g), p.div_ncb));
            int c0 = (g - tap * p.ncb) * 32;
            if (tap >= taps) {  // past the last tap: a box beyond the channels, all zero fill
                tap = taps - 1;
                c0 = p.ncb * 32;
            }
            const int r = static_cast<int>(fastdiv(static_cast<uint32_t>(tap), p.div_s));
            const int sc = tap - r * p.s;
            tma_load_4d(a_tile + j * kASlabBytes, ta, bar, c0, t.j0 + r * p.wp + sc, t.img, 0);
            tma_load_4d(b_tile + j * kBSlabBytes, tb, bar, c0, t.f0, tap, 0);
        }
    }

    // Per slab [plane][rows][32 channels], 128B swizzle: 8-row groups 1 KiB apart; a K step is 32 B.
    __device__ static uint64_t a_desc(uint32_t addr, int pl, int ks) {
        return umma_smem_desc(addr + (ks / 4) * kASlabBytes + pl * kTcBM * 128 + (ks % 4) * 32, 16, 1024,
                              kLayoutSwizzle128B);
    }
    __device__ static uint64_t b_desc(uint32_t addr, int pl, int ks) {
        return umma_smem_desc(addr + (ks / 4) * kBSlabBytes + pl * BN * 128 + (ks % 4) * 32, 16, 1024,
                              kLayoutSwizzle128B);
    }

    // Scatters COUNT filters of one output position to NCHW: y = acc + bias[f].
    template <int COUNT>
    __device__ static void store(const Params& p, const Tile& t, int row_in_tile, int col0_in_tile, const float* v) {
        const int j = t.j0 + row_in_tile;
        const int pr = j / p.wp;
        const int q = j - pr * p.wp;
        if (pr >= p.p_out || q >= p.q_out) return;
        const long long plane = static_cast<long long>(p.p_out) * p.q_out;
        float* base = p.y + static_cast<long long>(t.img) * p.kf * plane + static_cast<long long>(pr) * p.q_out + q;
#pragma unroll
        for (int e = 0; e < COUNT; ++e) {
            const int f = t.f0 + col0_in_tile + e;
            if (f < p.kf) base[f * plane] = p.bias ? v[e] + p.bias[f] : v[e];
        }
    }
};

// ------------------------------------------------------------------------------------
// Weight gradient, stride 1: dW[f][c][r][s] = sum_{n,p,q} dY[n][f][p][q] * Xpad[n][c][p+r][q+s].
//
// GEMM view: D[m][f] with m = tap * Cg + c (Cg = C rounded up to 32; rows of one 32-row
// group share a tap), reduced over K = (image, output position j = p*Wp + q in the
// padded-width space of X). A = X planes [n][Hp*Wp][Cp] read MN-major (channels
// contiguous): the 32-channel x 32-position box of row group g sits at position
// j0 + r*Wp + s of its tap. B = dY planes [n][K][P*Wp] (zeros for q >= Q) read K-major.
// K is cut into `splits` equal ranges, one per output-tile work unit; each unit writes
// its 128 x BN partial tile and conv_wgrad_reduce_kernel sums the splits in order.
// K blocks past the last image read the maps' zero fill.
// ------------------------------------------------------------------------------------
struct ConvWgradParams {
    int n_img, c, kf, r, s;
    int cg;              // C rounded up to 32
    int wp;              // padded width of X (output positions live in this width)
    int kb_per_img;      // ceil(P * Wp / (32 * KS))
    FastDiv div_kb_per_img;
    int kb_per_split;
    int splits;
    int tiles_m, tiles_f;
    int rows_total;      // r * s * cg
    int ld_partial;      // tiles_f * BN
    float* partial;      // [splits][rows_total rounded up to 128][ld_partial]
    unsigned long long wait_limit_ns;
};

// KS = 32-position slabs per stage (a K block is 32 * KS positions; see ConvProblem).
template <int BN_, int PLANES_, int KS_ = 1>
struct ConvWgradProblem {
    using Params = ConvWgradParams;
    static constexpr int BN = BN_, PLANES = PLANES_, A_MN = 1, B_MN = 0;
    static constexpr int KS = KS_;
    static constexpr bool kStackB = PLANES_ == 2 && BN_ <= 64;  // dY tiles are K-major: hi, lo rows adjacent
    static constexpr int kASlabBytes = PLANES * kTcBM * 128;
    static constexpr int kBSlabBytes = PLANES * BN * 128;
    static constexpr int kATileBytes = KS * kASlabBytes;
    static constexpr int kBTileBytes = KS * kBSlabBytes;
    static constexpr int STAGES = (196608 / (kATileBytes + kBTileBytes)) > 8 ? 8 : (196608 / (kATileBytes + kBTileBytes));
    static constexpr int kKSteps = 4 * KS;
    static constexpr int kChunkKbOverride = 2 / KS;  // strict chunks stay 64 positions deep
    static_assert(STAGES >= 2, "wgrad tile configuration");

    // The box coordinates of the tile's four 32-row groups (channel, position shift of the
    // tap) and where its K range starts (image, K block within the image) are fixed per
    // tile; the producer derives them once here instead of per K block.
    struct Tile {
        int m0, f0, split;
        int img0, kb0;  // first K block of the split: image, block within the image
        int c0[kTcBM / 32], shift[kTcBM / 32];
    };

    __device__ static int num_tiles(const Params& p) { return p.tiles_m * p.tiles_f * p.splits; }
    __device__ static int num_kb(const Params& p) { return p.kb_per_split; }

    __device__ static Tile tile(const Params& p, int t) {
        const int split = t / (p.tiles_m * p.tiles_f);
        const int rest = t - split * p.tiles_m * p.tiles_f;
        Tile out;
        out.m0 = (rest / p.tiles_f) * kTcBM;
        out.f0 = (rest % p.tiles_f) * BN;
        out.split = split;
        const long long kg = static_cast<long long>(split) * p.kb_per_split;
        out.img0 = static_cast<int>(kg / p.kb_per_img);
        out.kb0 = static_cast<int>(kg - static_cast<long long>(out.img0) * p.kb_per_img);
#pragma unroll
        for (int g = 0; g < kTcBM / 32; ++g) {
            const int m = out.m0 + 32 * g;
            const int tap = m / p.cg;
            // rows past the last tap read channel coordinates beyond the map: zeros
            const bool real = tap < p.r * p.s;
            const int rr = real ? tap / p.s : 0;
            out.c0[g] = real ? m - tap * p.cg : p.cg;
            out.shift[g] = real ? rr * p.wp + (tap - rr * p.s) : 0;
        }
        return out;
    }

    __device__ static int valid_cols(const Params& p, const Tile& t) { return min(BN, p.kf - t.f0); }

    // K block kb of the split: positions [j0, j0 + 32 * KS) of one image (p.kb_per_img blocks per image);
    // slab j holds positions j0 + 32 j .. +31. t.kb0 + kb stays below 2^31 (checked on the host).
    __device__ static void load(const Params& p, const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* a_tile,
                                uint8_t* b_tile, uint64_t* bar, const Tile& t, int kb) {
        const int rel = t.kb0 + kb;
        const int q = static_cast<int>(fastdiv(static_cast<uint32_t>(rel), p.div_kb_per_img));
        const int img = t.img0 + q;
        const int j0 = (rel - q * p.kb_per_img) * 32 * KS;
#pragma unroll
        for (int j = 0; j < KS; ++j) {
            const int js = j0 + 32 * j;
#pragma unroll
            for (int g = 0; g < kTcBM / 32; ++g)
                tma_load_4d(a_tile + j * kASlabBytes + g * PLANES * 4096, ta, bar, t.c0[g], js + t.shift[g], img, 0);
            tma_load_4d(b_tile + j * kBSlabBytes, tb, bar, js, t.f0, img, 0);
        }
    }

    // Per slab A: [group of 32 M][plane][32 K rows][32 M] (128B swizzle, 32-byte atoms); B: [plane][BN][32 K].
    __device__ static uint64_t a_desc(uint32_t addr, int pl, int ks) {
        return umma_smem_desc(addr + (ks / 4) * kASlabBytes + pl * 4096 + (ks % 4) * 1024, PLANES * 4096, 512,
                              kLayoutSwizzle128B_Base32B);
    }
    __device__ static uint64_t b_desc(uint32_t addr, int pl, int ks) {
        return umma_smem_desc(addr + (ks / 4) * kBSlabBytes + pl * BN * 128 + (ks % 4) * 32, 16, 1024,
                              kLayoutSwizzle128B);
    }

    template <int COUNT>
    __device__ static void store(const Params& p, const Tile& t, int row_in_tile, int col0_in_tile, const float* v) {
        const long long rows_alloc = static_cast<long long>(p.tiles_m) * kTcBM;
        float* dst = p.partial + (static_cast<long long>(t.split) * rows_alloc + t.m0 + row_in_tile) * p.ld_partial +
                     t.f0 + col0_in_tile;
#pragma unroll
        for (int e = 0; e < COUNT; e += 4) *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
    }
};

}  // namespace mfb
