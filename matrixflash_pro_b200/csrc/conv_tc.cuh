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

#include "tc_kernel.cuh"

namespace mfb {

struct ConvTcParams {
    int n_img, c, h, w, kf, r, s, pad;
    int hp, wp;         // padded input height / width
    int p_out, q_out;   // output height / width
    int ncb;            // 32-channel K blocks per tap
    int num_kb;         // r * s * ncb
    int tiles_pos;      // ceil(p_out * wp / 128) position tiles per image
    int tiles_f;        // filter tiles
    float* y;
    const float* bias;
    unsigned long long wait_limit_ns;
};

template <int BN, int PLANES>
constexpr int conv_stages() {
    return (196608 / (PLANES * (kTcBM + BN) * 128)) > 8 ? 8 : (196608 / (PLANES * (kTcBM + BN) * 128));
}

template <int BN_, int PLANES_>
struct ConvProblem {
    using Params = ConvTcParams;
    static constexpr int BN = BN_, PLANES = PLANES_, A_MN = 0, B_MN = 0;
    static constexpr bool kStackB = PLANES_ == 2 && BN_ <= 64;  // K-major weight tiles: hi, lo rows adjacent
    static constexpr int STAGES = conv_stages<BN_, PLANES_>();
    static constexpr int kATileBytes = PLANES * kTcBM * 128;
    static constexpr int kBTileBytes = PLANES * BN * 128;
    static constexpr int kKSteps = 4;  // 32 channels = 4 K steps of 8
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

    __device__ static void load(const Params& p, const CUtensorMap* ta, const CUtensorMap* tb, uint8_t* a_tile,
                                uint8_t* b_tile, uint64_t* bar, const Tile& t, int kb) {
        const int tap = kb / p.ncb;
        const int c0 = (kb - tap * p.ncb) * 32;
        const int r = tap / p.s;
        const int sc = tap - r * p.s;
        tma_load_4d(a_tile, ta, bar, c0, t.j0 + r * p.wp + sc, t.img, 0);
        tma_load_4d(b_tile, tb, bar, c0, t.f0, tap, 0);
    }

    // [plane][rows][32 channels], 128B swizzle: 8-row groups 1 KiB apart; a K step is 32 B.
    __device__ static uint64_t a_desc(uint32_t addr, int pl, int ks) {
        return umma_smem_desc(addr + pl * kTcBM * 128 + ks * 32, 16, 1024, kLayoutSwizzle128B);
    }
    __device__ static uint64_t b_desc(uint32_t addr, int pl, int ks) {
        return umma_smem_desc(addr + pl * BN * 128 + ks * 32, 16, 1024, kLayoutSwizzle128B);
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
            if (f < p.kf) base[f * plane] = v[e] + p.bias[f];
        }
    }
};

}  // namespace mfb
