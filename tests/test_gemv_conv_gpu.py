"""GPU tier: GEMV / skinny GEMM and conv2d forward against the oracle.

GEMV replaces gemm_gemv (src/ops/gemm/gemm_gemv.cu:86-110); conv2d replaces
conv2d_kernel (src/nn/conv.cu:22-49). Known answers: tests/unit/test_conv.cpp:31-67,117-121."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import assert_strict, assert_tf32, to_dev

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["gemv_128x1x640", "skinny_128x4x640", "skinny_100x16x700", "rowvec_1x127x2048"])
def test_gemv_golden(golden_gemm, name):
    g = golden_gemm[name]
    m, n, k = int(g["m"]), int(g["n"]), int(g["k"])
    lda, ldb, ldc = int(g["lda"]), int(g["ldb"]), int(g["ldc"])
    A = to_dev(g["a"][: m * lda].reshape(m, lda))[:, :k]
    B = to_dev(g["b"][: k * ldb].reshape(k, ldb))[:, :n]
    C = to_dev(g["c_in"].reshape(m, ldc).copy())
    mf.gemv(A, B, C[:, :n], float(g["alpha"]), float(g["beta"]))
    mf.sync()
    got = C.cpu().numpy()[:, :n]
    ref32 = g["c_out"].reshape(m, ldc)[:, :n]
    ref64 = oracle.gemm_f64(m, n, k, g["a"], lda, g["b"], ldb, g["c_in"], ldc, float(g["alpha"]), float(g["beta"]))
    assert_strict(got, ref32, ref64, k, np.abs(g["a"]).max(), np.abs(g["b"]).max(), name)


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 8, 9, 16])
def test_gemv_widths_and_strides(n):
    m, k = 1003, 1537
    lda, ldb, ldc = k + 3, n + 1, n + 2
    a = oracle.seeded(m * lda, seed=n)
    b = oracle.seeded(k * ldb, "normal", seed=n + 1)
    c0 = oracle.seeded(m * ldc, "normal", seed=n + 2)
    A = to_dev(a.reshape(m, lda))[:, :k]
    B = to_dev(b.reshape(k, ldb))[:, :n]
    C = to_dev(c0.reshape(m, ldc).copy())
    mf.gemv(A, B, C[:, :n], 0.75, -0.5)
    mf.sync()
    got = C.cpu().numpy()
    ref = c0.copy()
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, ref, ldc, 0.75, -0.5)
    ref = ref.reshape(m, ldc)
    assert np.array_equal(got[:, n:], ref[:, n:])
    assert_strict(got[:, :n], ref[:, :n], oracle.gemm_f64(m, n, k, a, lda, b, ldb, c0, ldc, 0.75, -0.5), k,
                  np.abs(a).max(), np.abs(b).max())


# 16-byte aligned operands with lda, ldb multiples of 4 (or a contiguous x for n = 1) take
# the TMA tile kernel. The shapes cover the 1-, 4-, 8- and 16-column variants, each
# rows-per-lane instance (tile rows <= 32, <= 64, <= 112, <= 128), CTAs that own two
# tiles (m = 20000), k not a multiple of the 128-k stage, and a k shorter than one stage.
@pytest.mark.parametrize("m,n,k,ldb", [(1003, 5, 1537, 12), (300, 8, 5000, 12), (6000, 9, 700, 16),
                                       (16000, 16, 300, 20), (20000, 12, 513, 16), (17000, 16, 129, 16),
                                       (2000, 16, 40, 16), (5000, 1, 777, 1), (20000, 1, 1000, 1),
                                       (3000, 1, 600, 4), (9000, 3, 1100, 4), (16384, 4, 2000, 8)])
def test_gemv_tile_kernel_shapes(m, n, k, ldb):
    lda, ldc = (k + 3) // 4 * 4 + 4, n + 3
    a = oracle.seeded(m * lda, seed=m + n)
    b = oracle.seeded(k * ldb, "normal", seed=k)
    c0 = oracle.seeded(m * ldc, "normal", seed=n)
    A = to_dev(a.reshape(m, lda))[:, :k]
    B = to_dev(b.reshape(k, ldb))[:, :n]
    C = to_dev(c0.reshape(m, ldc).copy())
    assert A.data_ptr() % 16 == 0 and B.data_ptr() % 16 == 0
    mf.gemv(A, B, C[:, :n], 0.75, -0.5)
    mf.sync()
    got = C.cpu().numpy()
    ref = c0.copy()
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, ref, ldc, 0.75, -0.5)
    ref = ref.reshape(m, ldc)
    assert np.array_equal(got[:, n:], ref[:, n:]), "columns beyond n were written"
    assert_strict(got[:, :n], ref[:, :n], oracle.gemm_f64(m, n, k, a, lda, b, ldb, c0, ldc, 0.75, -0.5), k,
                  np.abs(a).max(), np.abs(b).max(), f"{m}x{n}x{k}")


def test_gemv_tile_kernel_bias_epilogues():
    """bias + ReLU / GELU through a plan whose path is the tile kernel (n = 12)."""
    m, n, k = 5000, 12, 1000
    a = oracle.seeded(m * k, seed=1)
    b = oracle.seeded(k * n, "normal", seed=2)
    bias = oracle.seeded(n, "normal", seed=3)
    for ep in (mf.GemmEpilogue.bias_relu, mf.GemmEpilogue.bias_gelu):
        C = torch.empty((m, n), device="cuda")
        mf.sgemm(to_dev(a.reshape(m, k)), to_dev(b.reshape(k, n)), C, 1.0, 0.0, mf.GemmOptions(epilogue=ep),
                 to_dev(bias))
        mf.sync()
        ref = np.zeros(m * n, np.float32)
        oracle.gemm_f32(m, n, k, a, k, b, n, ref, n)
        oracle.epilogue_f32(ref, n, bias, m, n, int(ep) - 1)  # oracle modes: 0 bias, 1 +ReLU, 2 +GELU
        err = np.abs(C.cpu().numpy() - ref.reshape(m, n)).max()
        # ReLU is 1-Lipschitz and tanh-GELU at most 1.13: the GEMM bound carries over.
        assert err <= 1.13 * oracle.elementwise_bound(k, np.abs(a).max(), np.abs(b).max()), (ep, err)


@pytest.mark.slow
@pytest.mark.parametrize("n", [1, 4, 16])
def test_gemv_full_size_sampled_rows(n):
    """The 16384 x 16384 GEMV configuration: sampled rows against the oracle (1 GiB operand)."""
    m = k = 16384
    g = torch.Generator(device="cuda").manual_seed(7)
    A = torch.rand((m, k), device="cuda", generator=g) * 2 - 1
    X = torch.randn((k, n), device="cuda", generator=g)
    Y = torch.empty((m, n), device="cuda")
    mf.gemv(A, X, Y)
    mf.sync()
    rows = np.array([0, 1, 4095, 8191, 12000, 16383])
    a_rows = A[torch.as_tensor(rows, device="cuda")].cpu().numpy()
    x = X.cpu().numpy()
    ref32 = oracle.gemm_f32_sampled(np.arange(len(rows)), np.arange(n), n, k, a_rows, k, x, n)
    ref64 = a_rows.astype(np.float64) @ x.astype(np.float64)
    got = Y[torch.as_tensor(rows, device="cuda")].cpu().numpy()
    assert_strict(got, ref32, ref64, k, 1.0, float(np.abs(x).max()))


@pytest.mark.parametrize("precision", [mf.GemmPrecision.fp32, mf.GemmPrecision.tf32])
def test_conv_golden(golden_conv, precision):
    for name, g in golden_conv.items():
        y = mf.conv2d(to_dev(g["x"]), to_dev(g["w"]), to_dev(g["bias"]), int(g["stride"]), int(g["pad"]), precision)
        got = y.cpu().numpy()
        assert got.shape == g["y"].shape
        y64 = oracle.conv2d_f64(g["x"], g["w"], g["bias"], int(g["stride"]), int(g["pad"]))
        tol = 1e-6 if precision == mf.GemmPrecision.fp32 else 5e-3
        assert oracle.normwise_rel(got, y64) <= max(tol, oracle.normwise_rel(g["y"], y64)), name


def test_conv_known_answers():
    """test_conv.cpp:31-67,117-121."""
    one = to_dev(np.ones((1, 1, 1, 1), np.float32))
    b0 = to_dev(np.zeros(1, np.float32))
    x2 = to_dev(np.arange(1, 5, dtype=np.float32).reshape(1, 1, 2, 2))
    y = mf.conv2d(x2, one, b0).cpu().numpy()
    assert y.shape == (1, 1, 2, 2) and abs(y[0, 0, 1, 1] - 4.0) < 1e-5
    x3 = to_dev(np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3))
    k2 = to_dev(np.ones((1, 1, 2, 2), np.float32))
    y = mf.conv2d(x3, k2, b0).cpu().numpy()
    assert abs(y[0, 0, 0, 0] - 12) < 1e-4 and abs(y[0, 0, 1, 1] - 28) < 1e-4
    y = mf.conv2d(x3, k2, to_dev(np.array([10.0], np.float32))).cpu().numpy()
    assert abs(y[0, 0, 0, 0] - 22) < 1e-4
    assert mf.conv2d(x2, one, b0, 1, 1).shape == (1, 1, 4, 4)
    x4 = to_dev(np.arange(1, 17, dtype=np.float32).reshape(1, 1, 4, 4))
    y = mf.conv2d(x4, one, b0, 2, 0).cpu().numpy()
    assert y.shape == (1, 1, 2, 2) and (y[0, 0, 0, 0], y[0, 0, 0, 1], y[0, 0, 1, 1]) == (1.0, 3.0, 11.0)


@pytest.mark.parametrize("n,c,h,w,k,r,s,stride,pad", [
    (2, 64, 56, 56, 64, 3, 3, 1, 1), (3, 7, 13, 11, 5, 3, 3, 1, 1), (1, 16, 20, 24, 32, 5, 5, 2, 2),
    # 3 channels, 28 MFLOP: the direct kernel (narrow-channel rule), past the plain FLOP cutoff
    (32, 3, 32, 32, 16, 3, 3, 1, 1),
    (2, 3, 9, 9, 4, 1, 1, 1, 0), (1, 33, 17, 15, 48, 3, 1, 1, 1),
    # wide rows (a 128-position tile spans less than two padded rows); 200 filters: one
    # 256-wide filter tile (no stacked B); 160 filters: BN = 256 as well
    (8, 8, 8, 100, 16, 3, 3, 1, 1), (2, 40, 6, 130, 200, 3, 3, 1, 1), (1, 32, 12, 12, 160, 3, 3, 1, 1),
    # BN = 32 and BN = 128 filter tiles (stacked B only up to 64 filters)
    (8, 16, 20, 20, 24, 3, 3, 1, 1), (1, 64, 14, 14, 128, 3, 3, 1, 1),
    # padded width beyond the row-wise prepass tile: the generic 64-position prepass
    (16, 4, 3, 520, 8, 3, 3, 1, 1),
    # odd channels / widths / filter counts above the direct-kernel cutoff (1e7 FLOP): tcgen05 path
    (8, 7, 33, 31, 40, 3, 3, 1, 1), (8, 33, 17, 15, 48, 3, 1, 1, 1), (64, 32, 20, 20, 64, 1, 1, 1, 0),
    (3, 5, 45, 37, 19, 5, 5, 1, 2),
    # many stacked-B tiles per SM; the second case leaves most of each image's last tile empty
    (40, 20, 30, 30, 64, 3, 3, 1, 1), (150, 33, 17, 15, 48, 3, 3, 1, 1),
    # 7x7 stem (49 taps, one channel slab each); 96 channels = 3 slabs per tap, so two-slab K blocks
    # straddle taps
    (8, 3, 64, 64, 64, 7, 7, 1, 3), (4, 96, 20, 20, 64, 3, 3, 1, 1)])
def test_conv_seeded_against_restatement(n, c, h, w, k, r, s, stride, pad):
    x = oracle.seeded((n, c, h, w), seed=c)
    wt = oracle.seeded((k, c, r, s), "normal", seed=k, scale=float(np.sqrt(2.0 / (c * r * s))))
    bias = oracle.seeded((k,), "normal", seed=3, scale=0.1)
    got = mf.conv2d(to_dev(x), to_dev(wt), to_dev(bias), stride, pad).cpu().numpy()
    ref = oracle.conv2d_f32(x, wt, bias, stride, pad)
    ref64 = oracle.conv2d_f64(x, wt, bias, stride, pad)
    assert oracle.normwise_rel(got, ref64) <= max(1e-6, oracle.normwise_rel(ref, ref64))
    assert oracle.max_abs(got, ref) <= 1e-5 * c * r * s * float(np.abs(x).max() * np.abs(wt).max())


# TF32 tiles: 16/32/64 filters take four 32-channel slabs per K block, which straddle taps when
# the channels fill 1, 2 or 3 slabs per tap; 128 and 256 filters take one slab.
@pytest.mark.parametrize("n,c,h,w,k,r,s,pad", [
    (8, 16, 20, 20, 24, 3, 3, 1), (8, 40, 18, 18, 32, 3, 3, 1), (4, 96, 20, 20, 64, 3, 3, 1),
    (8, 3, 64, 64, 64, 7, 7, 3), (2, 64, 20, 20, 128, 3, 3, 1), (2, 32, 14, 14, 200, 3, 3, 1)])
def test_conv_tf32_seeded(n, c, h, w, k, r, s, pad):
    x = oracle.seeded((n, c, h, w), seed=c + 1)
    wt = oracle.seeded((k, c, r, s), "normal", seed=k + 1, scale=float(np.sqrt(2.0 / (c * r * s))))
    bias = oracle.seeded((k,), "normal", seed=5, scale=0.1)
    got = mf.conv2d(to_dev(x), to_dev(wt), to_dev(bias), 1, pad, mf.GemmPrecision.tf32).cpu().numpy()
    assert_tf32(got, oracle.conv2d_f32(x, wt, bias, 1, pad), f"conv tf32 {(n, c, h, w, k, r, s)}")


@pytest.mark.slow
def test_conv_full_size_sampled():
    """256 x 64 x 56 x 56 with 64 3x3 filters: sampled images against the restatement."""
    n, c, h, w, k = 256, 64, 56, 56, 64
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.rand((n, c, h, w), device="cuda", generator=g) * 2 - 1
    wt = torch.randn((k, c, 3, 3), device="cuda", generator=g) * float(np.sqrt(2.0 / (c * 9)))
    bias = torch.zeros(k, device="cuda")
    y = mf.conv2d(x, wt, bias, 1, 1)
    mf.sync()
    for img in (0, 131, 255):
        xs = x[img:img + 1].cpu().numpy()
        ref = oracle.conv2d_f32(xs, wt.cpu().numpy(), bias.cpu().numpy(), 1, 1)
        ref64 = oracle.conv2d_f64(xs, wt.cpu().numpy(), bias.cpu().numpy(), 1, 1)
        got = y[img:img + 1].cpu().numpy()
        assert oracle.normwise_rel(got, ref64) <= max(1e-6, oracle.normwise_rel(ref, ref64))
