"""GPU tier: conv2d backward (mfb_conv2d_bwd_data / _filter / _bias) against the oracle.

Replaces conv2d_input_backward / conv2d_weight_backward / conv2d_bias_backward
(include/matrix_pro/nn/conv.hpp:25-29; kernels src/nn/backward/convolution_kernels.cuh:9-95).
Known answers: tests/integration/test_autograd.cpp:280-301. Seeded cases compare with the
oracle's restatements of the reference kernels (FP32, FMA) and with FP64."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import STRICT_NORMWISE, to_dev

pytestmark = pytest.mark.gpu

FP32, TF32 = mf.GemmPrecision.fp32, mf.GemmPrecision.tf32


def test_known_answers_test_autograd():
    """All-ones upstream gradient: sum(dx) = 4 * sum(w) = 6, sum(dw) = 80, db = 4."""
    x = to_dev(np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3))
    w = to_dev(np.array([0.25, -0.5, 1.0, 0.75], np.float32).reshape(1, 1, 2, 2))
    g = torch.ones((1, 1, 2, 2), device="cuda")
    assert abs(float(mf.conv2d_input_backward(g, x, w).sum()) - 6.0) < 1e-3
    assert abs(float(mf.conv2d_weight_backward(g, x, w).sum()) - 80.0) < 1e-3
    assert abs(float(mf.conv2d_bias_backward(g)[0]) - 4.0) < 1e-3


def _inputs(n, c, h, w, k, r, s, stride, pad, seed):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, s)) * np.sqrt(2.0 / (c * r * s))).astype(np.float32)
    p, q = (h + 2 * pad - r) // stride + 1, (w + 2 * pad - s) // stride + 1
    g = rng.standard_normal((n, k, p, q)).astype(np.float32)
    return x, wt, g


def _gate(got, ref32, ref64, length, max_a, max_b, what):
    err = oracle.normwise_rel(got, ref64)
    gate = max(STRICT_NORMWISE, oracle.normwise_rel(ref32, ref64))
    assert err <= gate, f"{what}: normwise {err:.3e} > {gate:.3e}"
    bound = oracle.elementwise_bound(length, max_a, max_b)
    assert oracle.max_abs(got, ref32) <= bound, f"{what}: elementwise bound {bound:.3e}"


SHAPES = [
    # (n, c, h, w, k, r, s, stride, pad): stride 1 above 1e7 FLOP runs on tcgen05
    (4, 64, 28, 28, 64, 3, 3, 1, 1),     # stacked-B tiles, cg = 64: 5 row tiles of the weight GEMM
    (8, 7, 33, 31, 40, 3, 3, 1, 1),      # odd channels (cg = 32), 40 filters
    (2, 33, 17, 15, 130, 3, 1, 1, 1),    # non-square filter, 130 filters (256-wide tiles)
    (3, 16, 21, 19, 24, 5, 5, 1, 2),     # 5x5, pad 2
    (2, 32, 20, 20, 48, 3, 3, 1, 0),     # pad 0: input-gradient padding R - 1 = 2
    (64, 32, 12, 12, 64, 1, 1, 1, 0),    # 1x1
    (52, 48, 24, 24, 40, 3, 3, 1, 1),    # 48 channels: the input gradient's conv has 48 "filters"
    (4, 3, 32, 32, 64, 7, 7, 1, 3),      # 7x7, 3 channels: 49 taps of one 32-row group each (13 row tiles)
    (2, 6, 11, 9, 5, 3, 3, 2, 1),        # stride 2: direct kernels
    (1, 3, 8, 8, 4, 3, 3, 1, 1),         # tiny: direct kernels
]


@pytest.mark.parametrize("shape", SHAPES)
def test_backward_against_oracle(shape):
    n, c, h, w, k, r, s, stride, pad = shape
    x, wt, g = _inputs(*shape, seed=sum(shape))
    X, W, G = to_dev(x), to_dev(wt), to_dev(g)
    p, q = g.shape[2], g.shape[3]
    dx = mf.conv2d_input_backward(G, X, W, stride, pad).cpu().numpy()
    dx32 = oracle.conv2d_input_backward(g, wt, x.shape, stride, pad)
    dx64 = oracle.conv2d_input_backward(g, wt, x.shape, stride, pad, f64=True)
    _gate(dx, dx32, dx64, k * r * s, float(np.abs(g).max()), float(np.abs(wt).max()), f"dx {shape}")
    dw = mf.conv2d_weight_backward(G, X, W, stride, pad).cpu().numpy()
    dw32 = oracle.conv2d_weight_backward(g, x, wt.shape, stride, pad)
    dw64 = oracle.conv2d_weight_backward(g, x, wt.shape, stride, pad, f64=True)
    _gate(dw, dw32, dw64, n * p * q, float(np.abs(g).max()), 1.0, f"dw {shape}")
    db = mf.conv2d_bias_backward(G).cpu().numpy()
    db32 = oracle.conv2d_bias_backward(g)
    db64 = oracle.conv2d_bias_backward(g, f64=True)
    _gate(db, db32, db64, n * p * q, float(np.abs(g).max()), 1.0, f"db {shape}")


@pytest.mark.parametrize("shape", [(4, 64, 28, 28, 64, 3, 3, 1, 1), (4, 96, 20, 20, 40, 3, 3, 1, 1),
                                   (4, 3, 32, 32, 64, 7, 7, 1, 3)])
def test_tf32_precision(shape):
    pad = shape[8]
    x, wt, g = _inputs(*shape, seed=3)
    X, W, G = to_dev(x), to_dev(wt), to_dev(g)
    dx = mf.conv2d_input_backward(G, X, W, 1, pad, TF32).cpu().numpy()
    assert oracle.normwise_rel(dx, oracle.conv2d_input_backward(g, wt, x.shape, 1, pad)) <= 5e-3
    dw = mf.conv2d_weight_backward(G, X, W, 1, pad, TF32).cpu().numpy()
    assert oracle.normwise_rel(dw, oracle.conv2d_weight_backward(g, x, wt.shape, 1, pad)) <= 5e-3


def test_full_size_sampled():
    """256 x 64 x 56 x 56, 64 3x3 filters, pad 1: dx of image 0 against the oracle, and 8 sampled
    (filter, channel) slices of dw (9 taps each, sums over all 802816 positions) against FP64."""
    n, c, h, w, k = 256, 64, 56, 56, 64
    gen = torch.Generator(device="cuda").manual_seed(21)
    X = torch.rand((n, c, h, w), device="cuda", generator=gen) * 2 - 1
    W = torch.randn((k, c, 3, 3), device="cuda", generator=gen) * float(np.sqrt(2.0 / (c * 9)))
    G = torch.randn((n, k, h, w), device="cuda", generator=gen)
    dx = mf.conv2d_input_backward(G, X, W, 1, 1)
    dw = mf.conv2d_weight_backward(G, X, W, 1, 1).cpu().numpy()
    mf.sync()
    g0, w0 = G[:1].cpu().numpy(), W.cpu().numpy()
    ref = oracle.conv2d_input_backward(g0, w0, (1, c, h, w), 1, 1)
    ref64 = oracle.conv2d_input_backward(g0, w0, (1, c, h, w), 1, 1, f64=True)
    _gate(dx[:1].cpu().numpy(), ref, ref64, k * 9, float(np.abs(g0).max()), float(np.abs(w0).max()), "dx image 0")
    rng = np.random.default_rng(4)
    pairs = [(int(f), int(ch)) for f, ch in zip(rng.choice(k, 8, replace=False), rng.choice(c, 8, replace=False))]
    got, want = [], []
    for f, ch in pairs:
        gf = G[:, f].double().cpu().numpy()                          # (n, h, w)
        xc = torch.nn.functional.pad(X[:, ch], (1, 1, 1, 1)).double().cpu().numpy()  # (n, h+2, w+2)
        for r in range(3):
            for s_ in range(3):
                want.append(float((gf * xc[:, r:r + h, s_:s_ + w]).sum()))
                got.append(float(dw[f, ch, r, s_]))
    err = oracle.normwise_rel(np.array(got), np.array(want))
    assert err <= STRICT_NORMWISE, f"dw sampled slices: normwise {err:.3e}"


def test_validation_errors():
    x = torch.zeros((1, 2, 5, 5), device="cuda")
    w = torch.zeros((3, 2, 3, 3), device="cuda")
    g = torch.zeros((1, 3, 3, 3), device="cuda")
    with pytest.raises(mf.ShapeMismatchError):
        mf.conv2d_input_backward(torch.zeros((1, 3, 4, 4), device="cuda"), x, w)
    with pytest.raises(mf.ShapeMismatchError):
        mf.conv2d_weight_backward(g, torch.zeros((1, 4, 5, 5), device="cuda"), w)
    with pytest.raises(mf.InvalidArgumentError):
        mf.conv2d_bias_backward(torch.zeros((3, 3), device="cuda"))
    with pytest.raises(mf.InvalidArgumentError):
        mf.conv2d_input_backward(g, x[0], w)
    empty = mf.conv2d_weight_backward(torch.zeros((0, 3, 3, 3), device="cuda"), torch.zeros((0, 2, 5, 5),
                                                                                              device="cuda"), w)
    assert float(empty.abs().max()) == 0.0
