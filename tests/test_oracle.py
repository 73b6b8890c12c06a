"""CPU tier: the oracle itself is pinned before anything is compared against it.

* The C restatement of gemm_f32 must equal, bit for bit, the golden outputs that the
  reference's own gemm_f32 produced (tests/golden/make_golden.py), and the compiled
  reference itself wherever oracle/_ref was built.
* Known answers from the reference's tests: tests/unit/test_gemm_plan.cpp:14-34,36-50,
  tests/unit/test_operations.cpp:30-47, tests/unit/test_conv.cpp:31-67,117-121.
"""
import numpy as np
import pytest

import oracle


def test_restatement_matches_reference_golden_bit_exact(golden_gemm):
    assert len(golden_gemm) >= 10
    for name, g in golden_gemm.items():
        c = np.array(g["c_in"], dtype=np.float32, copy=True)
        oracle.gemm_f32(int(g["m"]), int(g["n"]), int(g["k"]), g["a"], int(g["lda"]), g["b"], int(g["ldb"]), c,
                        int(g["ldc"]), float(g["alpha"]), float(g["beta"]))
        assert np.array_equal(c.view(np.uint32), g["c_out"].view(np.uint32)), name


@pytest.mark.skipif(not oracle.reference_available(), reason="reference CPU GEMM not built here")
@pytest.mark.parametrize("m,n,k,lda,ldb,ldc,alpha,beta", [
    (1, 1, 1, 1, 1, 1, 1.0, 0.0), (5, 17, 1025, 1030, 20, 21, -1.5, 2.0), (130, 250, 513, 520, 256, 260, 1.0, 1.0),
    (64, 64, 600, 600, 64, 64, 1.0, 0.0), (4, 16, 3, 3, 16, 16, 0.5, 1.0), (31, 33, 512, 512, 40, 33, 1.0, -0.25)])
def test_restatement_matches_compiled_reference(m, n, k, lda, ldb, ldc, alpha, beta):
    a = oracle.seeded(m * lda, seed=m + 1)
    b = oracle.seeded(k * ldb, "normal", seed=n + 2)
    c0 = oracle.seeded(m * ldc, "normal", seed=k + 3)
    c_ref, c_rest = c0.copy(), c0.copy()
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, c_ref, ldc, alpha, beta, impl="reference")
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, c_rest, ldc, alpha, beta, impl="restatement")
    assert np.array_equal(c_ref.view(np.uint32), c_rest.view(np.uint32))
    s_ref, s_rest = c0.copy(), c0.copy()
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, s_ref, ldc, alpha, beta, impl="reference_scalar")
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, s_rest, ldc, alpha, beta, impl="scalar")
    assert np.array_equal(s_ref.view(np.uint32), s_rest.view(np.uint32))


@pytest.mark.skipif(not oracle.reference_available(), reason="reference CPU GEMM not built here")
def test_reference_reports_avx2_kernel():
    info = oracle.reference_info()
    assert info["gemm_kernel_name"] in ("avx2-4x16", "reference")
    assert 1 <= info["worker_count"] <= 32


def test_sampled_block_equals_full_product():
    m, n, k = 70, 90, 777
    a = oracle.seeded(m * k, seed=5)
    b = oracle.seeded(k * n, seed=6)
    c = np.zeros(m * n, np.float32)
    oracle.gemm_f32(m, n, k, a, k, b, n, c, n)
    rows = np.array([0, 3, 69, 33])
    cols = np.array([0, 15, 16, 89, 80])
    s = oracle.gemm_f32_sampled(rows, cols, n, k, a, k, b, n)
    assert np.array_equal(s, c.reshape(m, n)[np.ix_(rows, cols)])


def test_plan_known_answer_all_layouts(golden_gemm):
    """test_gemm_plan.cpp:14-34: 7x9x5, alpha 0.7, beta -0.3, C = ones, double-dot at 3e-5."""
    g = golden_gemm["plan_7x9x5"]
    m, n, k = 7, 9, 5
    a = g["a"].reshape(m, k).astype(np.float64)
    b = g["b"].reshape(k, n).astype(np.float64)
    ref = 0.7 * (a @ b) - 0.3
    out = g["c_out"].reshape(m, n)
    assert np.max(np.abs(out - ref)) < 3e-5
    for mode in (0, 1, 2):
        c = out.copy()
        oracle.epilogue_f32(c.reshape(-1), n, g["bias"], m, n, mode)
        r = ref + g["bias"].astype(np.float64)
        if mode == 1:
            r = np.maximum(r, 0)
        if mode == 2:
            r = 0.5 * r * (1 + np.tanh(0.7978845608 * (r + 0.044715 * r ** 3)))
        assert np.max(np.abs(c - r)) < 3e-5


def test_empty_k_applies_beta(golden_gemm):
    g = golden_gemm["empty_k_3x4"]
    assert np.array_equal(g["c_out"], (g["c_in"] * np.float32(-2.0)).astype(np.float32))


def test_operations_known_answers():
    """test_operations.cpp:30-47: [[1,2],[3,4]] x [[2,0],[1,2]] = [[4,4],[10,8]]; bias+ReLU."""
    a = np.array([1, 2, 3, 4], np.float32)
    b = np.array([2, 0, 1, 2], np.float32)
    c = np.zeros(4, np.float32)
    oracle.gemm_f32(2, 2, 2, a, 2, b, 2, c, 2)
    assert c.tolist() == [4, 4, 10, 8]
    oracle.epilogue_f32(c, 2, np.array([1, -10], np.float32), 2, 2, 1)
    assert c.tolist() == [5, 0, 11, 0]


def test_conv_restatement_known_answers():
    """test_conv.cpp:31-67,117-121."""
    one = np.ones((1, 1, 1, 1), np.float32)
    zero_b = np.zeros(1, np.float32)
    x2 = np.arange(1, 5, dtype=np.float32).reshape(1, 1, 2, 2)
    y = oracle.conv2d_f32(x2, one, zero_b)
    assert y.shape == (1, 1, 2, 2) and y[0, 0, 1, 1] == 4.0
    x3 = np.arange(1, 10, dtype=np.float32).reshape(1, 1, 3, 3)
    k2 = np.ones((1, 1, 2, 2), np.float32)
    y = oracle.conv2d_f32(x3, k2, zero_b)
    assert y.shape == (1, 1, 2, 2) and y[0, 0, 0, 0] == 12.0 and y[0, 0, 1, 1] == 28.0
    y = oracle.conv2d_f32(x3, k2, np.array([10.0], np.float32))
    assert y[0, 0, 0, 0] == 22.0
    assert oracle.conv2d_f32(x2, one, zero_b, 1, 1).shape == (1, 1, 4, 4)
    x4 = np.arange(1, 17, dtype=np.float32).reshape(1, 1, 4, 4)
    y = oracle.conv2d_f32(x4, one, zero_b, 2, 0)
    assert y.shape == (1, 1, 2, 2) and (y[0, 0, 0, 0], y[0, 0, 0, 1], y[0, 0, 1, 1]) == (1.0, 3.0, 11.0)


def test_conv_golden_reproduces(golden_conv):
    for name, g in golden_conv.items():
        y = oracle.conv2d_f32(g["x"], g["w"], g["bias"], int(g["stride"]), int(g["pad"]))
        assert np.array_equal(y, g["y"]), name
        y64 = oracle.conv2d_f64(g["x"], g["w"], g["bias"], int(g["stride"]), int(g["pad"]))
        assert oracle.normwise_rel(y, y64) < 1e-6, name


def test_oracle_own_error_against_fp64_is_recorded():
    """The strict gate compares against max(1e-6, err(gemm_f32, FP64)); check that quantity is sane."""
    m, n, k = 32, 32, 4096
    a = oracle.seeded(m * k, seed=1)
    b = oracle.seeded(k * n, seed=2)
    c = np.zeros(m * n, np.float32)
    oracle.gemm_f32(m, n, k, a, k, b, n, c, n)
    err = oracle.normwise_rel(c.reshape(m, n), oracle.gemm_f64(m, n, k, a, k, b, n))
    assert 1e-8 < err < 5e-6
