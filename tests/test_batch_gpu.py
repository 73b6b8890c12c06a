"""GPU tier: strided-batched GEMM (batch_matmul and its backward) against the oracle.

Replaces cublasSgemmStridedBatched in src/nn/batch.cu:12-35 and
src/nn/backward/batched_matmul.inc:7-55. Known answers: tests/integration/test_batch.cpp:21-43
and tests/integration/test_autograd.cpp:262-279; every other case compares each batch entry
with the oracle's gemm_f32 and an FP64 product under the strict-FP32 gates."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import assert_strict, assert_tf32, to_dev

pytestmark = pytest.mark.gpu

FP32, TF32 = mf.GemmPrecision.fp32, mf.GemmPrecision.tf32


def _t(values, shape):
    return to_dev(np.asarray(values, np.float32).reshape(shape))


def test_known_answers_test_batch():
    left = _t([1, 2, 3, 4, 5, 6, 7, 8], (2, 2, 2))
    right = _t([1, 0, 0, 1, 2, 1, 1, 2], (2, 2, 2))
    result = mf.batch_matmul(left, right)
    assert tuple(result.shape) == (2, 2, 2)
    r = result.cpu().numpy().reshape(-1)
    assert abs(r[0] - 1.0) < 1e-4 and abs(r[3] - 4.0) < 1e-4  # batch 0 equals A0 * B0 = A0
    np.testing.assert_allclose(result.cpu().numpy()[1], [[5 * 2 + 6, 5 + 12], [7 * 2 + 8, 7 + 16]], rtol=0, atol=1e-5)
    identity = _t([1, 0, 0, 1, 1, 0, 0, 1], (2, 2, 2))
    gl = mf.batch_matmul_backward_left(identity, right).cpu().numpy().reshape(-1)
    assert abs(gl[1]) < 1e-4 and abs(gl[2]) < 1e-4  # B0^T = I
    gr = mf.batch_matmul_backward_right(identity, left).cpu().numpy().reshape(-1)
    assert abs(gr[1] - 3.0) < 1e-4 and abs(gr[2] - 2.0) < 1e-4  # A0^T = [[1,3],[2,4]]


def test_known_answers_test_autograd():
    """grad A = G x B^T and grad B = A^T x G with G = I: B^T and A^T per batch entry."""
    a = np.arange(1, 9, dtype=np.float32).reshape(2, 2, 2)
    b = np.array([0.5, 0.1, 0.2, 0.3, 0.4, 0.2, 0.1, 0.6], np.float32).reshape(2, 2, 2)
    g = np.tile(np.eye(2, dtype=np.float32), (2, 1, 1))
    ga = mf.batch_matmul_backward_left(to_dev(g), to_dev(b)).cpu().numpy()
    gb = mf.batch_matmul_backward_right(to_dev(g), to_dev(a)).cpu().numpy()
    assert np.abs(ga - b.transpose(0, 2, 1)).max() < 1e-3
    assert np.abs(gb - a.transpose(0, 2, 1)).max() < 1e-3


def _per_entry_reference(a_list, b_list, c_list, alpha, beta):
    """Oracle gemm_f32 and FP64 per batch entry on contiguous copies."""
    ref32, ref64 = [], []
    for a, b, c in zip(a_list, b_list, c_list):
        m, k = a.shape
        n = b.shape[1]
        r = np.ascontiguousarray(c, np.float32).copy().reshape(-1)
        oracle.gemm_f32(m, n, k, np.ascontiguousarray(a), k, np.ascontiguousarray(b), n, r, n, alpha, beta)
        ref32.append(r.reshape(m, n))
        ref64.append(alpha * (a.astype(np.float64) @ b.astype(np.float64)) + beta * c.astype(np.float64))
    return ref32, ref64


@pytest.mark.parametrize("precision", [FP32, TF32])
def test_seeded_padded_batch_against_oracle(precision):
    batch, m, n, k = 5, 300, 200, 333
    lda, ldb, ldc = k + 5, n + 3, n + 7
    sa, sb, sc = m * lda + 16, k * ldb + 4, m * ldc + 32
    rng = np.random.default_rng(11)
    abuf = rng.uniform(-1, 1, batch * sa).astype(np.float32)
    bbuf = rng.standard_normal(batch * sb).astype(np.float32)
    cbuf = rng.standard_normal(batch * sc).astype(np.float32)
    A = to_dev(abuf).as_strided((batch, m, k), (sa, lda, 1))
    B = to_dev(bbuf).as_strided((batch, k, n), (sb, ldb, 1))
    Cflat = to_dev(cbuf)
    C = Cflat.as_strided((batch, m, n), (sc, ldc, 1))
    mf.sgemm_strided_batched(A, B, C, 0.5, -1.0, mf.GemmOptions(precision=precision))
    mf.sync()
    got_flat = Cflat.cpu().numpy()
    a_list = [abuf[i * sa:i * sa + m * lda].reshape(m, lda)[:, :k] for i in range(batch)]
    b_list = [bbuf[i * sb:i * sb + k * ldb].reshape(k, ldb)[:, :n] for i in range(batch)]
    c_list = [cbuf[i * sc:i * sc + m * ldc].reshape(m, ldc)[:, :n] for i in range(batch)]
    ref32, ref64 = _per_entry_reference(a_list, b_list, c_list, 0.5, -1.0)
    for i in range(batch):
        block = got_flat[i * sc:i * sc + m * ldc].reshape(m, ldc)
        assert np.array_equal(block[:, n:], cbuf[i * sc:i * sc + m * ldc].reshape(m, ldc)[:, n:]), "padding written"
        if precision == FP32:
            assert_strict(block[:, :n], ref32[i], ref64[i], k, 1.0, float(np.abs(b_list[i]).max()), f"entry {i}")
        else:
            assert_tf32(block[:, :n], ref32[i], f"entry {i}")
    gaps = [got_flat[i * sc + m * ldc:(i + 1) * sc] for i in range(batch)]
    for i, gap in enumerate(gaps):
        assert np.array_equal(gap, cbuf[i * sc + m * ldc:(i + 1) * sc]), f"gap after entry {i} written"


def test_backward_products_against_oracle():
    batch, m, n, k = 3, 130, 70, 150
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (batch, m, k)).astype(np.float32)
    bm = rng.uniform(-1, 1, (batch, k, n)).astype(np.float32)
    g = rng.standard_normal((batch, m, n)).astype(np.float32)
    ga = mf.batch_matmul_backward_left(to_dev(g), to_dev(bm)).cpu().numpy()
    gb = mf.batch_matmul_backward_right(to_dev(g), to_dev(a)).cpu().numpy()
    for i in range(batch):
        r32, r64 = _per_entry_reference([g[i]], [bm[i].T.copy()], [np.zeros((m, k), np.float32)], 1.0, 0.0)
        assert_strict(ga[i], r32[0], r64[0], n, float(np.abs(g).max()), 1.0, f"G x B^T entry {i}")
        r32, r64 = _per_entry_reference([a[i].T.copy()], [g[i]], [np.zeros((k, n), np.float32)], 1.0, 0.0)
        assert_strict(gb[i], r32[0], r64[0], m, 1.0, float(np.abs(g).max()), f"A^T x G entry {i}")


def test_stride_zero_reuses_one_operand_and_epilogue():
    batch, m, n, k = 4, 96, 80, 64
    rng = np.random.default_rng(8)
    a = rng.uniform(-1, 1, (batch, m, k)).astype(np.float32)
    w = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    W = to_dev(w).unsqueeze(0).expand(batch, k, n)  # batch stride 0
    out = torch.empty((batch, m, n), device="cuda")
    mf.sgemm_strided_batched(to_dev(a), W, out, 1.0, 0.0, mf.GemmOptions(epilogue=mf.GemmEpilogue.bias_relu),
                             to_dev(bias))
    got = out.cpu().numpy()
    for i in range(batch):
        r = np.zeros(m * n, np.float32)
        oracle.gemm_f32(m, n, k, a[i], k, w, n, r, n)
        oracle.epilogue_f32(r, n, bias, m, n, 1)
        assert np.abs(got[i] - r.reshape(m, n)).max() <= oracle.elementwise_bound(k, 1.0, 1.0)


def test_many_small_entries():
    """300 entries of 17x9x13: more tiles than SMs, each entry a single partial tile."""
    batch, m, n, k = 300, 17, 9, 13
    rng = np.random.default_rng(2)
    a = rng.uniform(-1, 1, (batch, m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (batch, k, n)).astype(np.float32)
    got = mf.batch_matmul(to_dev(a), to_dev(b)).cpu().numpy()
    ref64 = np.einsum("bmk,bkn->bmn", a.astype(np.float64), b.astype(np.float64))
    assert oracle.normwise_rel(got, ref64) <= 1e-6
    assert np.abs(got - ref64).max() <= oracle.elementwise_bound(k, 1.0, 1.0)


def test_empty_and_invalid():
    z = mf.batch_matmul(torch.empty((0, 3, 4), device="cuda"), torch.empty((0, 4, 5), device="cuda"))
    assert tuple(z.shape) == (0, 3, 5)
    e = mf.batch_matmul(torch.ones((2, 3, 0), device="cuda"), torch.ones((2, 0, 5), device="cuda"))
    assert tuple(e.shape) == (2, 3, 5)  # k = 0: C = 0 (beta = 0)
    assert float(e.abs().max()) == 0.0
    with pytest.raises(mf.InvalidArgumentError):
        mf.batch_matmul(torch.ones((3, 4), device="cuda"), torch.ones((1, 4, 5), device="cuda"))
    with pytest.raises(mf.ShapeMismatchError):
        mf.batch_matmul(torch.ones((2, 3, 4), device="cuda"), torch.ones((3, 4, 5), device="cuda"))
    with pytest.raises(mf.ShapeMismatchError):
        mf.batch_matmul(torch.ones((2, 3, 4), device="cuda"), torch.ones((2, 5, 5), device="cuda"))
    # Overlapping outputs are rejected by the C ABI.
    buf = torch.zeros(64 * 64, device="cuda")
    overlapping = buf.as_strided((2, 8, 8), (8, 8, 1))
    with pytest.raises(mf.InvalidArgumentError):
        mf.sgemm_strided_batched(torch.ones((2, 8, 4), device="cuda"), torch.ones((2, 4, 8), device="cuda"),
                                 overlapping)
