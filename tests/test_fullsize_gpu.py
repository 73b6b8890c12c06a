"""GPU tier: the benchmark configurations at full size.

* 2048^3 (square bench): the whole C against the reference's compiled gemm_f32 and FP64.
* 8192 x 4096 x 11008 linear layer, padded strides, alpha 0.5, beta 1 (strict and TF32):
  a seeded 64 x 64 block against the oracle's per-element gemm_f32 and FP64, plus the
  reference benchmark's own 97-position rule (benchmarks/bench_gemm_fair.cpp:76-95).
* 32768^3 (the multi-GPU configuration on one GPU): a seeded 64 x 64 block, as the
  configuration's own validation prescribes.
Inputs are generated on the device (seeded) and only the sampled rows/columns travel."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import assert_fair_bench_rule, assert_strict, assert_tf32

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _sample(m, n, count=64, seed=3):
    rng = np.random.default_rng(seed)
    rows = np.sort(rng.choice(m, size=count, replace=False))
    cols = np.sort(rng.choice(n, size=count, replace=False))
    return rows, cols


def _gpu_uniform(shape, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.rand(shape, device="cuda", generator=g) * 2 - 1


def test_square_2048_whole_matrix_against_reference():
    n = 2048
    A, B = _gpu_uniform((n, n), 1), _gpu_uniform((n, n), 2)
    C = mf.gemm(A, B)
    torch.cuda.synchronize()
    a, b, got = A.cpu().numpy(), B.cpu().numpy(), C.cpu().numpy()
    ref32 = np.zeros(n * n, np.float32)
    oracle.gemm_f32(n, n, n, a, n, b, n, ref32, n, impl="reference" if oracle.reference_available() else "restatement")
    ref64 = a.astype(np.float64) @ b.astype(np.float64)
    e = assert_strict(got, ref32.reshape(n, n), ref64, n, 1.0, 1.0, "2048^3")
    assert e["gpu_vs_fp64"] < 5e-7  # measured 2.2e-7; the CPU oracle is at 8.1e-7


@pytest.mark.parametrize("precision", [mf.GemmPrecision.fp32, mf.GemmPrecision.tf32])
def test_linear_layer_full_size_sampled(precision):
    m, k, n, lda, ldb, ldc = 8192, 4096, 11008, 4128, 11040, 11040
    g = torch.Generator(device="cuda").manual_seed(20261001)
    Abuf = torch.randn((m, lda), device="cuda", generator=g)
    Bbuf = torch.randn((k, ldb), device="cuda", generator=g) / 64.0
    Cbuf = torch.randn((m, ldc), device="cuda", generator=g)
    rows, cols = _sample(m, n)
    c_in = Cbuf[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")].cpu().numpy()
    pad_before = Cbuf[:, n:].clone()
    mf.sgemm(Abuf[:, :k], Bbuf[:, :n], Cbuf[:, :n], 0.5, 1.0, mf.GemmOptions(precision=precision))
    mf.sync()
    assert torch.equal(Cbuf[:, n:], pad_before)
    a_rows = Abuf[torch.as_tensor(rows, device="cuda"), :k].cpu().numpy()
    b_cols = Bbuf[:, torch.as_tensor(cols, device="cuda")].cpu().numpy()
    got = Cbuf[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")].cpu().numpy()
    # The sampled oracle needs the full-size column-tile semantics: n = 11008 is a multiple of 16,
    # so every element is one FMA chain; the gathered block reproduces it exactly.
    ref32 = oracle.gemm_f32_sampled(np.arange(64), np.arange(64), 64, k, a_rows, k, b_cols, 64, c_in, 0.5, 1.0)
    ref64 = 0.5 * (a_rows.astype(np.float64) @ b_cols.astype(np.float64)) + c_in
    if precision == mf.GemmPrecision.fp32:
        assert_strict(got, ref32, ref64, k, float(np.abs(a_rows).max()), float(np.abs(b_cols).max()), "linear")
    else:
        assert_tf32(got, ref32, "linear tf32")
    assert_fair_bench_rule(got - c_in, 0.5 * a_rows, b_cols, precision == mf.GemmPrecision.tf32, "linear")


def test_square_32768_sampled_block():
    n = 32768
    A, B = _gpu_uniform((n, n), 11), _gpu_uniform((n, n), 12)
    C = torch.empty((n, n), device="cuda")
    mf.sgemm(A, B, C)
    mf.sync()
    rows, cols = _sample(n, n, seed=5)
    a_rows = A[torch.as_tensor(rows, device="cuda")].cpu().numpy()
    b_cols = B[:, torch.as_tensor(cols, device="cuda")].cpu().numpy()
    got = C[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")].cpu().numpy()
    del A, B, C
    torch.cuda.empty_cache()
    ref32 = oracle.gemm_f32_sampled(np.arange(64), np.arange(64), 64, n, a_rows, n, b_cols, 64)
    ref64 = a_rows.astype(np.float64) @ b_cols.astype(np.float64)
    e = assert_strict(got, ref32, ref64, n, 1.0, 1.0, "32768^3")
    assert e["gemm_f32_vs_fp64"] > e["gpu_vs_fp64"]  # the device result is closer to FP64 than the CPU oracle
