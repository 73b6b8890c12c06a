"""GPU tier (2+ GPUs): mfb_sgemm_multi, the row split over the GPUs of one process.

Row blocks of A and C sit on different GPUs, B (and the bias) on the root's; B reaches the
other GPUs by NCCL broadcasts in column panels. The assembled C is checked against the
oracle (the reference's gemm_f32 and FP64) with the strict-FP32 and TF32 gates; padding
beyond n of every C row must stay untouched. Skipped with fewer than 2 GPUs."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import assert_strict, assert_tf32
from matrixflash_pro_b200.distributed import sgemm_multi

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]

M, N, K, LDA, LDB, LDC = 1000, 1500, 2080, 2084, 1504, 1508
IMPL = "reference" if oracle.reference_available() else "restatement"


def _inputs(seed=5):
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1, 1, (M, LDA)).astype(np.float32)
    b = rng.standard_normal((K, LDB)).astype(np.float32)
    c = rng.standard_normal((M, LDC)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    return a, b, c, bias


def _oracle(a, b, c, alpha, beta, bias=None, epilogue=0):
    ref32 = c.copy()
    oracle.gemm_f32(M, N, K, a, LDA, b, LDB, ref32, LDC, alpha, beta, impl=IMPL)
    ref32 = np.ascontiguousarray(ref32[:, :N])
    ref64 = oracle.gemm_f64(M, N, K, a, LDA, b, LDB, c, LDC, alpha, beta)
    if epilogue:
        oracle.epilogue_f32(ref32, N, bias, M, N, epilogue - 1)
        ref64 = ref64 + bias.astype(np.float64)
        if epilogue == 2:
            ref64 = np.maximum(ref64, 0.0)
    return ref32, ref64


def _run(splits, devices, root, precision, alpha, beta, epilogue=0):
    a, b, c, bias = _inputs()
    a_blocks, c_blocks, bufs = [], [], []
    r0 = 0
    for rows, dev in zip(splits, devices):
        A = torch.from_numpy(a[r0:r0 + rows]).to(f"cuda:{dev}")
        C = torch.from_numpy(c[r0:r0 + rows]).to(f"cuda:{dev}")
        a_blocks.append(A[:, :K])
        c_blocks.append(C[:, :N])
        bufs.append(C)
        r0 += rows
    B = torch.from_numpy(b).to(f"cuda:{devices[root]}")[:, :N]
    bias_t = torch.from_numpy(bias).to(f"cuda:{devices[root]}") if epilogue else None
    sgemm_multi(a_blocks, B, c_blocks, alpha, beta, precision, root, bias_t, epilogue)
    got = np.concatenate([buf.cpu().numpy() for buf in bufs])
    assert np.array_equal(got[:, N:], c[:, N:]), "row padding of C was written"
    ref32, ref64 = _oracle(a, b, c, alpha, beta, bias, epilogue)
    if precision == mf.GemmPrecision.fp32:
        assert_strict(got[:, :N], ref32, ref64, K, np.abs(a[:, :K]).max(), np.abs(b[:, :N]).max(), "sgemm_multi")
    else:
        assert_tf32(got[:, :N], ref32, "sgemm_multi")
    for dev in set(devices):
        assert mf.device_status(dev) == 0


@pytest.mark.parametrize("precision", [mf.GemmPrecision.fp32, mf.GemmPrecision.tf32])
def test_two_gpus_b_on_the_first(precision):
    _run([600, 400], [0, 1], 0, precision, 0.5, 1.0)


def test_b_on_the_second_gpu_with_bias_relu():
    _run([333, 667], [1, 0], 1, mf.GemmPrecision.fp32, 0.75, -0.5, epilogue=2)


def test_a_gpu_without_rows_still_joins_the_broadcast():
    _run([1000, 0], [0, 1], 1, mf.GemmPrecision.fp32, 1.0, 0.0)


def test_one_block_runs_without_nccl():
    _run([1000], [1], 0, mf.GemmPrecision.fp32, 0.5, 1.0)
