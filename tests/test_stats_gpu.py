"""GPU tier: covariance / correlation (mfb_covariance, mfb_correlation) against the oracle.

Replaces matrix_pro::covariance / correlation (src/ops/reductions/covariance.inc:23-60), whose
product ran on cublasSgemm. Known answers: tests/unit/test_linalg.cpp:135-151. Seeded cases
compare with the oracle's restatement (col_mean_f32 / covariance_f32 / correlation_f32) and
with FP64 under the strict gates."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from helpers import STRICT_NORMWISE, to_dev

pytestmark = pytest.mark.gpu


def test_known_answers_test_linalg():
    cov = mf.covariance(to_dev(np.array([[1, 2], [3, 4], [5, 6]], np.float32))).cpu().numpy()
    assert cov.shape == (2, 2)
    assert abs(cov[0, 0] - 4.0) < 1e-2 and abs(cov[1, 1] - 4.0) < 1e-2
    corr = mf.correlation(to_dev(np.array([[1, 2], [2, 5]], np.float32))).cpu().numpy()
    assert abs(corr[0, 0] - 1.0) < 1e-3 and abs(corr[1, 1] - 1.0) < 1e-3 and abs(corr[0, 1] - 1.0) < 1e-3


def _check_cov(got, x, what):
    ref32 = oracle.covariance_f32(x)
    ref64 = np.cov(x.astype(np.float64), rowvar=False, ddof=1) if x.shape[0] > 1 else np.zeros((x.shape[1],) * 2)
    gate = max(STRICT_NORMWISE, oracle.normwise_rel(ref32, ref64))
    err = oracle.normwise_rel(got, ref64)
    assert err <= gate, f"{what}: normwise {err:.3e} > {gate:.3e}"
    xc = x - oracle.col_mean_f32(x)[None, :]
    bound = oracle.elementwise_bound(x.shape[0], float(np.abs(xc).max()), float(np.abs(xc).max()))
    bound /= max(x.shape[0] - 1, 1)
    assert np.abs(got - ref32).max() <= bound, what
    return err


@pytest.mark.parametrize("rows,cols,pad,offset", [(1001, 37, 0, 3.0), (5000, 300, 5, -1.5), (70000, 64, 0, 10.0),
                                                  (3, 200, 0, 0.0), (129, 1, 3, 2.0)])
def test_covariance_against_oracle(rows, cols, pad, offset):
    rng = np.random.default_rng(rows + cols)
    x = (rng.standard_normal((rows, cols)) + offset).astype(np.float32)
    buf = np.zeros((rows, cols + pad), np.float32)
    buf[:, :cols] = x
    X = to_dev(buf)[:, :cols]
    got = mf.covariance(X).cpu().numpy()
    _check_cov(got, x, f"{rows}x{cols}")


def test_covariance_tf32_and_correlation():
    rng = np.random.default_rng(4)
    x = (rng.standard_normal((4000, 96)) * np.linspace(0.1, 3.0, 96)[None, :] + 1.0).astype(np.float32)
    got_tf32 = mf.covariance(to_dev(x), mf.GemmPrecision.tf32).cpu().numpy()
    assert oracle.normwise_rel(got_tf32, oracle.covariance_f32(x)) <= 5e-3
    corr = mf.correlation(to_dev(x)).cpu().numpy()
    ref = oracle.correlation_f32(oracle.covariance_f32(x))
    assert np.all(np.diag(corr) == 1.0)
    assert np.abs(corr - ref).max() <= 1e-5
    assert np.abs(corr - np.corrcoef(x.astype(np.float64), rowvar=False)).max() <= 1e-5


def test_edge_cases():
    one_row = mf.covariance(to_dev(np.array([[1.0, 2.0, 3.0]], np.float32))).cpu().numpy()
    assert np.all(one_row == 0.0)  # centered row is zero; divisor max(rows - 1, 1) = 1
    x = np.array([[1, 5, 2], [1, 6, 4], [1, 7, 7]], np.float32)  # column 0 has zero variance
    corr = mf.correlation(to_dev(x)).cpu().numpy()
    assert np.all(np.diag(corr) == 1.0) and corr[0, 1] == 0.0 and corr[2, 0] == 0.0
    assert tuple(mf.covariance(torch.empty((0, 4), device="cuda")).shape) == (0, 4)
    assert tuple(mf.correlation(torch.empty((5, 0), device="cuda")).shape) == (5, 0)
