"""CPU tier: the covariance/correlation oracle pinned on the reference's known answers
(tests/unit/test_linalg.cpp:135-151) and against FP64, and host tensors rejected by the
product API (no CPU path)."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle


def test_oracle_known_answers():
    cov = oracle.covariance_f32(np.array([[1, 2], [3, 4], [5, 6]], np.float32))
    assert abs(cov[0, 0] - 4.0) < 1e-2 and abs(cov[1, 1] - 4.0) < 1e-2
    corr = oracle.correlation_f32(oracle.covariance_f32(np.array([[1, 2], [2, 5]], np.float32)))
    assert abs(corr[0, 0] - 1.0) < 1e-3 and abs(corr[1, 1] - 1.0) < 1e-3 and abs(corr[0, 1] - 1.0) < 1e-3


def test_oracle_against_fp64():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal((1001, 37)) + 3).astype(np.float32)
    assert oracle.normwise_rel(oracle.covariance_f32(x), np.cov(x.astype(np.float64), rowvar=False)) < 2e-6
    mean = oracle.col_mean_f32(x)
    assert np.abs(mean - x.astype(np.float64).mean(axis=0)).max() < 1e-5


def test_host_tensors_are_rejected():
    with pytest.raises(mf.InvalidArgumentError):
        mf.covariance(torch.ones(4, 3))
    with pytest.raises(mf.InvalidArgumentError):
        mf.correlation(torch.ones(4, 3))
