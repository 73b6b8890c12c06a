"""Shared checks for the GPU parity tests.

Tolerances (stated here once, used everywhere):
* strict FP32 (3xTF32): ||C_gpu - C_fp64||_F / ||C_fp64||_F <= max(1e-6, err(gemm_f32, FP64)),
  because the reference's own gemm_f32 is already at 8e-7 (k=2048) .. 3e-6 (k=32768)
  against FP64; and max |C_gpu - C_gemm_f32| <= 1e-5 * k * max|A| * max|B|.
* TF32: ||C_gpu - C_gemm_f32||_F / ||C_gemm_f32||_F <= 5e-3.
* The reference's benchmark gate (benchmarks/bench_gemm_fair.cpp:76-95): at up to 97
  deterministic positions |c - dot| <= 1e-5 + (2e-6 strict | 2e-3 tf32) * sum|a_i b_i|.
"""
from __future__ import annotations

import numpy as np
import torch

import oracle

STRICT_NORMWISE = 1e-6
TF32_NORMWISE = 5e-3


def to_dev(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def strict_errors(gpu, ref_f32, ref_f64):
    return {
        "gpu_vs_gemm_f32": oracle.normwise_rel(gpu, ref_f32),
        "gpu_vs_fp64": oracle.normwise_rel(gpu, ref_f64),
        "gemm_f32_vs_fp64": oracle.normwise_rel(ref_f32, ref_f64),
        "max_abs_vs_gemm_f32": oracle.max_abs(gpu, ref_f32),
    }


def assert_strict(gpu, ref_f32, ref_f64, k, max_a, max_b, what=""):
    e = strict_errors(gpu, ref_f32, ref_f64)
    gate = max(STRICT_NORMWISE, e["gemm_f32_vs_fp64"])
    assert e["gpu_vs_fp64"] <= gate, f"{what}: {e} gate {gate:.3e}"
    bound = oracle.elementwise_bound(k, max_a, max_b)
    assert e["max_abs_vs_gemm_f32"] <= bound, f"{what}: {e} elementwise bound {bound:.3e}"
    return e


def assert_tf32(gpu, ref_f32, what=""):
    err = oracle.normwise_rel(gpu, ref_f32)
    assert err <= TF32_NORMWISE, f"{what}: tf32 normwise {err:.3e}"
    return err


def fair_positions(m, n, count=97):
    count = min(m * n, count)
    idx = [q * (m * n - 1) // max(1, count - 1) for q in range(count)]
    return [(i // n, i % n) for i in idx]


def assert_fair_bench_rule(c_gpu, a, b, tf32: bool, what=""):
    """bench_gemm_fair.cpp:76-95 on a (m x k) @ (k x n) product held as 2-D arrays."""
    m, n = c_gpu.shape
    coef = 2e-3 if tf32 else 2e-6
    for (i, j) in fair_positions(m, n):
        prods = a[i, :].astype(np.float64) * b[:, j].astype(np.float64)
        ref = prods.sum()
        tol = 1e-5 + coef * np.abs(prods).sum()
        v = float(c_gpu[i, j])
        assert np.isfinite(v) and abs(v - ref) <= tol, f"{what}: ({i},{j}) {v} vs {ref} tol {tol}"
