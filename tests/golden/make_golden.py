"""Generates the golden fixtures in tests/golden/ by running the reference's OWN CPU code.

Every GEMM output here comes from the reference's gemm_f32 (src/hw/gemm.cpp:73,
avx2-4x16 path), compiled from its unmodified sources into oracle/_ref/libmfref_cpu.so
by oracle/Makefile. This script runs where the reference tree exists; the .npz files it
writes are committed and are what the tests read everywhere else (the GPU box has no
reference tree).

The reference has no CPU conv2d; conv fixtures come from the restatement of
conv2d_kernel (src/nn/conv.cu:22-49) and are pinned by the known answers of
tests/unit/test_conv.cpp:31-67,117-121, which tests/test_oracle.py checks.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def plan_case_inputs():
    """The deterministic operands of tests/unit/test_gemm_plan.cpp:16-23 (m,n,k = 7,9,5)."""
    m, n, k = 7, 9, 5
    av = np.array([((i % 11) - 5) * 0.17 for i in range(m * k)], dtype=np.float32)
    bv = np.array([((i % 7) - 3) * 0.23 for i in range(k * n)], dtype=np.float32)
    bias = np.array([(i - 4) * 0.11 for i in range(n)], dtype=np.float32)
    return m, n, k, av, bv, bias


def gemm_ref(m, n, k, a, lda, b, ldb, c, ldc, alpha, beta):
    out = np.array(c, dtype=np.float32, copy=True).reshape(-1)
    oracle.gemm_f32(m, n, k, a, lda, b, ldb, out, ldc, alpha, beta, impl="reference")
    return out


def main():
    if not oracle.reference_available():
        oracle.build()
    info = oracle.reference_info()
    cases = {}

    # 1. test_gemm_plan.cpp:14-34 operands, C = ones, alpha 0.7, beta -0.3 (row-major view;
    #    the transposed variants multiply the same logical matrices).
    m, n, k, av, bv, bias = plan_case_inputs()
    c0 = np.ones(m * n, dtype=np.float32)
    cases["plan_7x9x5"] = dict(m=m, n=n, k=k, lda=k, ldb=n, ldc=n, alpha=0.7, beta=-0.3, a=av, b=bv, c_in=c0,
                               bias=bias, c_out=gemm_ref(m, n, k, av, k, bv, n, c0, n, 0.7, -0.3))

    # 2. Seeded cases with padded strides, ragged 16-column tiles and the C2 distributions.
    specs = [
        ("edge_33x47x129", 33, 47, 129, 131, 52, 50, 0.5, 1.0, "uniform", "normal"),
        ("linear_64x80x300", 64, 80, 300, 300 + 32, 80 + 32, 80 + 32, 0.5, 1.0, "normal", "normal"),
        ("square_96", 96, 96, 96, 96, 96, 96, 1.0, 0.0, "uniform", "uniform"),
        ("kpanel_40x70x1100", 40, 70, 1100, 1100, 70, 70, 1.0, 0.0, "uniform", "uniform"),
        ("gemv_128x1x640", 128, 1, 640, 640, 1, 1, 1.0, 0.0, "uniform", "normal"),
        ("skinny_128x4x640", 128, 4, 640, 644, 4, 4, 1.0, 0.0, "uniform", "normal"),
        ("skinny_100x16x700", 100, 16, 700, 700, 16, 16, 0.5, 1.0, "uniform", "normal"),
        ("rowvec_1x127x2048", 1, 127, 2048, 2048, 127, 127, 1.0, 0.0, "uniform", "uniform"),
    ]
    for (name, m, n, k, lda, ldb, ldc, alpha, beta, da, db) in specs:
        seed = sum(map(ord, name))
        a = oracle.seeded(m * lda, da, seed=seed)
        b = oracle.seeded(k * ldb, db, seed=seed + 1, scale=(1.0 / 64.0) if name.startswith("linear") else 1.0)
        c_in = oracle.seeded(m * ldc, "normal", seed=seed + 2) if beta != 0.0 else np.zeros(m * ldc, np.float32)
        cases[name] = dict(m=m, n=n, k=k, lda=lda, ldb=ldb, ldc=ldc, alpha=alpha, beta=beta, a=a, b=b, c_in=c_in,
                           bias=np.zeros(n, np.float32), c_out=gemm_ref(m, n, k, a, lda, b, ldb, c_in, ldc, alpha,
                                                                       beta))

    # 3. k == 0: beta scaling only (gemm_f32 -> gemm_reference, src/hw/gemm.cpp:79-81).
    c0 = oracle.seeded(3 * 4, "normal", seed=77)
    cases["empty_k_3x4"] = dict(m=3, n=4, k=0, lda=1, ldb=4, ldc=4, alpha=1.0, beta=-2.0, a=np.zeros(1, np.float32),
                                b=np.zeros(4, np.float32), c_in=c0, bias=np.zeros(4, np.float32),
                                c_out=gemm_ref(3, 4, 0, np.zeros(1, np.float32), 1, np.zeros(4, np.float32), 4, c0,
                                               4, 1.0, -2.0))

    out = {}
    for name, d in cases.items():
        for key, val in d.items():
            out[f"{name}__{key}"] = np.asarray(val)
    out["meta__kernel"] = np.array(info["gemm_kernel_name"])
    np.savez_compressed(os.path.join(HERE, "gemm_golden.npz"), **out)

    # 4. conv2d: restatement outputs (see module docstring) on the C4a bench shape and small odd shapes.
    conv = {}
    conv_specs = [("c4a_8x3x32x32_k16", 8, 3, 32, 32, 16, 3, 3, 1, 1), ("odd_2x5x9x7_k6_s2", 2, 5, 9, 7, 6, 3, 2, 2, 1),
                  ("k1_1x4x6x6_k3", 1, 4, 6, 6, 3, 1, 1, 1, 0)]
    for (name, n, c, h, w, kf, r, s, stride, pad) in conv_specs:
        seed = sum(map(ord, name))
        x = oracle.seeded((n, c, h, w), "uniform", seed=seed)
        wt = oracle.seeded((kf, c, r, s), "normal", seed=seed + 1, scale=float(np.sqrt(2.0 / (c * r * s))))
        bias = oracle.seeded((kf,), "normal", seed=seed + 2, scale=0.1)
        y = oracle.conv2d_f32(x, wt, bias, stride, pad)
        for key, val in dict(x=x, w=wt, bias=bias, y=y, stride=stride, pad=pad).items():
            conv[f"{name}__{key}"] = np.asarray(val)
    np.savez_compressed(os.path.join(HERE, "conv_golden.npz"), **conv)
    print("wrote", sorted(cases), sorted(k.split("__")[0] for k in conv if k.endswith("__y")))


if __name__ == "__main__":
    main()
