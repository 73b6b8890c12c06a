"""GPU tier: mfb_sgemm_host, the GEMM whose operands may live in host memory.

Replaces the GPU share of HeterogeneousScheduler::gemm (src/hw/scheduler.cpp:236-312):
B, A and C copied in, hw::cuda_gemm, C copied out. Here the rows of C stream through
the GPU in panels with the copies overlapping the GEMM; the results must meet the same
strict-FP32 gate as the device GEMM, whatever mix of host (pinned or pageable) and
device operands a call gets, including ragged last panels and every transpose."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
from helpers import STRICT_NORMWISE

pytestmark = pytest.mark.gpu

FP32, TF32 = mf.GemmPrecision.fp32, mf.GemmPrecision.tf32


def _rand(shape, gen, pin=True):
    t = torch.rand(shape, generator=gen) * 2 - 1
    return t.pin_memory() if pin else t


def _check(got, want64, precision=FP32):
    err = float((got.double() - want64).norm() / want64.norm())
    assert err <= (STRICT_NORMWISE if precision == FP32 else 5e-3), err


def _ref(a, b, c0, alpha, beta, ta=False, tb=False):
    A = a.cuda().double()
    B = b.cuda().double()
    A = A.t() if ta else A
    B = B.t() if tb else B
    return (alpha * (A @ B) + beta * c0.cuda().double()).cpu()


@pytest.mark.parametrize("precision", [FP32, TF32])
def test_host_operands_stream_in_panels(precision):
    """m = 6000 rows in panels of 1280 (4 full panels and a ragged one), pinned A, B, C, beta = 1."""
    gen = torch.Generator().manual_seed(5)
    m, n, k = 6000, 4096, 1024
    a, b, c0 = _rand((m, k), gen), _rand((k, n), gen), _rand((m, n), gen)
    c = c0.clone().pin_memory()
    mf.sgemm_host(a, b, c, 0.5, 1.0, mf.GemmOptions(precision=precision))
    mf.sync()
    _check(c, _ref(a, b, c0, 0.5, 1.0), precision)


def test_host_single_panel_equals_device_gemm():
    """A call that fits one panel runs the device GEMM of the same shape: identical bits."""
    gen = torch.Generator().manual_seed(6)
    m, n, k = 700, 900, 333
    a, b, c0 = _rand((m, k), gen), _rand((k, n), gen), _rand((m, n), gen)
    c = c0.clone().pin_memory()
    mf.sgemm_host(a, b, c, 1.5, -0.5)
    want = c0.cuda()
    mf.sgemm(a.cuda(), b.cuda(), want, 1.5, -0.5)
    mf.sync()
    assert torch.equal(c, want.cpu())


@pytest.mark.parametrize("where", ["pageable_a", "device_b", "device_a_host_c", "device_c"])
def test_mixed_host_and_device_operands(where):
    gen = torch.Generator().manual_seed(7)
    m, n, k = 5000, 3000, 768
    a, b, c0 = _rand((m, k), gen, pin=where != "pageable_a"), _rand((k, n), gen), _rand((m, n), gen)
    A = a.cuda() if where == "device_a_host_c" else a
    B = b.cuda() if where == "device_b" else b
    C = c0.cuda() if where == "device_c" else c0.clone().pin_memory()
    mf.sgemm_host(A, B, C, 1.0, 0.75)
    mf.sync()
    _check(C.cpu(), _ref(a, b, c0, 1.0, 0.75))


@pytest.mark.parametrize("ta,tb", [(True, False), (False, True), (True, True)])
def test_transposed_host_operands(ta, tb):
    gen = torch.Generator().manual_seed(8 + 2 * ta + tb)
    m, n, k = 4500, 2500, 640
    a = _rand((k, m) if ta else (m, k), gen)
    b = _rand((n, k) if tb else (k, n), gen)
    c0 = _rand((m, n), gen)
    c = c0.clone().pin_memory()
    mf.sgemm_host(a, b, c, 1.0, 1.0, mf.GemmOptions(transpose_left=ta, transpose_right=tb))
    mf.sync()
    _check(c, _ref(a, b, c0, 1.0, 1.0, ta, tb))


def test_padded_rows_beta_zero_and_bias_epilogue():
    """Padded host rows stay untouched; beta = 0 never reads C; a host bias feeds the epilogue."""
    gen = torch.Generator().manual_seed(9)
    m, n, k = 12289, 2051, 515  # panels of 4864 rows: two full, one ragged
    a_buf, b_buf = _rand((m, k + 5), gen), _rand((k, n + 3), gen)
    a, b = a_buf[:, :k], b_buf[:, :n]
    c_buf = torch.full((m, n + 7), float("nan")).pin_memory()
    c = c_buf[:, :n]
    bias = _rand((n,), gen)
    o = mf.GemmOptions(epilogue=mf.GemmEpilogue.bias_relu)
    mf.sgemm_host(a, b, c, 1.0, 0.0, o, bias)
    mf.sync()
    want = torch.relu(_ref(a, b, torch.zeros(m, n), 1.0, 0.0) + bias.double())
    _check(c, want)
    assert torch.isnan(c_buf[:, n:]).all()  # padding columns never written


def test_alternating_shapes_and_streams():
    """Buffers grow, the panel plan is replaced, and calls on two streams stay ordered."""
    gen = torch.Generator().manual_seed(10)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    cases = [(3000, 2048, 512, s1), (9000, 1024, 256, s2), (3000, 2048, 512, s2), (64, 64, 64, s1)]
    outs = []
    for m, n, k, s in cases:
        a, b, c0 = _rand((m, k), gen), _rand((k, n), gen), _rand((m, n), gen)
        c = c0.clone().pin_memory()
        with torch.cuda.stream(s):
            mf.sgemm_host(a, b, c, 1.0, 1.0)
        outs.append((a, b, c0, c, s))
    for a, b, c0, c, s in outs:
        s.synchronize()
        _check(c, _ref(a, b, c0, 1.0, 1.0))
    assert mf.device_status() == 0


def test_k_zero_and_alpha_zero_scale_host_c():
    gen = torch.Generator().manual_seed(11)
    c0 = _rand((300, 200), gen)
    c = c0.clone().pin_memory()
    mf.sgemm_host(torch.empty((300, 0)), torch.empty((0, 200)), c, 1.0, 2.0)
    mf.sync()
    assert torch.equal(c, c0 * 2.0)
    a, b = _rand((300, 50), gen), _rand((50, 200), gen)
    mf.sgemm_host(a, b, c, 0.0, 0.5)
    mf.sync()
    assert torch.equal(c, c0)


def test_validation():
    with pytest.raises(mf.ShapeMismatchError):
        mf.sgemm_host(torch.zeros(4, 5), torch.zeros(6, 4), torch.zeros(4, 4))
    with pytest.raises(mf.InvalidArgumentError):
        mf.sgemm_host(torch.zeros(4, 4, dtype=torch.float64), torch.zeros(4, 4), torch.zeros(4, 4))
