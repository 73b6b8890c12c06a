"""GPU tier, collected last: the allocation-free GEMM entry point, mfb_sgemm_noalloc.

Some callers cannot allocate device memory when they call a GEMM: code under a framework
that owns the device-memory budget, latency-critical paths where cudaMalloc/cudaFree
(which synchronize the device) or an out-of-memory failure mid-call are not acceptable,
and plugins that may not touch their host process's allocator. mfb_sgemm_noalloc keeps
its operand scratch in a static 64 MiB device array instead of allocating it.

Every result here is gated against the oracle (the reference's gemm_f32 and an FP64
product) with the tolerances of the other GPU tests, and also compared with mfb_sgemm (the
allocating entry point) on the same inputs. Calls run back to back, so each one runs over
what the previous call left in the shared array."""
import ctypes

import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from matrixflash_pro_b200 import _lib
from helpers import assert_strict, assert_tf32

pytestmark = pytest.mark.gpu

NOALLOC_LIMIT_BYTES = 64 << 20  # MFB_NOALLOC_SCRATCH_BYTES in include/mfb.h
IMPL = "reference" if oracle.reference_available() else "restatement"


def _plane_bytes(rows, cols):
    """One TF32 plane of a stored rows x cols operand: rows padded to 4 floats, 256-byte granules."""
    cols4 = -(-cols // 4) * 4
    return -(-(rows * cols4) // 64) * 64 * 4


def _scratch_bytes(m, n, k, strict=True, ta=False, tb=False):
    planes = 2 if strict else 1
    a_rows, a_cols = (k, m) if ta else (m, k)
    b_rows, b_cols = (n, k) if tb else (k, n)
    return planes * (_plane_bytes(a_rows, a_cols) + _plane_bytes(b_rows, b_cols))


def _call(fn_name, desc, A, B, C, bias=None, stream=None):
    s = stream.cuda_stream if stream is not None else torch.cuda.current_stream().cuda_stream
    fn = getattr(_lib.lib(), fn_name)
    _lib.check(fn(0, s, ctypes.byref(desc), A.data_ptr(), B.data_ptr(), C.data_ptr(),
                  bias.data_ptr() if bias is not None else 0), fn_name)


def _both(desc, A, B, C0, bias=None):
    """(noalloc result, mfb_sgemm result) on copies of C0, as host arrays."""
    got, ref = C0.clone(), C0.clone()
    _call("mfb_sgemm_noalloc", desc, A, B, got, bias)
    _call("mfb_sgemm", desc, A, B, ref, bias)
    mf.sync()
    return got.cpu().numpy(), ref.cpu().numpy()


def _oracle(m, n, k, a, b, c0, alpha, beta, bias=None, epilogue=0):
    """gemm_f32 (+ the column-bias epilogue) and the FP64 product (+ the epilogue in FP64) of the
    untransposed row-major operands a (m x k), b (k x n), c0 (m x n)."""
    ref32 = c0.copy()
    oracle.gemm_f32(m, n, k, a, k, b, n, ref32, n, alpha, beta, impl=IMPL)
    ref64 = alpha * (a.astype(np.float64) @ b.astype(np.float64)) + beta * c0.astype(np.float64)
    if epilogue:
        # the oracle numbers the epilogues from bias alone: 0 bias, 1 bias+ReLU, 2 bias+GELU
        oracle.epilogue_f32(ref32, n, bias, m, n, epilogue - 1)
        ref64 = ref64 + bias.astype(np.float64)
        if epilogue == 2:
            ref64 = np.maximum(ref64, 0.0)
        elif epilogue == 3:
            ref64 = 0.5 * ref64 * (1.0 + np.tanh(0.7978845608 * (ref64 + 0.044715 * ref64 ** 3)))
    return ref32, ref64


def _gate(got, ref32, ref64, k, a, b, strict, what):
    if strict:
        return assert_strict(got, ref32, ref64, k, float(np.abs(a).max()), float(np.abs(b).max()), what)
    return assert_tf32(got, ref32, what)


def test_noalloc_two_calls_in_a_row_against_oracle():
    torch.cuda.set_device(0)
    # Call 1: 1000 x 1100 x 900 with padded strides and beta, strict FP32. Call 2, right
    # after: another shape in TF32 over what call 1 left in the array.
    cases = [(1000, 1100, 900, 912, 1104, 1108, 0.5, 1.0, True),
             (700, 333, 1500, 1500, 336, 333, 1.0, 0.0, False)]
    for m, n, k, lda, ldb, ldc, alpha, beta, strict in cases:
        rng = np.random.default_rng(m + n + k)
        a = rng.uniform(-1, 1, (m, lda)).astype(np.float32)
        b = rng.standard_normal((k, ldb)).astype(np.float32)
        c0 = rng.standard_normal((m, ldc)).astype(np.float32)
        prec = mf.GemmPrecision.fp32 if strict else mf.GemmPrecision.tf32
        desc = mf.make_desc(m, n, k, lda, ldb, ldc, alpha, beta, int(prec))
        got, twin = _both(desc, torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(c0).cuda())
        assert np.array_equal(got[:, n:], c0[:, n:]), "row padding of C was written"
        ref32, ref64 = _oracle(m, n, k, np.ascontiguousarray(a[:, :k]), np.ascontiguousarray(b[:, :n]),
                               np.ascontiguousarray(c0[:, :n]), alpha, beta)
        _gate(got[:, :n], ref32, ref64, k, a[:, :k], b[:, :n], strict, f"noalloc {m}x{n}x{k}")
        assert oracle.normwise_rel(got[:, :n], twin[:, :n]) <= (1e-6 if strict else 5e-3)
    assert mf.device_status(0) == 0


def test_noalloc_at_its_limit_2048_cubed_strict():
    """2048^3 strict: the hi and lo planes of A and B take exactly the 64 MiB the array holds."""
    m = n = k = 2048
    assert _scratch_bytes(m, n, k) == NOALLOC_LIMIT_BYTES
    rng = np.random.default_rng(2048)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c0 = np.zeros((m, n), np.float32)
    desc = mf.make_desc(m, n, k, k, n, n, 1.0, 0.0, int(mf.GemmPrecision.fp32))
    got, twin = _both(desc, torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(c0).cuda())
    ref32, ref64 = _oracle(m, n, k, a, b, c0, 1.0, 0.0)
    e = _gate(got, ref32, ref64, k, a, b, True, "noalloc 2048^3")
    assert e["gpu_vs_fp64"] < 1e-6
    assert oracle.normwise_rel(got, twin) <= 1e-6


def test_noalloc_rejects_problems_beyond_its_scratch():
    A = torch.empty(1, device="cuda")
    # The next larger problem than the limit case (one more row of A: 16 KiB more of planes),
    # and one far beyond it. Nothing is launched for either.
    for m, n, k in [(2049, 2048, 2048), (4096, 4096, 4096)]:
        need = _scratch_bytes(m, n, k)
        assert need > NOALLOC_LIMIT_BYTES
        desc = mf.make_desc(m, n, k, k, n, n)
        st = _lib.lib().mfb_sgemm_noalloc(0, None, ctypes.byref(desc), A.data_ptr(), A.data_ptr() + 16,
                                          A.data_ptr() + 32, 0)
        assert st == _lib.MFB_EINVAL
        msg = _lib.last_error()
        assert str(NOALLOC_LIMIT_BYTES) in msg and str(need) in msg, msg
    # TF32 needs one plane per operand, so the same 2049-row problem fits.
    assert _scratch_bytes(2049, 2048, 2048, strict=False) <= NOALLOC_LIMIT_BYTES


@pytest.mark.parametrize("strict", [True, False])
def test_noalloc_transposed_operands_with_bias_gelu(strict):
    m, n, k = 300, 260, 513
    rng = np.random.default_rng(7)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    prec = mf.GemmPrecision.fp32 if strict else mf.GemmPrecision.tf32
    desc = mf.make_desc(m, n, k, m, k, n, 0.75, -0.5, int(prec), trans_a=1, trans_b=1, epilogue=3)
    A = torch.from_numpy(a.T.copy()).cuda()  # stored k x m
    B = torch.from_numpy(b.T.copy()).cuda()  # stored n x k
    got, twin = _both(desc, A, B, torch.from_numpy(c0).cuda(), torch.from_numpy(bias).cuda())
    ref32, ref64 = _oracle(m, n, k, a, b, c0, 0.75, -0.5, bias, 3)
    _gate(got, ref32, ref64, k, a, b, strict, "noalloc trans_a trans_b bias+gelu")
    assert oracle.normwise_rel(got, twin) <= (1e-6 if strict else 5e-3)


@pytest.mark.parametrize("m,n,k", [(3000, 8, 1500), (1, 700, 2000)])
def test_noalloc_vectors_run_tcgen05_and_match_the_gemv_path(m, n, k):
    """mfb_sgemm sends n <= 16 and m == 1 to the GEMV kernels; the allocation-free entry
    point runs them on the tcgen05 GEMM. Both must agree with the oracle."""
    rng = np.random.default_rng(m * n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    c0 = rng.standard_normal((m, n)).astype(np.float32)
    desc = mf.make_desc(m, n, k, k, n, n, 0.5, 1.0, int(mf.GemmPrecision.fp32))
    got, twin = _both(desc, torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda(), torch.from_numpy(c0).cuda())
    ref32, ref64 = _oracle(m, n, k, a, b, c0, 0.5, 1.0)
    _gate(got, ref32, ref64, k, a, b, True, f"noalloc vector {m}x{n}x{k}")
    _gate(twin, ref32, ref64, k, a, b, True, f"mfb_sgemm vector {m}x{n}x{k}")


def test_noalloc_allocates_no_device_memory():
    """On a stream the library has never seen, mfb_sgemm takes scratch for that stream (free
    device memory drops); mfb_sgemm_noalloc takes none (free memory stays the same)."""
    m, n, k = 1536, 1024, 1024
    g = torch.Generator(device="cuda").manual_seed(11)
    A = torch.rand((m, k), device="cuda", generator=g)
    B = torch.rand((k, n), device="cuda", generator=g)
    C = torch.zeros((m, n), device="cuda")
    desc = mf.make_desc(m, n, k, k, n, n, 1.0, 0.0, int(mf.GemmPrecision.fp32))
    _call("mfb_sgemm_noalloc", desc, A, B, C)  # kernels loaded, address looked up
    mf.sync()
    unchanged = False
    for _ in range(3):  # a change made by anything else on the device shows up only once
        fresh = torch.cuda.Stream()
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        _call("mfb_sgemm_noalloc", desc, A, B, C, stream=fresh)
        fresh.synchronize()
        if torch.cuda.mem_get_info()[0] == free0:
            unchanged = True
            break
    assert unchanged, "mfb_sgemm_noalloc changed the device's free memory"
    want = torch.zeros_like(C)
    fresh = torch.cuda.Stream()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    _call("mfb_sgemm", desc, A, B, want, stream=fresh)
    fresh.synchronize()
    assert torch.cuda.mem_get_info()[0] < free0, "control: mfb_sgemm should take scratch for a new stream"
    assert torch.equal(C, want)
    assert mf.device_status(0) == 0
