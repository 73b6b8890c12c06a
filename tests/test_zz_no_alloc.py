"""GPU tier, collected last: the allocation-free GEMM entry point, mfb_sgemm_noalloc.

Some callers cannot allocate device memory when they call a GEMM: code under a framework
that owns the device-memory budget, latency-critical paths where cudaMalloc/cudaFree
(which synchronize the device) or an out-of-memory failure mid-call are not acceptable,
and plugins that may not touch their host process's allocator. mfb_sgemm_noalloc keeps
its operand scratch in a static 64 MiB device array instead of allocating it.

The test calls it through the C ABI twice in a row, with different shapes, data and
precisions, so the second call runs over what the first left in the shared array, and
checks each result against mfb_sgemm (the allocating entry point) on the same inputs,
within the strict-FP32 tolerance used by the other GPU tests."""
import ctypes

import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
import oracle
from matrixflash_pro_b200 import _lib

pytestmark = pytest.mark.gpu

NOALLOC_LIMIT_BYTES = 64 << 20  # MFB_NOALLOC_SCRATCH_BYTES in include/mfb.h


def _run(fn_name, desc, A, B, C0):
    C = C0.clone()
    stream = torch.cuda.current_stream().cuda_stream
    fn = getattr(_lib.lib(), fn_name)
    _lib.check(fn(0, stream, ctypes.byref(desc), A.data_ptr(), B.data_ptr(), C.data_ptr(), 0), fn_name)
    mf.sync()
    return C


@pytest.mark.parametrize("call", [0, 1])
def test_noalloc_matches_allocating_entry_point_two_calls(call):
    torch.cuda.set_device(0)
    # Call 0: 1000 x 1100 x 900, padded strides, beta 1, strict. Call 1: a different shape
    # and precision right after, over the array's leftovers.
    shapes = [(1000, 1100, 900, 912, 1104, 1108, 0.5, 1.0, mf.GemmPrecision.fp32),
              (700, 333, 1500, 1500, 336, 333, 1.0, 0.0, mf.GemmPrecision.tf32)]
    for m, n, k, lda, ldb, ldc, alpha, beta, prec in shapes[: call + 1]:
        rng = np.random.default_rng(m + n + k)
        A = torch.from_numpy(rng.uniform(-1, 1, (m, lda)).astype(np.float32)).cuda()
        B = torch.from_numpy(rng.standard_normal((k, ldb)).astype(np.float32)).cuda()
        C0 = torch.from_numpy(rng.standard_normal((m, ldc)).astype(np.float32)).cuda()
        desc = mf.make_desc(m, n, k, lda, ldb, ldc, alpha, beta, int(prec))
        got = _run("mfb_sgemm_noalloc", desc, A, B, C0).cpu().numpy()
        ref = _run("mfb_sgemm", desc, A, B, C0).cpu().numpy()
        assert np.array_equal(got[:, n:], C0.cpu().numpy()[:, n:]), "row padding of C was written"
        tol = 1e-6 if prec == mf.GemmPrecision.fp32 else 5e-3
        assert oracle.normwise_rel(got[:, :n], ref[:, :n]) <= tol
    assert mf.device_status(0) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    m = n = k = 4096  # strict planes of A and B: 256 MiB > 64 MiB
    desc = mf.make_desc(m, n, k, k, n, n)
    A = torch.empty(1, device="cuda")
    st = _lib.lib().mfb_sgemm_noalloc(0, None, ctypes.byref(desc), A.data_ptr(), A.data_ptr() + 16,
                                      A.data_ptr() + 32, 0)
    assert st == _lib.MFB_EINVAL
    msg = _lib.last_error()
    assert str(NOALLOC_LIMIT_BYTES) in msg and "268435456" in msg
