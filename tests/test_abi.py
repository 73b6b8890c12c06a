"""CPU tier: the drop-in boundary. libmfb.so loads, exports exactly what include/mfb.h
declares, and rejects bad arguments through the C ABI before touching a device (the
reference's validation rules, src/ops/gemm/plan/implementation.inc:88-110)."""
import ctypes
import os
import re
import subprocess

import pytest

import matrixflash_pro_b200 as mf
from matrixflash_pro_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "mfb.h")).read()
    return sorted(set(re.findall(r"MFB_API\s+[\w\s\*]+?\b(mfb_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert sorted(_lib.EXPORTED_SYMBOLS) == declared_symbols()


def test_library_exports_every_declared_symbol():
    lib = mf.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", mf.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\b(mfb_\w+)$", out.stdout, re.M))
    assert set(declared_symbols()) <= exported
    # Nothing else leaks from the C ABI namespace.
    assert exported <= set(declared_symbols())


def test_version_and_status_strings():
    lib = mf.lib()
    assert b"sm_100a" in lib.mfb_version()
    for code in range(8):
        assert lib.mfb_status_string(code).startswith(b"MFB_")


def _desc(**kw):
    base = dict(m=4, n=4, k=4, lda=4, ldb=4, ldc=4)
    base.update(kw)
    return mf.make_desc(base["m"], base["n"], base["k"], base["lda"], base["ldb"], base["ldc"],
                        precision=kw.get("precision", 0), trans_a=kw.get("trans_a", 0),
                        trans_b=kw.get("trans_b", 0), epilogue=kw.get("epilogue", 0))


@pytest.mark.parametrize("kw,expected,needle", [
    (dict(lda=3), _lib.MFB_EINVAL, "lda"),
    (dict(ldb=3), _lib.MFB_EINVAL, "ldb"),
    (dict(ldc=2), _lib.MFB_EINVAL, "ldc"),
    (dict(m=-1), _lib.MFB_EINVAL, "non-negative"),
    (dict(precision=7), _lib.MFB_EINVAL, "precision"),
    (dict(epilogue=9), _lib.MFB_EINVAL, "epilogue"),
    (dict(trans_a=1, lda=3), _lib.MFB_EINVAL, "lda"),
    (dict(trans_b=1, ldb=3), _lib.MFB_EINVAL, "ldb"),
])
def test_sgemm_rejects_bad_descriptors(kw, expected, needle):
    lib = mf.lib()
    d = _desc(**kw)
    for entry in (lib.mfb_sgemm, lib.mfb_sgemm_host):  # checked before any CUDA call
        st = entry(0, None, ctypes.byref(d), 16, 32, 48, 0)
        assert st == expected
        assert needle in _lib.last_error()


def test_sgemm_rejects_alias_and_missing_bias():
    lib = mf.lib()
    d = _desc()
    assert lib.mfb_sgemm(0, None, ctypes.byref(d), 16, 32, 16, 0) == _lib.MFB_EINVAL
    assert "alias" in _lib.last_error()
    d = _desc(epilogue=2)
    assert lib.mfb_sgemm(0, None, ctypes.byref(d), 16, 32, 48, 0) == _lib.MFB_ESHAPE
    assert "bias" in _lib.last_error()
    assert lib.mfb_sgemm(0, None, ctypes.byref(d), 16, 32, 48, 48) == _lib.MFB_EINVAL


def test_check_maps_status_to_reference_exceptions():
    with pytest.raises(mf.InvalidArgumentError):
        _lib.check(_lib.MFB_EINVAL)
    with pytest.raises(mf.ShapeMismatchError):
        _lib.check(_lib.MFB_ESHAPE)
    with pytest.raises(mf.DeviceTimeoutError):
        _lib.check(_lib.MFB_ETIMEOUT)
    with pytest.raises(mf.CudaError):
        _lib.check(_lib.MFB_ECUDA)
    assert issubclass(mf.DeviceTimeoutError, mf.CudaError) and issubclass(mf.CudaError, mf.MatrixProError)


def test_gemv_and_conv_validation():
    lib = mf.lib()
    d = _desc(n=32, m=8)
    assert lib.mfb_gemv(0, None, ctypes.byref(d), 16, 32, 48, 0) == _lib.MFB_EINVAL
    d = _desc(trans_a=1)
    assert lib.mfb_gemv(0, None, ctypes.byref(d), 16, 32, 48, 0) == _lib.MFB_EINVAL
    # stride 0 and an oversized kernel are the reference's ShapeMismatchError cases.
    assert lib.mfb_conv2d_fwd(0, None, 1, 1, 4, 4, 1, 3, 3, 0, 0, 16, 32, 48, 64, 0) == _lib.MFB_ESHAPE
    assert lib.mfb_conv2d_fwd(0, None, 1, 1, 2, 2, 1, 5, 5, 1, 0, 16, 32, 48, 64, 0) == _lib.MFB_ESHAPE
    assert lib.mfb_conv2d_fwd(0, None, 1, 1, 4, 4, 1, 3, 3, 1, 0, 16, 32, 48, 64, 3) == _lib.MFB_EINVAL


def test_wait_limit_round_trip():
    lib = mf.lib()
    old = lib.mfb_get_wait_limit_ns()
    assert lib.mfb_set_wait_limit_ns(10) == _lib.MFB_EINVAL
    assert lib.mfb_set_wait_limit_ns(123456789) == _lib.MFB_OK
    assert lib.mfb_get_wait_limit_ns() == 123456789
    assert lib.mfb_set_wait_limit_ns(old) == _lib.MFB_OK


def test_plan_create_rejects_bad_options_without_a_device():
    lib = mf.lib()
    h = ctypes.c_void_p()
    d = _desc(precision=5)
    assert lib.mfb_plan_create(0, ctypes.byref(d), ctypes.byref(h)) == _lib.MFB_EINVAL
    assert not h.value
    assert lib.mfb_plan_execute(None, None, 0, 0, 0, 1.0, 0.0, 0) == _lib.MFB_EINVAL
    assert lib.mfb_plan_destroy(None) == _lib.MFB_OK


def test_checked_dim_matches_reference_limit():
    with pytest.raises(mf.InvalidArgumentError):
        mf.checked_dim(2 ** 31)
    assert mf.checked_dim(2 ** 31 - 1) == 2 ** 31 - 1


def test_conv_python_validation_on_cpu_tensors():
    import torch
    x = torch.zeros(1, 2, 4, 4)
    with pytest.raises(mf.ShapeMismatchError):
        mf.conv2d(torch.zeros(2, 4, 4), torch.zeros(1, 2, 3, 3), torch.zeros(1))
    with pytest.raises(mf.InvalidArgumentError):
        mf.conv2d(x, torch.zeros(1, 2, 3), torch.zeros(1))
    with pytest.raises(mf.ShapeMismatchError):
        mf.conv2d(x, torch.zeros(1, 3, 3, 3), torch.zeros(1))
    with pytest.raises(mf.ShapeMismatchError):
        mf.conv2d(x, torch.zeros(1, 2, 7, 7), torch.zeros(1))
    with pytest.raises(mf.InvalidArgumentError):
        mf.conv2d(x, torch.zeros(1, 2, 3, 3), torch.zeros(1))  # CPU tensors: no fallback
