"""Oracle — TEST INFRASTRUCTURE ONLY.

CPU checkers for the dense FP32 contraction path:

* ``libmfb_oracle.so`` — a C restatement (``oracle/mfb_oracle.c``) of the
  reference's ``gemm_f32`` arithmetic (src/hw/gemm_avx2.cpp:75-451), of
  ``gemm_reference`` (src/hw/gemm_scalar.cpp:12-33), of ``conv2d_kernel``
  (src/nn/conv.cu:22-49), of the three conv2d backward kernels
  (src/nn/backward/convolution_kernels.cuh:9-95) and of the column-bias epilogue
  (src/ops/gemm/gemm_fused.cu:23-40), plus FP64 references.
* ``_ref/libmfref_cpu.so`` — the reference's own ``gemm_f32`` compiled from its
  sources by ``oracle/Makefile`` (present wherever that build ran).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this package, and only as the checker or the timed CPU
baseline. The product (``matrixflash_pro_b200``) never imports it.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
RESTATEMENT_SO = os.path.join(_HERE, "libmfb_oracle.so")
REFERENCE_SO = os.path.join(_HERE, "_ref", "libmfref_cpu.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i32p = ctypes.POINTER(ctypes.c_int)

_rest = None
_ref = None


def build(reference_root: str = "/root/reference") -> None:
    """Compile the restatement and, where the reference tree exists, the reference CPU GEMM."""
    args = ["make", "-s", "-C", _HERE]
    if os.path.isdir(reference_root):
        args.append(f"REF_ROOT={reference_root}")
    subprocess.run(args, check=True)


def _restatement():
    global _rest
    if _rest is None:
        if not os.path.exists(RESTATEMENT_SO):
            build()
        lib = ctypes.CDLL(RESTATEMENT_SO)
        gemm_sig = [ctypes.c_int] * 3 + [_f32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p, ctypes.c_int,
                                         ctypes.c_float, ctypes.c_float]
        for name in ("oracle_gemm_f32", "oracle_gemm_reference_f32"):
            getattr(lib, name).argtypes = gemm_sig
            getattr(lib, name).restype = None
        lib.oracle_gemm_f32_rows.argtypes = [ctypes.c_int] * 4 + [_f32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p,
                                                                  ctypes.c_int, ctypes.c_float, ctypes.c_float]
        lib.oracle_gemm_f32_sampled.argtypes = [ctypes.c_int, _i32p, ctypes.c_int, _i32p, ctypes.c_int,
                                                ctypes.c_int, _f32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p,
                                                ctypes.c_float, ctypes.c_float, _f32p]
        lib.oracle_gemm_f64.argtypes = [ctypes.c_int] * 3 + [_f32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p,
                                                             ctypes.c_int, ctypes.c_double, ctypes.c_double,
                                                             _f64p, ctypes.c_int]
        conv_sig = [ctypes.c_int] * 9 + [_f32p, _f32p, _f32p]
        lib.oracle_conv2d_f32.argtypes = conv_sig + [_f32p]
        lib.oracle_conv2d_f64.argtypes = conv_sig + [_f64p]
        lib.oracle_epilogue_f32.argtypes = [_f32p, ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        bwd_sig = [ctypes.c_int] * 9 + [_f32p, _f32p]
        for suffix, outp in (("f32", _f32p), ("f64", _f64p)):
            getattr(lib, f"oracle_conv2d_input_backward_{suffix}").argtypes = bwd_sig + [outp]
            getattr(lib, f"oracle_conv2d_weight_backward_{suffix}").argtypes = bwd_sig + [outp]
            getattr(lib, f"oracle_conv2d_bias_backward_{suffix}").argtypes = [ctypes.c_int] * 4 + [_f32p, outp]
        _rest = lib
    return _rest


def reference_available() -> bool:
    return os.path.exists(REFERENCE_SO)


def _reference():
    global _ref
    if _ref is None:
        if not reference_available():
            raise FileNotFoundError(f"{REFERENCE_SO} is not built (run make -C oracle where the reference exists)")
        lib = ctypes.CDLL(REFERENCE_SO)
        sig = [ctypes.c_int] * 3 + [_f32p, ctypes.c_int, _f32p, ctypes.c_int, _f32p, ctypes.c_int,
                                    ctypes.c_float, ctypes.c_float]
        lib.mfref_gemm_f32.argtypes = sig
        lib.mfref_gemm_f32.restype = ctypes.c_int
        lib.mfref_gemm_reference.argtypes = sig
        lib.mfref_gemm_reference.restype = ctypes.c_int
        lib.mfref_gemm_kernel_name.restype = ctypes.c_char_p
        lib.mfref_worker_count.restype = ctypes.c_int
        _ref = lib
    return _ref


def _p32(x: np.ndarray):
    assert x.dtype == np.float32
    return x.ctypes.data_as(_f32p)


def _p64(x: np.ndarray):
    assert x.dtype == np.float64
    return x.ctypes.data_as(_f64p)


def _check_buffer(buf: np.ndarray, rows: int, cols: int, ld: int, name: str) -> None:
    if rows > 0 and cols > 0:
        need = (rows - 1) * ld + cols
        if buf.size < need or ld < cols:
            raise ValueError(f"{name}: buffer of {buf.size} floats too small for {rows}x{cols} ld={ld}")


# ---------------------------------------------------------------------------------------------
# GEMM checkers. Buffers are flat (or 2-D) float32 arrays with explicit leading dimensions,
# exactly like the reference's pointer interface.
# ---------------------------------------------------------------------------------------------
def gemm_f32(m, n, k, a, lda, b, ldb, c, ldc, alpha=1.0, beta=0.0, impl="restatement"):
    """C = alpha*A*B + beta*C in place, with the reference's gemm_f32 arithmetic.

    ``impl='restatement'`` runs oracle/mfb_oracle.c; ``impl='reference'`` runs the
    reference's own compiled gemm_f32 (multi-threaded, src/hw/gemm.cpp:73).
    """
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    assert c.dtype == np.float32 and c.flags["C_CONTIGUOUS"]
    _check_buffer(a, m, k, lda, "A")
    _check_buffer(b, k, n, ldb, "B")
    _check_buffer(c.reshape(-1), m, n, ldc, "C")
    if impl == "reference":
        rc = _reference().mfref_gemm_f32(m, n, k, _p32(a), lda, _p32(b), ldb, _p32(c), ldc, alpha, beta)
        if rc != 0:
            raise RuntimeError("reference gemm_f32 raised")
    elif impl == "restatement":
        _restatement().oracle_gemm_f32(m, n, k, _p32(a), lda, _p32(b), ldb, _p32(c), ldc, alpha, beta)
    elif impl == "scalar":
        _restatement().oracle_gemm_reference_f32(m, n, k, _p32(a), lda, _p32(b), ldb, _p32(c), ldc, alpha, beta)
    elif impl == "reference_scalar":
        _reference().mfref_gemm_reference(m, n, k, _p32(a), lda, _p32(b), ldb, _p32(c), ldc, alpha, beta)
    else:
        raise ValueError(impl)
    return c


def gemm_f32_sampled(rows, cols, n, k, a, lda, b, ldb, c_in=None, alpha=1.0, beta=0.0):
    """Elements (rows[r], cols[s]) of the full gemm_f32 result, as a (len(rows), len(cols)) array."""
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    cols = np.ascontiguousarray(cols, dtype=np.int32)
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    out = np.zeros((rows.size, cols.size), dtype=np.float32)
    cin = None
    if c_in is not None:
        cin = np.ascontiguousarray(c_in, dtype=np.float32).reshape(rows.size, cols.size)
    _restatement().oracle_gemm_f32_sampled(rows.size, rows.ctypes.data_as(_i32p), cols.size,
                                           cols.ctypes.data_as(_i32p), n, k, _p32(a), lda, _p32(b), ldb,
                                           _p32(cin) if cin is not None else None, alpha, beta, _p32(out))
    return out


def gemm_f64(m, n, k, a, lda, b, ldb, c_in=None, ldc=None, alpha=1.0, beta=0.0):
    """FP64 reference of alpha*A*B + beta*C as an (m, n) float64 array."""
    a = np.ascontiguousarray(a, dtype=np.float32).reshape(-1)
    b = np.ascontiguousarray(b, dtype=np.float32).reshape(-1)
    out = np.zeros((m, n), dtype=np.float64)
    if c_in is not None:
        c_in = np.ascontiguousarray(c_in, dtype=np.float32).reshape(-1)
    _restatement().oracle_gemm_f64(m, n, k, _p32(a), lda, _p32(b), ldb,
                                   _p32(c_in) if c_in is not None else None, ldc or n, alpha,
                                   beta if c_in is not None else 0.0, _p64(out), n)
    return out


def conv2d_f32(x, w, bias, stride=1, padding=0):
    """NCHW conv2d forward with the arithmetic of the reference's conv2d_kernel."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    n, c, h, wd = x.shape
    k, c2, r, s = w.shape
    assert c == c2 and bias.shape == (k,)
    p = (h + 2 * padding - r) // stride + 1
    q = (wd + 2 * padding - s) // stride + 1
    y = np.zeros((n, k, p, q), dtype=np.float32)
    _restatement().oracle_conv2d_f32(n, c, h, wd, k, r, s, stride, padding, _p32(x), _p32(w), _p32(bias), _p32(y))
    return y


def conv2d_f64(x, w, bias, stride=1, padding=0):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    p = (h + 2 * padding - r) // stride + 1
    q = (wd + 2 * padding - s) // stride + 1
    y = np.zeros((n, k, p, q), dtype=np.float64)
    _restatement().oracle_conv2d_f64(n, c, h, wd, k, r, s, stride, padding, _p32(x), _p32(w), _p32(bias), _p64(y))
    return y


def _bwd_shapes(grad, x_shape, w_shape, stride, padding):
    n, c, h, wd = x_shape
    k, c2, r, s = w_shape
    p = (h + 2 * padding - r) // stride + 1
    q = (wd + 2 * padding - s) // stride + 1
    assert c == c2 and tuple(grad.shape) == (n, k, p, q), "conv2d backward shape mismatch"
    return n, c, h, wd, k, r, s


def conv2d_input_backward(grad, w, x_shape, stride=1, padding=0, f64=False):
    """dL/dinput with the arithmetic of conv2d_input_backward_kernel (convolution_kernels.cuh:9-47)."""
    grad = np.ascontiguousarray(grad, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, c, h, wd, k, r, s = _bwd_shapes(grad, x_shape, w.shape, stride, padding)
    out = np.zeros((n, c, h, wd), dtype=np.float64 if f64 else np.float32)
    fn = _restatement().oracle_conv2d_input_backward_f64 if f64 else _restatement().oracle_conv2d_input_backward_f32
    fn(n, c, h, wd, k, r, s, stride, padding, _p32(grad), _p32(w), _p64(out) if f64 else _p32(out))
    return out


def conv2d_weight_backward(grad, x, w_shape, stride=1, padding=0, f64=False):
    """dL/dweights with the arithmetic of conv2d_weight_backward_kernel (convolution_kernels.cuh:50-82)."""
    grad = np.ascontiguousarray(grad, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, c, h, wd, k, r, s = _bwd_shapes(grad, x.shape, w_shape, stride, padding)
    out = np.zeros((k, c, r, s), dtype=np.float64 if f64 else np.float32)
    fn = _restatement().oracle_conv2d_weight_backward_f64 if f64 else _restatement().oracle_conv2d_weight_backward_f32
    fn(n, c, h, wd, k, r, s, stride, padding, _p32(grad), _p32(x), _p64(out) if f64 else _p32(out))
    return out


def conv2d_bias_backward(grad, f64=False):
    """dL/dbias with the arithmetic of conv2d_bias_backward_kernel (convolution_kernels.cuh:85-95)."""
    grad = np.ascontiguousarray(grad, dtype=np.float32)
    n, k, p, q = grad.shape
    out = np.zeros(k, dtype=np.float64 if f64 else np.float32)
    fn = _restatement().oracle_conv2d_bias_backward_f64 if f64 else _restatement().oracle_conv2d_bias_backward_f32
    fn(n, k, p, q, _p32(grad), _p64(out) if f64 else _p32(out))
    return out


def col_mean_f32(x):
    """Column means as the reference forms them: col_sum_kernel's four interleaved FP32
    accumulators over rows 4i, 4i+1, 4i+2, 4i+3, the remainder into the first, combined as
    (s0 + s1) + (s2 + s3) (src/ops/reductions/axis_kernels.cuh:25-45), then multiplied by
    the float 1/rows (src/ops/reductions/covariance.inc:28)."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    s = np.zeros((4, cols), np.float32)
    full = rows // 4 * 4
    for r in range(0, full, 4):
        s += x[r:r + 4]
    for r in range(full, rows):
        s[0] += x[r]
    total = (s[0] + s[1]) + (s[2] + s[3])
    return total * np.float32(1.0 / np.float32(rows))


def covariance_f32(x, impl="restatement"):
    """matrix_pro::covariance (src/ops/reductions/covariance.inc:23-47) on the CPU: center the
    columns (center_columns_kernel, moment_kernels.cuh:5-10), then
    (1/max(rows-1, 1)) * X_c^T X_c with gemm_f32 standing in for the reference's cublasSgemm."""
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    xc = x - col_mean_f32(x)[None, :]
    xt = np.ascontiguousarray(xc.T)
    out = np.zeros(cols * cols, np.float32)
    alpha = float(np.float32(1.0) / np.float32(rows - 1 if rows > 1 else 1))
    gemm_f32(cols, cols, rows, xt, rows, xc, cols, out, cols, alpha, 0.0, impl=impl)
    return out.reshape(cols, cols)


def correlation_f32(cov):
    """covariance_to_correlation_kernel (src/ops/reductions/moment_kernels.cuh:51-67)."""
    cov = np.asarray(cov, np.float32)
    d = np.diag(cov).astype(np.float32)
    denom = np.sqrt((d[:, None] * d[None, :]).astype(np.float32)).astype(np.float32)
    ok = (d[:, None] > 0) & (d[None, :] > 0)
    corr = np.where(ok, cov / np.where(ok, denom, np.float32(1.0)), np.float32(0.0)).astype(np.float32)
    np.fill_diagonal(corr, 1.0)
    return corr


def epilogue_f32(c, ldc, bias, m, n, mode):
    """In-place column-bias epilogue (mode 0 bias, 1 bias+ReLU, 2 bias+tanh-GELU)."""
    bias = np.ascontiguousarray(bias, dtype=np.float32)
    _restatement().oracle_epilogue_f32(_p32(c), ldc, _p32(bias), m, n, mode)
    return c


def reference_info() -> dict:
    """Kernel name and pool size of the reference's CPU GEMM on this host."""
    lib = _reference()
    return {"gemm_kernel_name": lib.mfref_gemm_kernel_name().decode(), "worker_count": lib.mfref_worker_count(),
            "nproc": os.cpu_count()}


# ---------------------------------------------------------------------------------------------
# Seeded inputs and error metrics.
# ---------------------------------------------------------------------------------------------
def seeded(shape, dist="uniform", seed=20261001, scale=1.0):
    """Deterministic float32 inputs: 'uniform' is U[-scale, scale], 'normal' is N(0, scale)."""
    rng = np.random.default_rng(seed)
    if dist == "uniform":
        return rng.uniform(-scale, scale, size=shape).astype(np.float32)
    if dist == "normal":
        return (rng.standard_normal(size=shape) * scale).astype(np.float32)
    raise ValueError(dist)


def sha256(*arrays) -> str:
    h = hashlib.sha256()
    for arr in arrays:
        h.update(np.ascontiguousarray(arr).tobytes())
    return h.hexdigest()


def normwise_rel(x, ref) -> float:
    """||x - ref||_F / ||ref||_F in double."""
    x = np.asarray(x, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    return float(num / den) if den > 0 else float(num)


def max_abs(x, ref) -> float:
    return float(np.max(np.abs(np.asarray(x, dtype=np.float64) - np.asarray(ref, dtype=np.float64)))) \
        if np.size(x) else 0.0


def elementwise_bound(k: int, max_a: float, max_b: float) -> float:
    """The strict-FP32 elementwise bound 1e-5 * k * max|A| * max|B|."""
    return 1e-5 * max(k, 1) * max_a * max_b
