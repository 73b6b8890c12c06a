"""Matrix-level GEMM API over libmfb.so, mirroring the reference's interface.

Reference interface (include/matrix_pro/ops/gemm.hpp:12-70):
  GemmPrecision {fp32, tf32}, GemmEpilogue {none, bias, bias_relu, bias_gelu},
  GemmOptions, GemmPlan (ctor/execute/tune/rows/cols/inner/candidate_count),
  gemm_into, gemm;  multiply/multiply_into (src/ops/matmul.cu:28-65) and
  matrix_pro::hw::cuda_gemm (include/matrix_pro/detail/cuda_hooks.hpp:17-18).

A "Matrix" here is a 2-D float32 CUDA tensor whose rows may be padded (stride
(ld, 1)); the reference's Matrix is the contiguous special case. Device memory and
streams come from torch; all arithmetic runs in libmfb.so's sm_100a kernels.
"""
from __future__ import annotations

import ctypes
import enum
import threading
from collections import OrderedDict
from dataclasses import dataclass

import torch

from . import _lib
from .errors import InvalidArgumentError, ShapeMismatchError

INT32_MAX = 2 ** 31 - 1


class GemmPrecision(enum.IntEnum):
    """fp32 forbids reduced-precision input conversion (strict, 3xTF32 on tcgen05);
    tf32 permits it (single pass). include/matrix_pro/ops/gemm.hpp:12."""
    fp32 = 0
    tf32 = 1


class GemmEpilogue(enum.IntEnum):
    """include/matrix_pro/ops/gemm.hpp:13."""
    none = 0
    bias = 1
    bias_relu = 2
    bias_gelu = 3


@dataclass
class GemmOptions:
    """include/matrix_pro/ops/gemm.hpp:15-23 (workspace_limit_bytes is accepted for
    source compatibility; plans size their own scratch)."""
    transpose_left: bool = False
    transpose_right: bool = False
    precision: GemmPrecision = GemmPrecision.fp32
    epilogue: GemmEpilogue = GemmEpilogue.none
    workspace_limit_bytes: int = 64 << 20


@dataclass
class GemmTuningResult:
    candidates_tested: int = 0
    selected_ms: float = 0.0


def checked_dim(value: int) -> int:
    """src/ops/gemm/plan/environment.inc:15-19."""
    if value < 0 or value > INT32_MAX:
        raise InvalidArgumentError("GEMM dimension exceeds the 32-bit backend limit")
    return int(value)


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream_handle(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _ld(t: torch.Tensor, what: str, host_ok: bool = False) -> int:
    """Leading dimension of a row-major (possibly row-padded) 2-D float32 CUDA tensor (or CPU
    tensor, where the entry point accepts host memory)."""
    if t.dtype != torch.float32:
        raise InvalidArgumentError(f"{what} must be float32")
    if not t.is_cuda and not host_ok:
        raise InvalidArgumentError(f"{what} must be a CUDA tensor")
    if t.dim() != 2:
        raise ShapeMismatchError(f"{what} must be a matrix")
    if t.numel() == 0:
        return max(1, t.shape[1])
    if t.stride(1) != 1 and t.shape[1] > 1:
        raise InvalidArgumentError(f"{what} must have unit column stride")
    return max(int(t.stride(0)), t.shape[1], 1) if t.shape[0] > 1 else max(t.shape[1], 1)


def make_desc(m, n, k, lda, ldb, ldc, alpha=1.0, beta=0.0, precision=0, trans_a=0, trans_b=0, epilogue=0):
    return _lib.GemmDesc(m, n, k, lda, ldb, ldc, float(alpha), float(beta), int(precision), int(trans_a),
                         int(trans_b), int(epilogue))


# ----------------------------------------------------------------------------------------
# Pointer-level entry points (the hw layer)
# ----------------------------------------------------------------------------------------
def cuda_gemm(device: int, m: int, n: int, k: int, a: int, lda: int, b: int, ldb: int, c: int, ldc: int,
              alpha: float, beta: float) -> None:
    """matrix_pro::hw::cuda_gemm: asynchronous strict-FP32 GEMM of device pointers on the
    device's internal stream; wait with cuda_sync(device)."""
    _lib.check(_lib.lib().mfb_cuda_gemm(device, m, n, k, a, lda, b, ldb, c, ldc, alpha, beta), "cuda_gemm")


def cuda_sync(device: int) -> None:
    """matrix_pro::hw::cuda_sync: wait for the device's internal stream; raises on
    CUDA errors and on device-side wait timeouts."""
    _lib.check(_lib.lib().mfb_cuda_sync(device), "cuda_sync")


def sgemm_ptr(device: int, stream: int, desc, a: int, b: int, c: int, bias: int = 0) -> None:
    _lib.check(_lib.lib().mfb_sgemm(device, stream, ctypes.byref(desc), a, b, c, bias), "sgemm")


def sync(device: int | None = None, stream=None) -> None:
    """Synchronize a stream and surface device-side timeouts as DeviceTimeoutError."""
    dev = torch.cuda.current_device() if device is None else device
    _lib.check(_lib.lib().mfb_sync(dev, _stream_handle(stream)), "sync")


def probe_tf32_mma_tflops(n: int = 256, device: int | None = None) -> float:
    """Measured TF32 tcgen05 MMA rate (TFLOP/s) of the device: back-to-back M=128, N=n, K=8
    MMAs on every SM from reused shared-memory operands (the tensor pipe's ceiling)."""
    dev = torch.cuda.current_device() if device is None else device
    out = ctypes.c_float(0.0)
    _lib.check(_lib.lib().mfb_probe_tf32_mma_tflops(dev, int(n), ctypes.byref(out)), "probe_tf32_mma_tflops")
    return float(out.value)


def device_status(device: int | None = None) -> int:
    """Read and clear the device status word (0 = no bounded wait gave up)."""
    dev = torch.cuda.current_device() if device is None else device
    bits = ctypes.c_uint32(0)
    st = _lib.lib().mfb_device_status(dev, ctypes.byref(bits))
    if st not in (_lib.MFB_OK, _lib.MFB_ETIMEOUT):
        _lib.check(st, "device_status")
    return int(bits.value)


def set_wait_limit_ns(limit_ns: int) -> None:
    _lib.check(_lib.lib().mfb_set_wait_limit_ns(int(limit_ns)), "set_wait_limit_ns")


def get_wait_limit_ns() -> int:
    return int(_lib.lib().mfb_get_wait_limit_ns())


# ----------------------------------------------------------------------------------------
# Tensor-level helpers
# ----------------------------------------------------------------------------------------
def _gemm_dims(left: torch.Tensor, right: torch.Tensor, o: GemmOptions):
    m = left.shape[1] if o.transpose_left else left.shape[0]
    k = left.shape[0] if o.transpose_left else left.shape[1]
    k2 = right.shape[1] if o.transpose_right else right.shape[0]
    n = right.shape[0] if o.transpose_right else right.shape[1]
    return m, n, k, k2


def sgemm(left: torch.Tensor, right: torch.Tensor, out: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
          options: GemmOptions | None = None, bias: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """One-shot out = epilogue(alpha*op(left)*op(right) + beta*out) on the current stream."""
    o = options or GemmOptions()
    m, n, k, k2 = _gemm_dims(left, right, o)
    if k != k2:
        raise ShapeMismatchError("GEMM inner dimension mismatch")
    if tuple(out.shape) != (m, n):
        raise ShapeMismatchError("GEMM output shape mismatch")
    desc = make_desc(checked_dim(m), checked_dim(n), checked_dim(k), _ld(left, "left"), _ld(right, "right"),
                     _ld(out, "output"), alpha, beta, int(o.precision), int(o.transpose_left),
                     int(o.transpose_right), int(o.epilogue))
    _check_bias(o, bias, n)
    sgemm_ptr(out.device.index, _stream_handle(stream), desc, _ptr(left), _ptr(right), _ptr(out), _ptr(bias))
    return out


def sgemm_host(left: torch.Tensor, right: torch.Tensor, out: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
               options: GemmOptions | None = None, bias: torch.Tensor | None = None, device: int | None = None,
               stream=None) -> torch.Tensor:
    """out = epilogue(alpha*op(left)*op(right) + beta*out) where each operand may be a CPU tensor
    (pinned memory copies at full PCIe speed) or a tensor on `device`: the GPU share of the
    reference's host-side GEMM (HeterogeneousScheduler::gemm, src/hw/scheduler.cpp:236-312),
    with the rows of out streamed through the GPU in panels so the copies overlap the GEMM
    (mfb_sgemm_host). Stream-ordered: a CPU `out` holds the result once `stream` (default: the
    current stream) has been synchronized."""
    o = options or GemmOptions()
    m, n, k, k2 = _gemm_dims(left, right, o)
    if k != k2:
        raise ShapeMismatchError("GEMM inner dimension mismatch")
    if tuple(out.shape) != (m, n):
        raise ShapeMismatchError("GEMM output shape mismatch")
    for t, what in ((left, "left"), (right, "right"), (out, "output")):
        if t.dtype != torch.float32:
            raise InvalidArgumentError(f"{what} must be float32")
    if o.epilogue != GemmEpilogue.none:
        if bias is None or bias.numel() != n:
            raise ShapeMismatchError("GEMM bias length must equal N")
        if bias.dtype != torch.float32 or not bias.is_contiguous():
            raise InvalidArgumentError("GEMM bias must be a contiguous float32 tensor")
    cuda = [t.device.index for t in (left, right, out, bias) if t is not None and t.is_cuda]
    dev = cuda[0] if cuda else (torch.cuda.current_device() if device is None else device)
    if any(i != dev for i in cuda):
        raise InvalidArgumentError("device operands of sgemm_host must share one device")
    desc = make_desc(checked_dim(m), checked_dim(n), checked_dim(k), _ld(left, "left", True),
                     _ld(right, "right", True), _ld(out, "output", True), alpha, beta, int(o.precision),
                     int(o.transpose_left), int(o.transpose_right), int(o.epilogue))
    with torch.cuda.device(dev):
        handle = _stream_handle(stream)
    _lib.check(_lib.lib().mfb_sgemm_host(dev, handle, ctypes.byref(desc), _ptr(left), _ptr(right), _ptr(out),
                                         _ptr(bias)), "sgemm_host")
    return out


def _check_bias(o: GemmOptions, bias, n: int) -> None:
    if o.epilogue != GemmEpilogue.none:
        if bias is None or bias.numel() != n:
            raise ShapeMismatchError("GEMM bias length must equal N")
        if bias.dtype != torch.float32 or not bias.is_cuda or not bias.is_contiguous():
            raise InvalidArgumentError("GEMM bias must be a contiguous float32 CUDA tensor")


def gemv(a: torch.Tensor, x: torch.Tensor, out: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
         stream=None) -> torch.Tensor:
    """Bandwidth-bound FP32 GEMV / skinny GEMM: out[m x n] = alpha*a[m x k] @ x[k x n] + beta*out
    for n <= 16 or m == 1 (replaces gemm_gemv, src/ops/gemm/gemm_gemv.cu:86)."""
    m, k = a.shape
    k2, n = x.shape
    if k != k2 or tuple(out.shape) != (m, n):
        raise ShapeMismatchError("GEMV operand shape mismatch")
    desc = make_desc(m, n, k, _ld(a, "a"), _ld(x, "x"), _ld(out, "out"), alpha, beta)
    _lib.check(_lib.lib().mfb_gemv(out.device.index, _stream_handle(stream), ctypes.byref(desc), _ptr(a), _ptr(x),
                                   _ptr(out), 0), "gemv")
    return out


def naive_sgemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, alpha: float = 1.0, beta: float = 0.0,
                stream=None) -> torch.Tensor:
    """Device correctness oracle: one thread per output, sequential FP32 FMA chain."""
    m, k = a.shape
    k2, n = b.shape
    if k != k2 or tuple(out.shape) != (m, n):
        raise ShapeMismatchError("GEMM operand shape mismatch")
    desc = make_desc(m, n, k, _ld(a, "a"), _ld(b, "b"), _ld(out, "out"), alpha, beta)
    _lib.check(_lib.lib().mfb_naive_sgemm(out.device.index, _stream_handle(stream), ctypes.byref(desc), _ptr(a),
                                          _ptr(b), _ptr(out), 0), "naive_sgemm")
    return out


# ----------------------------------------------------------------------------------------
# GemmPlan (include/matrix_pro/ops/gemm.hpp:36-62, src/ops/gemm/plan/*.inc)
# ----------------------------------------------------------------------------------------
class GemmPlan:
    """Reusable C = epilogue(alpha*op(A)*op(B) + beta*C).

    Construct on the intended device/thread/stream BEFORE graph capture; warm
    execute allocates nothing and is one launch (two for strict FP32: the split
    prepass, then the tcgen05 GEMM). Bound to its creating thread, device and
    stream, like the reference (implementation.inc:88-93)."""

    def __init__(self, m: int, n: int, k: int, options: GemmOptions | None = None, *, _empty: bool = False):
        self._handle = None
        if _empty:
            return
        o = options or GemmOptions()
        if int(o.precision) not in (0, 1):
            raise InvalidArgumentError("Invalid GEMM precision policy")
        if int(o.epilogue) < 0 or int(o.epilogue) > 3:
            raise InvalidArgumentError("Invalid GEMM epilogue")
        self.m, self.n, self.k = checked_dim(m), checked_dim(n), checked_dim(k)
        self.options = o
        self.device = torch.cuda.current_device()
        self.stream = torch.cuda.current_stream(self.device)
        self.owner = threading.get_ident()
        if torch.cuda.is_current_stream_capturing():
            raise InvalidArgumentError("Construct/tune GEMM plans before CUDA Graph capture")
        # Packed lds of contiguous operands; execute() re-validates the actual tensors.
        lda = max(1, self.m if o.transpose_left else self.k)
        ldb = max(1, self.k if o.transpose_right else self.n)
        desc = make_desc(self.m, self.n, self.k, lda, ldb, max(1, self.n), 1.0, 0.0, int(o.precision),
                         int(o.transpose_left), int(o.transpose_right), int(o.epilogue))
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().mfb_plan_create(self.device, ctypes.byref(desc), ctypes.byref(h)), "GemmPlan")
        self._handle = h
        self._candidates = self.info().candidates

    # -- lifetime ---------------------------------------------------------------------
    def __del__(self):
        self.close()

    def close(self) -> None:
        h, self._handle = getattr(self, "_handle", None), None
        if h is not None and h.value:
            try:
                _lib.lib().mfb_plan_destroy(h)
            except Exception:
                pass

    def move(self) -> "GemmPlan":
        """std::move analogue: the returned plan owns the state; this one becomes empty."""
        other = GemmPlan(0, 0, 0, _empty=True)
        other.__dict__.update(self.__dict__)
        self._handle = None
        return other

    # -- queries ----------------------------------------------------------------------
    def rows(self) -> int:
        return self.m if self._handle else 0

    def cols(self) -> int:
        return self.n if self._handle else 0

    def inner(self) -> int:
        return self.k if self._handle else 0

    def candidate_count(self) -> int:
        return self._candidates if self._handle else 0

    def select_candidate(self, index: int) -> None:
        """Run candidate `index` (0 = the plan's first choice) from now on, as tune() does
        with the fastest one."""
        if not self._handle:
            raise InvalidArgumentError("Cannot select on a moved-from GEMM plan")
        _lib.check(_lib.lib().mfb_plan_select_candidate(self._handle, int(index)), "plan select candidate")

    def uses_tcgen05(self) -> bool:
        return bool(self._handle) and self.info().path == 0

    def info(self) -> _lib.PlanInfo:
        if not self._handle:
            raise InvalidArgumentError("Cannot query a moved-from GEMM plan")
        info = _lib.PlanInfo()
        _lib.check(_lib.lib().mfb_plan_info_get(self._handle, ctypes.byref(info)), "plan info")
        return info

    # -- execution --------------------------------------------------------------------
    def _validate(self, left, right, output, bias):
        """src/ops/gemm/plan/implementation.inc:88-110."""
        if (threading.get_ident() != self.owner or torch.cuda.current_device() != self.device
                or torch.cuda.current_stream(self.device) != self.stream):
            raise InvalidArgumentError("GEMM plan must execute on its creating thread, device and stream")
        o = self.options
        exp_left = (self.k, self.m) if o.transpose_left else (self.m, self.k)
        exp_right = (self.n, self.k) if o.transpose_right else (self.k, self.n)
        if tuple(left.shape) != exp_left or tuple(right.shape) != exp_right or tuple(output.shape) != (self.m,
                                                                                                        self.n):
            raise ShapeMismatchError("GEMM plan operand shape mismatch")
        if output.numel() and (output.data_ptr() == left.data_ptr() or output.data_ptr() == right.data_ptr()):
            raise InvalidArgumentError("GEMM output cannot alias an input")
        if o.epilogue != GemmEpilogue.none:
            if bias is None or bias.numel() != self.n:
                raise ShapeMismatchError("GEMM bias length must equal N")
            if output.numel() and output.data_ptr() == bias.data_ptr():
                raise InvalidArgumentError("GEMM output cannot alias bias")

    def execute(self, left: torch.Tensor, right: torch.Tensor, output: torch.Tensor, alpha: float = 1.0,
                beta: float = 0.0, bias: torch.Tensor | None = None) -> None:
        if not self._handle:
            raise InvalidArgumentError("Cannot execute a moved-from GEMM plan")
        self._validate(left, right, output, bias)
        if self.m == 0 or self.n == 0:
            return
        lda, ldb, ldc = _ld(left, "left"), _ld(right, "right"), _ld(output, "output")
        o = self.options
        if (lda != max(1, self.m if o.transpose_left else self.k) or ldb != max(1, self.k if o.transpose_right
                                                                                 else self.n)
                or ldc != max(1, self.n)):
            raise InvalidArgumentError("GemmPlan operands must be contiguous matrices")
        _lib.check(_lib.lib().mfb_plan_execute(self._handle, _stream_handle(self.stream), _ptr(left), _ptr(right),
                                               _ptr(output), float(alpha), float(beta), _ptr(bias)),
                   "GemmPlan.execute")

    def prepare(self, left: torch.Tensor, right: torch.Tensor) -> None:
        """Operand prepass only (3xTF32 split into the plan's scratch); see mfb_plan_prepare."""
        if not self._handle:
            raise InvalidArgumentError("Cannot execute a moved-from GEMM plan")
        _lib.check(_lib.lib().mfb_plan_prepare(self._handle, _stream_handle(self.stream), _ptr(left), _ptr(right)),
                   "GemmPlan.prepare")

    def multiply(self, left: torch.Tensor, right: torch.Tensor, output: torch.Tensor, alpha: float = 1.0,
                 beta: float = 0.0, bias: torch.Tensor | None = None) -> None:
        """GEMM kernel only, on operands prepared by prepare(); see mfb_plan_multiply."""
        if not self._handle:
            raise InvalidArgumentError("Cannot execute a moved-from GEMM plan")
        self._validate(left, right, output, bias)
        _lib.check(_lib.lib().mfb_plan_multiply(self._handle, _stream_handle(self.stream), _ptr(left), _ptr(right),
                                                _ptr(output), float(alpha), float(beta), _ptr(bias)),
                   "GemmPlan.multiply")

    def set_sm_limit(self, sms: int) -> None:
        """Cap the persistent GEMM grid (0 = all SMs)."""
        _lib.check(_lib.lib().mfb_plan_set_sm_limit(self._handle, int(sms)), "GemmPlan.set_sm_limit")

    def tune(self, left: torch.Tensor, right: torch.Tensor, output: torch.Tensor, alpha: float = 1.0,
             beta: float = 0.0, bias: torch.Tensor | None = None, repeats: int = 5) -> GemmTuningResult:
        """Times every admissible tile configuration on a scratch output (output and
        beta's input stay unchanged) and keeps the fastest. Synchronizes; never capture it."""
        if not self._handle:
            raise InvalidArgumentError("Cannot tune a moved-from GEMM plan")
        self._validate(left, right, output, bias)
        if torch.cuda.is_current_stream_capturing():
            raise InvalidArgumentError("Construct/tune GEMM plans before CUDA Graph capture")
        scratch = torch.empty((max(self.m, 1), max(self.n, 1)), dtype=torch.float32, device=output.device)
        tested, best = ctypes.c_int(0), ctypes.c_float(0.0)
        _lib.check(_lib.lib().mfb_plan_tune(self._handle, _stream_handle(self.stream), _ptr(left), _ptr(right),
                                            _ptr(scratch), int(repeats), ctypes.byref(tested), ctypes.byref(best)),
                   "GemmPlan.tune")
        return GemmTuningResult(int(tested.value), float(best.value))


# ----------------------------------------------------------------------------------------
# Convenience API with a bounded per-thread plan cache (src/ops/gemm/plan/cache.inc:8-50)
# ----------------------------------------------------------------------------------------
_CACHE_LIMIT = 128
_tls = threading.local()


def _cached(m, n, k, o: GemmOptions) -> GemmPlan:
    cache = getattr(_tls, "plans", None)
    if cache is None:
        cache = _tls.plans = OrderedDict()
    dev = torch.cuda.current_device()
    key = (dev, torch.cuda.current_stream(dev).cuda_stream, m, n, k, bool(o.transpose_left),
           bool(o.transpose_right), int(o.precision), int(o.epilogue))
    plan = cache.get(key)
    if plan is None:
        if len(cache) >= _CACHE_LIMIT:
            _, old = cache.popitem(last=False)
            old.close()
        plan = GemmPlan(m, n, k, o)
        cache[key] = plan
    return plan


def gemm_into(left: torch.Tensor, right: torch.Tensor, output: torch.Tensor, options: GemmOptions | None = None,
              alpha: float = 1.0, beta: float = 0.0, bias: torch.Tensor | None = None) -> None:
    """src/ops/gemm/plan/convenience.inc:5-14. Set beta != 0 only when output holds valid data."""
    o = options or GemmOptions()
    m, n, k, k2 = _gemm_dims(left, right, o)
    if k != k2:
        raise ShapeMismatchError("GEMM inner dimension mismatch")
    _cached(m, n, k, o).execute(left, right, output, alpha, beta, bias)


def gemm(left: torch.Tensor, right: torch.Tensor, options: GemmOptions | None = None, alpha: float = 1.0,
         bias: torch.Tensor | None = None) -> torch.Tensor:
    """src/ops/gemm/plan/convenience.inc:15-27."""
    o = options or GemmOptions()
    m, n, k, k2 = _gemm_dims(left, right, o)
    checked_dim(m)
    checked_dim(n)
    if k != k2:
        raise ShapeMismatchError("GEMM inner dimension mismatch")
    out = torch.empty((m, n), dtype=torch.float32, device=left.device)
    gemm_into(left, right, out, o, alpha, 0.0, bias)
    return out


def multiply_into(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> None:
    """src/ops/matmul.cu:47-65 (strict FP32 here: no silent TF32 shape policy)."""
    gemm_into(a, b, out)


def multiply(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """src/ops/matmul.cu:28-45."""
    return gemm(a, b)


def gemm_bias_relu(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """src/ops/matmul.cu:67-85."""
    return gemm(a, b, GemmOptions(epilogue=GemmEpilogue.bias_relu), 1.0, bias.reshape(-1))


def gemm_bias_gelu(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """src/ops/matmul.cu:87-105."""
    return gemm(a, b, GemmOptions(epilogue=GemmEpilogue.bias_gelu), 1.0, bias.reshape(-1))
