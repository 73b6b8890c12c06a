"""ctypes binding of libmfb.so (the C ABI in include/mfb.h).

The library is built in-tree by ``matrixflash_pro_b200.build``. There is no
fallback: if libmfb.so is missing or cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .errors import CudaError, DeviceTimeoutError, InvalidArgumentError, MatrixProError, ShapeMismatchError

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmfb.so")

MFB_OK, MFB_EINVAL, MFB_ECUDA, MFB_ETIMEOUT, MFB_ENCCL, MFB_EUNSUPPORTED, MFB_ENOMEM, MFB_ESHAPE = range(8)

# Every symbol include/mfb.h declares, in header order.
EXPORTED_SYMBOLS = (
    "mfb_status_string", "mfb_last_error", "mfb_version", "mfb_device_status", "mfb_set_wait_limit_ns",
    "mfb_get_wait_limit_ns", "mfb_sync", "mfb_cuda_gemm", "mfb_cuda_sync", "mfb_cuda_device_count", "mfb_sgemm", "mfb_sgemm_host",
    "mfb_sgemm_multi", "mfb_sgemm_noalloc", "mfb_sgemm_strided_batched",
    "mfb_plan_create", "mfb_plan_execute", "mfb_plan_prepare", "mfb_plan_multiply", "mfb_plan_prepare_cols",
    "mfb_plan_multiply_cols", "mfb_plan_set_sm_limit",
    "mfb_plan_tune", "mfb_plan_select_candidate", "mfb_plan_info_get", "mfb_plan_destroy", "mfb_gemv",
    "mfb_conv2d_fwd", "mfb_naive_sgemm", "mfb_probe_wait_timeout", "mfb_covariance", "mfb_correlation",
    "mfb_probe_tf32_mma_tflops", "mfb_conv2d_bwd_data", "mfb_conv2d_bwd_filter", "mfb_conv2d_bwd_bias",
    "mfb_all_reduce", "mfb_broadcast", "mfb_all_gather", "mfb_reduce_scatter", "mfb_scatter", "mfb_gather",
    "mfb_cuda_nccl_allreduce",
)


class GemmDesc(ctypes.Structure):
    """mfb_gemm_desc (include/mfb.h)."""
    _fields_ = [("m", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int), ("lda", ctypes.c_int),
                ("ldb", ctypes.c_int), ("ldc", ctypes.c_int), ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
                ("precision", ctypes.c_int), ("trans_a", ctypes.c_int), ("trans_b", ctypes.c_int),
                ("epilogue", ctypes.c_int)]


class CollectiveBuffer(ctypes.Structure):
    """mfb_collective_buffer (include/mfb.h)."""
    _fields_ = [("data", ctypes.c_void_p), ("count", ctypes.c_size_t), ("device", ctypes.c_int)]


class RowBlock(ctypes.Structure):
    """mfb_row_block (include/mfb.h)."""
    _fields_ = [("device", ctypes.c_int), ("rows", ctypes.c_int), ("a", ctypes.c_void_p), ("c", ctypes.c_void_p)]


class PlanInfo(ctypes.Structure):
    """mfb_plan_info (include/mfb.h)."""
    _fields_ = [("m", ctypes.c_int), ("n", ctypes.c_int), ("k", ctypes.c_int), ("precision", ctypes.c_int),
                ("trans_a", ctypes.c_int), ("trans_b", ctypes.c_int), ("epilogue", ctypes.c_int),
                ("path", ctypes.c_int), ("tile_n", ctypes.c_int), ("stages", ctypes.c_int),
                ("candidates", ctypes.c_int), ("workspace_bytes", ctypes.c_size_t), ("kernel", ctypes.c_char * 64),
                ("sm_pair", ctypes.c_int), ("split_k", ctypes.c_int), ("stream_k_tiles", ctypes.c_int),
                ("workers", ctypes.c_int)]


_vp = ctypes.c_void_p
_lib = None
_lock = threading.Lock()


def _declare(lib):
    st = ctypes.c_int
    sig = {
        "mfb_status_string": (ctypes.c_char_p, [st]),
        "mfb_last_error": (ctypes.c_char_p, []),
        "mfb_version": (ctypes.c_char_p, []),
        "mfb_device_status": (st, [ctypes.c_int, ctypes.POINTER(ctypes.c_uint32)]),
        "mfb_set_wait_limit_ns": (st, [ctypes.c_uint64]),
        "mfb_get_wait_limit_ns": (ctypes.c_uint64, []),
        "mfb_sync": (st, [ctypes.c_int, _vp]),
        "mfb_cuda_gemm": (st, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp,
                               ctypes.c_int, _vp, ctypes.c_int, ctypes.c_float, ctypes.c_float]),
        "mfb_cuda_sync": (st, [ctypes.c_int]),
        "mfb_cuda_device_count": (st, [ctypes.POINTER(ctypes.c_int)]),
        "mfb_sgemm": (st, [ctypes.c_int, _vp, ctypes.POINTER(GemmDesc), _vp, _vp, _vp, _vp]),
        "mfb_sgemm_host": (st, [ctypes.c_int, _vp, ctypes.POINTER(GemmDesc), _vp, _vp, _vp, _vp]),
        "mfb_sgemm_noalloc": (st, [ctypes.c_int, _vp, ctypes.POINTER(GemmDesc), _vp, _vp, _vp, _vp]),
        "mfb_sgemm_multi": (st, [ctypes.POINTER(RowBlock), ctypes.c_int, ctypes.c_int, ctypes.POINTER(GemmDesc), _vp,
                                 _vp]),
        "mfb_all_reduce": (st, [ctypes.POINTER(CollectiveBuffer), ctypes.c_int, ctypes.c_int, ctypes.c_int]),
        "mfb_broadcast": (st, [ctypes.POINTER(CollectiveBuffer), ctypes.c_int, ctypes.c_int]),
        "mfb_all_gather": (st, [ctypes.POINTER(CollectiveBuffer), ctypes.c_int, ctypes.c_size_t]),
        "mfb_reduce_scatter": (st, [ctypes.POINTER(CollectiveBuffer), ctypes.c_int, ctypes.c_int]),
        "mfb_scatter": (st, [ctypes.POINTER(CollectiveBuffer), ctypes.c_int, ctypes.c_int, ctypes.c_size_t]),
        "mfb_gather": (st, [ctypes.POINTER(CollectiveBuffer), ctypes.c_int, ctypes.c_int, ctypes.c_size_t]),
        "mfb_cuda_nccl_allreduce": (st, [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                         ctypes.c_size_t, ctypes.c_int]),
        "mfb_conv2d_bwd_data": (st, [ctypes.c_int, _vp] + [ctypes.c_int] * 9 + [_vp, _vp, _vp, ctypes.c_int]),
        "mfb_conv2d_bwd_filter": (st, [ctypes.c_int, _vp] + [ctypes.c_int] * 9 + [_vp, _vp, _vp, ctypes.c_int]),
        "mfb_conv2d_bwd_bias": (st, [ctypes.c_int, _vp] + [ctypes.c_int] * 4 + [_vp, _vp]),
        "mfb_probe_tf32_mma_tflops": (st, [ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_float)]),
        "mfb_covariance": (st, [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int,
                                ctypes.c_int]),
        "mfb_correlation": (st, [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int, _vp, ctypes.c_int,
                                 ctypes.c_int]),
        "mfb_sgemm_strided_batched": (st, [ctypes.c_int, _vp, ctypes.POINTER(GemmDesc), _vp, ctypes.c_longlong, _vp,
                                           ctypes.c_longlong, _vp, ctypes.c_longlong, ctypes.c_int, _vp]),
        "mfb_plan_create": (st, [ctypes.c_int, ctypes.POINTER(GemmDesc), ctypes.POINTER(_vp)]),
        "mfb_plan_execute": (st, [_vp, _vp, _vp, _vp, _vp, ctypes.c_float, ctypes.c_float, _vp]),
        "mfb_plan_prepare": (st, [_vp, _vp, _vp, _vp]),
        "mfb_plan_multiply": (st, [_vp, _vp, _vp, _vp, _vp, ctypes.c_float, ctypes.c_float, _vp]),
        "mfb_plan_prepare_cols": (st, [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
        "mfb_plan_multiply_cols": (st, [_vp, _vp, _vp, _vp, ctypes.c_float, ctypes.c_float, _vp, ctypes.c_int,
                                        ctypes.c_int]),
        "mfb_plan_set_sm_limit": (st, [_vp, ctypes.c_int]),
        "mfb_plan_tune": (st, [_vp, _vp, _vp, _vp, _vp, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                               ctypes.POINTER(ctypes.c_float)]),
        "mfb_plan_select_candidate": (st, [_vp, ctypes.c_int]),
        "mfb_plan_info_get": (st, [_vp, ctypes.POINTER(PlanInfo)]),
        "mfb_plan_destroy": (st, [_vp]),
        "mfb_gemv": (st, [ctypes.c_int, _vp, ctypes.POINTER(GemmDesc), _vp, _vp, _vp, _vp]),
        "mfb_conv2d_fwd": (st, [ctypes.c_int, _vp] + [ctypes.c_int] * 9 + [_vp, _vp, _vp, _vp, ctypes.c_int]),
        "mfb_naive_sgemm": (st, [ctypes.c_int, _vp, ctypes.POINTER(GemmDesc), _vp, _vp, _vp, _vp]),
        "mfb_probe_wait_timeout": (st, [ctypes.c_int, _vp, ctypes.c_uint64]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def lib():
    """The loaded libmfb.so. Raises MatrixProError when it is not built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise MatrixProError(f"{LIB_PATH} is not built; run `python -m matrixflash_pro_b200.build` "
                                         "(there is no CPU fallback)")
                _lib = _declare(ctypes.CDLL(LIB_PATH))
    return _lib


def last_error() -> str:
    return lib().mfb_last_error().decode(errors="replace")


def check(status: int, what: str = "") -> None:
    """Map an mfb_status_t to the reference's exception types."""
    if status == MFB_OK:
        return
    detail = last_error()
    msg = f"{what}: {detail}" if what else detail
    if status == MFB_EINVAL:
        raise InvalidArgumentError(msg)
    if status == MFB_ESHAPE:
        raise ShapeMismatchError(msg)
    if status == MFB_ETIMEOUT:
        raise DeviceTimeoutError(msg)
    if status in (MFB_ECUDA, MFB_ENOMEM, MFB_ENCCL):
        raise CudaError(msg)
    raise MatrixProError(f"{lib().mfb_status_string(status).decode()}: {msg}")
