"""MatrixFlash-B200: B200-native (sm_100a) dense FP32 contraction path.

Drop-in for MatrixFlash-Pro's GEMM / GEMV / conv2d-forward hot path:
``cuda_gemm``/``cuda_sync`` (hw layer), ``GemmPlan``/``gemm``/``gemm_into``
(Matrix API), ``gemv``, ``conv2d`` forward and backward, the strided-batched ``batch_matmul`` family and
``covariance``/``correlation``.
All arithmetic runs in libmfb.so
(hand-written tcgen05/TMA kernels); there is no CPU fallback.
"""
from .errors import (CudaError, DeviceTimeoutError, InvalidArgumentError, MatrixProError,  # noqa: F401
                     ShapeMismatchError)
from .gemm import (GemmEpilogue, GemmOptions, GemmPlan, GemmPrecision, GemmTuningResult, checked_dim, cuda_gemm,  # noqa: F401,E501
                   cuda_sync, device_status, gemm, gemm_bias_gelu, gemm_bias_relu, gemm_into, gemv,
                   get_wait_limit_ns, make_desc, multiply, multiply_into, naive_sgemm, probe_tf32_mma_tflops,
                   set_wait_limit_ns, sgemm, sgemm_host,
                   sgemm_ptr, sync)
from .conv import (conv2d, conv2d_bias_backward, conv2d_input_backward, conv2d_into, conv2d_out_shape,  # noqa: F401
                   conv2d_weight_backward)
from .batch import (batch_matmul, batch_matmul_backward_left, batch_matmul_backward_right,  # noqa: F401
                    sgemm_strided_batched)
from .stats import correlation, covariance  # noqa: F401
from . import collectives  # noqa: F401
from ._lib import LIB_PATH, lib  # noqa: F401

__version__ = "0.1.0"
