"""conv2d forward and backward over libmfb.so with the reference's interface and checks.

Reference: matrix_pro::conv2d (include/matrix_pro/nn/conv.hpp:16-17, src/nn/conv.cu:110-163):
input (N,C,H,W), weights (K,C,R,S), bias (K), cross-correlation, output
(N, K, (H+2p-R)/s+1, (W+2p-S)/s+1).
"""
from __future__ import annotations

import torch

from . import _lib
from .errors import InvalidArgumentError, ShapeMismatchError
from .gemm import GemmPrecision, _stream_handle


def conv2d_out_shape(x_shape, w_shape, stride: int, padding: int):
    n, _, h, w = x_shape
    k, _, r, s = w_shape
    return (n, k, (h + 2 * padding - r) // stride + 1, (w + 2 * padding - s) // stride + 1)


def _validate(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, stride: int, padding: int) -> None:
    """src/nn/conv.cu:87-89,111-117."""
    if x.dim() != 4:
        raise ShapeMismatchError("CNN input must have shape [N,C,H,W]")
    if w.dim() != 4 or bias.dim() != 1:
        raise InvalidArgumentError("conv2d expects weights [K,C,R,S] and bias [K]")
    if w.shape[1] != x.shape[1] or bias.shape[0] != w.shape[0] or stride == 0:
        raise ShapeMismatchError("conv2d channel or stride mismatch")
    if x.shape[2] + 2 * padding < w.shape[2] or x.shape[3] + 2 * padding < w.shape[3]:
        raise ShapeMismatchError("conv2d kernel is larger than padded input")
    for t, name in ((x, "input"), (w, "weights"), (bias, "bias")):
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise InvalidArgumentError(f"conv2d {name} must be a contiguous float32 CUDA tensor")


def conv2d_into(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, out: torch.Tensor, stride: int = 1,
                padding: int = 0, precision: GemmPrecision = GemmPrecision.fp32, stream=None) -> torch.Tensor:
    _validate(x, w, bias, stride, padding)
    shape = conv2d_out_shape(x.shape, w.shape, stride, padding)
    if tuple(out.shape) != shape or not out.is_contiguous():
        raise ShapeMismatchError("conv2d output must be a contiguous (N,K,P,Q) tensor")
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    _lib.check(_lib.lib().mfb_conv2d_fwd(out.device.index, _stream_handle(stream), n, c, h, wd, k, r, s, int(stride),
                                         int(padding), x.data_ptr(), w.data_ptr(), bias.data_ptr(), out.data_ptr(),
                                         int(precision)), "conv2d")
    return out


def conv2d(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, stride: int = 1, padding: int = 0,
           precision: GemmPrecision = GemmPrecision.fp32) -> torch.Tensor:
    """Cross-correlation conv2d forward (include/matrix_pro/nn/conv.hpp:16)."""
    _validate(x, w, bias, stride, padding)
    out = torch.empty(conv2d_out_shape(x.shape, w.shape, stride, padding), dtype=torch.float32, device=x.device)
    return conv2d_into(x, w, bias, out, stride, padding, precision)


# ----------------------------------------------------------------------------------------
# Backward (include/matrix_pro/nn/conv.hpp:25-29, src/nn/backward/convolution.inc)
# ----------------------------------------------------------------------------------------
def _validate_backward(grad: torch.Tensor, x_shape, w_shape, stride: int, padding: int) -> None:
    """validate_conv (src/nn/backward/convolution_kernels.cuh:98-115)."""
    if len(x_shape) != 4:
        raise InvalidArgumentError("conv2d backward input must be [N,C,H,W]")
    if len(w_shape) != 4 or grad.dim() != 4:
        raise InvalidArgumentError("conv2d backward expects rank-4 grad/weights")
    n, c, h, w = x_shape
    k, c2, r, s = w_shape
    if c2 != c or grad.shape[0] != n or grad.shape[1] != k or stride <= 0:
        raise ShapeMismatchError("conv2d backward shape mismatch")
    if h + 2 * padding < r or w + 2 * padding < s:
        raise ShapeMismatchError("conv2d backward shape mismatch")
    p, q = (h + 2 * padding - r) // stride + 1, (w + 2 * padding - s) // stride + 1
    if grad.shape[2] != p or grad.shape[3] != q:
        raise ShapeMismatchError("conv2d backward shape mismatch")


def _device_tensor(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
        raise InvalidArgumentError(f"conv2d backward {name} must be a contiguous float32 CUDA tensor")


def conv2d_input_backward(grad: torch.Tensor, x: torch.Tensor, w: torch.Tensor, stride: int = 1, padding: int = 0,
                          precision: GemmPrecision = GemmPrecision.fp32, stream=None) -> torch.Tensor:
    """dL/dinput (N,C,H,W) of conv2d (src/nn/backward/convolution.inc:5-19); `x` gives the shape."""
    _validate_backward(grad, x.shape, w.shape, stride, padding)
    for t, name in ((grad, "grad"), (w, "weights")):
        _device_tensor(t, name)
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    out = torch.empty((n, c, h, wd), dtype=torch.float32, device=grad.device)
    _lib.check(_lib.lib().mfb_conv2d_bwd_data(out.device.index, _stream_handle(stream), n, c, h, wd, k, r, s,
                                              int(stride), int(padding), grad.data_ptr(), w.data_ptr(),
                                              out.data_ptr(), int(precision)), "conv2d_input_backward")
    return out


def conv2d_weight_backward(grad: torch.Tensor, x: torch.Tensor, w: torch.Tensor, stride: int = 1, padding: int = 0,
                           precision: GemmPrecision = GemmPrecision.fp32, stream=None) -> torch.Tensor:
    """dL/dweights (K,C,R,S) of conv2d (src/nn/backward/convolution.inc:21-35); `w` gives the shape."""
    _validate_backward(grad, x.shape, w.shape, stride, padding)
    for t, name in ((grad, "grad"), (x, "input")):
        _device_tensor(t, name)
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    out = torch.empty((k, c, r, s), dtype=torch.float32, device=grad.device)
    _lib.check(_lib.lib().mfb_conv2d_bwd_filter(out.device.index, _stream_handle(stream), n, c, h, wd, k, r, s,
                                                int(stride), int(padding), x.data_ptr(), grad.data_ptr(),
                                                out.data_ptr(), int(precision)), "conv2d_weight_backward")
    return out


def conv2d_bias_backward(grad: torch.Tensor, stream=None) -> torch.Tensor:
    """dL/dbias (K) of conv2d (src/nn/backward/convolution.inc:37-48)."""
    if grad.dim() != 4:
        raise InvalidArgumentError("conv2d bias backward expects a rank-4 gradient")
    _device_tensor(grad, "grad")
    n, k, p, q = grad.shape
    out = torch.empty((k,), dtype=torch.float32, device=grad.device)
    _lib.check(_lib.lib().mfb_conv2d_bwd_bias(out.device.index, _stream_handle(stream), n, k, p, q, grad.data_ptr(),
                                              out.data_ptr()), "conv2d_bias_backward")
    return out
