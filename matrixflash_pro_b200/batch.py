"""Batched GEMM for rank-3 tensors over libmfb.so (mfb_sgemm_strided_batched).

Mirrors include/matrix_pro/nn/batch.hpp:10-14:
  batch_matmul(left[b,m,k], right[b,k,n]) -> [b,m,n]          (src/nn/batch.cu:12-35)
  batch_matmul_backward_left(grad[b,m,n], right[b,k,n]) -> G x B^T   [b,m,k]
  batch_matmul_backward_right(grad[b,m,n], left[b,m,k]) -> A^T x G   [b,k,n]
                                                   (src/nn/backward/batched_matmul.inc:7-55)
with the same errors: InvalidArgumentError for tensors that are not rank 3,
ShapeMismatchError for mismatched shapes. The reference runs these on
cublasSgemmStridedBatched in pedantic FP32; here every batch entry is one tile range
of a single tcgen05 launch (strict 3xTF32 by default, TF32 on request).

A rank-3 operand here is a float32 CUDA tensor with unit stride in its last dimension;
its row stride (padding) and batch stride are taken from the tensor (a batch stride of
0, e.g. from expand(), reuses one matrix for every entry).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .errors import InvalidArgumentError, ShapeMismatchError
from .gemm import GemmEpilogue, GemmOptions, GemmPrecision, _ptr, _stream_handle, checked_dim, make_desc


def _geometry(t: torch.Tensor, what: str):
    """(row stride, batch stride) of a rank-3 float32 CUDA tensor with unit last-dim stride."""
    if t.dim() != 3:
        raise InvalidArgumentError("batch_matmul requires rank-3 tensors")
    if t.dtype != torch.float32:
        raise InvalidArgumentError(f"{what} must be float32")
    if not t.is_cuda:
        raise InvalidArgumentError(f"{what} must be a CUDA tensor")
    b, rows, cols = t.shape
    if t.numel() == 0:
        return max(1, cols), max(1, rows * cols)
    if t.stride(2) != 1 and cols > 1:
        raise InvalidArgumentError(f"{what} must have unit stride in its last dimension")
    ld = max(int(t.stride(1)), cols, 1) if rows > 1 else max(cols, 1)
    bs = int(t.stride(0)) if b > 1 else 0
    if bs < 0:
        raise InvalidArgumentError(f"{what} has a negative batch stride")
    return ld, bs


def sgemm_strided_batched(left: torch.Tensor, right: torch.Tensor, out: torch.Tensor, alpha: float = 1.0,
                          beta: float = 0.0, options: GemmOptions | None = None, bias: torch.Tensor | None = None,
                          stream=None) -> torch.Tensor:
    """out[i] = epilogue(alpha * op(left[i]) @ op(right[i]) + beta * out[i]) for every i, in one launch.
    op() transposes per options.transpose_left / transpose_right (stored shapes then are
    [b,k,m] / [b,n,k])."""
    o = options or GemmOptions()
    lda, sa = _geometry(left, "left")
    ldb, sb = _geometry(right, "right")
    ldc, sc = _geometry(out, "out")
    batch = out.shape[0]
    if left.shape[0] != batch or right.shape[0] != batch:
        raise ShapeMismatchError("batch_matmul shape mismatch")
    m, k = (left.shape[2], left.shape[1]) if o.transpose_left else (left.shape[1], left.shape[2])
    k2, n = (right.shape[2], right.shape[1]) if o.transpose_right else (right.shape[1], right.shape[2])
    if k != k2 or tuple(out.shape[1:]) != (m, n):
        raise ShapeMismatchError("batch_matmul shape mismatch")
    if o.epilogue != GemmEpilogue.none and (bias is None or bias.numel() != n):
        raise ShapeMismatchError("GEMM bias length must equal N")
    desc = make_desc(checked_dim(m), checked_dim(n), checked_dim(k), lda, ldb, ldc, alpha, beta, int(o.precision),
                     int(o.transpose_left), int(o.transpose_right), int(o.epilogue))
    dev = out.device.index if out.is_cuda else torch.cuda.current_device()
    _lib.check(_lib.lib().mfb_sgemm_strided_batched(dev, _stream_handle(stream), ctypes.byref(desc), _ptr(left), sa,
                                                    _ptr(right), sb, _ptr(out), sc, int(batch), _ptr(bias)),
               "sgemm_strided_batched")
    return out


def _precision_options(precision: GemmPrecision, transpose_left=False, transpose_right=False) -> GemmOptions:
    return GemmOptions(transpose_left=transpose_left, transpose_right=transpose_right,
                       precision=GemmPrecision(precision))


def batch_matmul(left: torch.Tensor, right: torch.Tensor,
                 precision: GemmPrecision = GemmPrecision.fp32) -> torch.Tensor:
    """[b,m,k] x [b,k,n] -> [b,m,n] (src/nn/batch.cu:12-35)."""
    if left.dim() != 3 or right.dim() != 3:
        raise InvalidArgumentError("batch_matmul requires rank-3 tensors")
    a, b = left.shape, right.shape
    if a[0] != b[0] or a[2] != b[1]:
        raise ShapeMismatchError("batch_matmul shape mismatch")
    out = torch.empty((a[0], a[1], b[2]), device=left.device, dtype=torch.float32)
    if out.numel() == 0:
        return out
    return sgemm_strided_batched(left, right, out, 1.0, 0.0, _precision_options(precision))


def batch_matmul_backward_left(grad: torch.Tensor, right: torch.Tensor,
                               precision: GemmPrecision = GemmPrecision.fp32) -> torch.Tensor:
    """dL/dA = G x B^T per batch entry: [b,m,n], [b,k,n] -> [b,m,k]
    (src/nn/backward/batched_matmul.inc:7-30)."""
    if grad.dim() != 3 or right.dim() != 3:
        raise InvalidArgumentError("batch_matmul backward requires rank-3 tensors")
    g, b = grad.shape, right.shape
    if g[0] != b[0] or g[2] != b[2]:
        raise ShapeMismatchError("batch_matmul backward shape mismatch")
    out = torch.empty((g[0], g[1], b[1]), device=grad.device, dtype=torch.float32)
    if out.numel() == 0:
        return out
    return sgemm_strided_batched(grad, right, out, 1.0, 0.0, _precision_options(precision, transpose_right=True))


def batch_matmul_backward_right(grad: torch.Tensor, left: torch.Tensor,
                                precision: GemmPrecision = GemmPrecision.fp32) -> torch.Tensor:
    """dL/dB = A^T x G per batch entry: [b,m,n], [b,m,k] -> [b,k,n]
    (src/nn/backward/batched_matmul.inc:32-55)."""
    if grad.dim() != 3 or left.dim() != 3:
        raise InvalidArgumentError("batch_matmul backward requires rank-3 tensors")
    g, a = grad.shape, left.shape
    if g[0] != a[0] or g[1] != a[1]:
        raise ShapeMismatchError("batch_matmul backward shape mismatch")
    out = torch.empty((g[0], a[2], g[2]), device=grad.device, dtype=torch.float32)
    if out.numel() == 0:
        return out
    return sgemm_strided_batched(left, grad, out, 1.0, 0.0, _precision_options(precision, transpose_left=True))
