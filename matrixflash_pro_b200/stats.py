"""Column covariance and correlation over libmfb.so (mfb_covariance / mfb_correlation).

Mirrors matrix_pro::covariance / correlation and Matrix::covariance / correlation
(include/matrix_pro/ops/advanced.hpp:17-18, src/ops/reductions/covariance.inc:23-74): for an
(rows x cols) matrix, covariance is (cols x cols) X_c^T X_c / max(rows - 1, 1) with X_c the
column-centered matrix; correlation normalizes it by sqrt(var_i var_j). As in the reference,
an empty input gives an empty (rows x cols) result. The product is the tcgen05 GEMM (strict
FP32 by default, matching the reference's pedantic-FP32 cuBLAS call; TF32 on request).
"""
from __future__ import annotations

import torch

from . import _lib
from .gemm import GemmPrecision, _ld, _stream_handle, checked_dim


def _run(symbol: str, matrix: torch.Tensor, precision: GemmPrecision) -> torch.Tensor:
    ldx = _ld(matrix, "matrix")  # float32 CUDA matrix with unit column stride, or raises
    rows, cols = checked_dim(matrix.shape[0]), checked_dim(matrix.shape[1])
    if rows == 0 or cols == 0:
        return torch.empty((rows, cols), device=matrix.device, dtype=torch.float32)
    out = torch.empty((cols, cols), device=matrix.device, dtype=torch.float32)
    fn = getattr(_lib.lib(), symbol)
    _lib.check(fn(matrix.device.index, _stream_handle(), rows, cols, matrix.data_ptr(), ldx, out.data_ptr(), cols,
                  int(precision)), symbol)
    return out


def covariance(matrix: torch.Tensor, precision: GemmPrecision = GemmPrecision.fp32) -> torch.Tensor:
    """(cols x cols) sample covariance of the columns (src/ops/reductions/covariance.inc:23-47)."""
    return _run("mfb_covariance", matrix, precision)


def correlation(matrix: torch.Tensor, precision: GemmPrecision = GemmPrecision.fp32) -> torch.Tensor:
    """(cols x cols) correlation of the columns (src/ops/reductions/covariance.inc:49-61)."""
    return _run("mfb_correlation", matrix, precision)
