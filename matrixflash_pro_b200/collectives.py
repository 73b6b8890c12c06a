"""Collectives over per-GPU buffers of one process (mfb_all_reduce & co., on NCCL).

Mirrors include/matrix_pro/distributed/collectives.hpp:20-32: ReduceOp {Sum, Mean, Max},
CollectiveAlgorithm {Ring, Tree}, and all_reduce / broadcast / all_gather / reduce_scatter /
scatter / gather over one buffer per rank. Here a rank's buffer is a contiguous float32 CUDA
tensor (count = numel, device = its GPU). Results land where the reference writes them
(src/hw/collectives.cpp:185-311); ranks on distinct GPUs communicate through NCCL over
NVLink/NVSwitch instead of the reference's host staging, ranks all on one GPU use
device-local copies. Calls are blocking, as in the reference.
"""
from __future__ import annotations

import ctypes
import enum
from typing import Sequence

import torch

from . import _lib
from .errors import InvalidArgumentError


class ReduceOp(enum.IntEnum):
    Sum = 0
    Mean = 1
    Max = 2


class CollectiveAlgorithm(enum.IntEnum):
    """Accepted for source compatibility; NCCL chooses ring or tree itself."""
    Ring = 0
    Tree = 1


def _buffers(tensors: Sequence[torch.Tensor]):
    if len(tensors) == 0:
        raise InvalidArgumentError("collective: no ranks")
    arr = (_lib.CollectiveBuffer * len(tensors))()
    for i, t in enumerate(tensors):
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise InvalidArgumentError("collective buffers must be contiguous float32 CUDA tensors")
        arr[i].data = t.data_ptr() if t.numel() else None
        arr[i].count = t.numel()
        arr[i].device = t.device.index
    return arr, len(tensors)


def all_reduce(tensors: Sequence[torch.Tensor], op: ReduceOp = ReduceOp.Sum,
               algorithm: CollectiveAlgorithm = CollectiveAlgorithm.Ring) -> None:
    arr, n = _buffers(tensors)
    _lib.check(_lib.lib().mfb_all_reduce(arr, n, int(op), int(algorithm)), "all_reduce")


def broadcast(tensors: Sequence[torch.Tensor], root: int) -> None:
    arr, n = _buffers(tensors)
    _lib.check(_lib.lib().mfb_broadcast(arr, n, int(root)), "broadcast")


def all_gather(tensors: Sequence[torch.Tensor], count_per_rank: int) -> None:
    arr, n = _buffers(tensors)
    _lib.check(_lib.lib().mfb_all_gather(arr, n, int(count_per_rank)), "all_gather")


def reduce_scatter(tensors: Sequence[torch.Tensor], op: ReduceOp = ReduceOp.Sum) -> None:
    arr, n = _buffers(tensors)
    _lib.check(_lib.lib().mfb_reduce_scatter(arr, n, int(op)), "reduce_scatter")


def scatter(tensors: Sequence[torch.Tensor], root: int, count_per_rank: int) -> None:
    arr, n = _buffers(tensors)
    _lib.check(_lib.lib().mfb_scatter(arr, n, int(root), int(count_per_rank)), "scatter")


def gather(tensors: Sequence[torch.Tensor], root: int, count_per_rank: int) -> None:
    arr, n = _buffers(tensors)
    _lib.check(_lib.lib().mfb_gather(arr, n, int(root), int(count_per_rank)), "gather")


def cuda_nccl_allreduce(tensors: Sequence[torch.Tensor], op: ReduceOp = ReduceOp.Sum) -> None:
    """hw::cuda_nccl_allreduce (include/matrix_pro/detail/cuda_hooks.hpp:35): in place, equal counts."""
    arr, n = _buffers(tensors)
    ptrs = (ctypes.c_void_p * n)(*[arr[i].data for i in range(n)])
    devs = (ctypes.c_int * n)(*[arr[i].device for i in range(n)])
    _lib.check(_lib.lib().mfb_cuda_nccl_allreduce(ptrs, devs, n, arr[0].count, int(op)), "cuda_nccl_allreduce")
