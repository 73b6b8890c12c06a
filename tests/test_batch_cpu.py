"""CPU tier: host-side checks of the batched GEMM API (no device work).

The reference's batch_matmul throws InvalidArgumentError for tensors that are not rank 3
and ShapeMismatchError for mismatched shapes (src/nn/batch.cu:13-16,
src/nn/backward/batched_matmul.inc:8-13,33-38); so does the mirror, before any launch."""
import pytest
import torch

import matrixflash_pro_b200 as mf


def test_rank_and_shape_errors_precede_any_launch():
    with pytest.raises(mf.InvalidArgumentError):
        mf.batch_matmul(torch.ones(3, 4), torch.ones(1, 4, 5))
    with pytest.raises(mf.ShapeMismatchError):
        mf.batch_matmul(torch.ones(2, 3, 4), torch.ones(3, 4, 5))
    with pytest.raises(mf.ShapeMismatchError):
        mf.batch_matmul(torch.ones(2, 3, 4), torch.ones(2, 5, 5))
    with pytest.raises(mf.InvalidArgumentError):
        mf.batch_matmul_backward_left(torch.ones(2, 3), torch.ones(2, 4, 5))
    with pytest.raises(mf.ShapeMismatchError):
        mf.batch_matmul_backward_left(torch.ones(2, 3, 5), torch.ones(2, 4, 6))
    with pytest.raises(mf.ShapeMismatchError):
        mf.batch_matmul_backward_right(torch.ones(2, 3, 5), torch.ones(2, 4, 6))


def test_host_tensors_are_rejected():
    """The product has no CPU path: host tensors fail loudly instead of computing."""
    with pytest.raises(mf.InvalidArgumentError):
        mf.sgemm_strided_batched(torch.ones(2, 3, 4), torch.ones(2, 4, 5), torch.empty(2, 3, 5))


def test_collectives_reject_host_tensors():
    with pytest.raises(mf.InvalidArgumentError):
        mf.collectives.all_reduce([torch.ones(4), torch.ones(4)])
    with pytest.raises(mf.InvalidArgumentError):
        mf.collectives.broadcast([], 0)
