"""CPU tier: the oracle check that bench.py runs on a sampled block of every rank's C.

The operator under check is a CPU stand-in here: an FP64 product (must pass) and a product
with an error planted on the CPU (must fail), so the gates themselves are exercised without
a GPU."""
import numpy as np
import pytest
import torch

import bench


def _operands(m=300, n=200, k=500, seed=3):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn((m, k), generator=g)
    B = torch.randn((k, n), generator=g) / 64.0
    C = torch.randn((m, n), generator=g)
    return A, B, C


def _fp64_op(A, B, C, alpha, beta):
    C.copy_((alpha * (A.double() @ B.double()) + beta * C.double()).float())


@pytest.mark.parametrize("strict", [True, False])
def test_check_passes_a_correct_product(strict):
    A, B, C = _operands()
    chk = bench.SampledCheck(torch, A.shape[0], B.shape[1], A.shape[1], C, rank=0)
    res = chk.run(torch, _fp64_op, A, B, B.clone(), C, 0.5, 1.0, strict, rank=0)
    s = bench.SampledCheck.summarize([res], strict)
    assert s["ok"], s
    assert s["normwise"] <= s["gate"]


def test_check_restores_c_before_its_step():
    # The timed steps accumulate into C (beta = 1); the check must start from C's first values.
    A, B, C = _operands()
    C0 = C.clone()
    chk = bench.SampledCheck(torch, A.shape[0], B.shape[1], A.shape[1], C, rank=1)
    for _ in range(3):
        _fp64_op(A, B, C, 0.5, 1.0)
    res = chk.run(torch, _fp64_op, A, B, B.clone(), C, 0.5, 1.0, True, rank=1)
    assert res[5] == 1.0
    rows = torch.from_numpy(chk.rows)
    want = (0.5 * (A.double() @ B.double()) + C0.double()).float()
    assert torch.allclose(C.index_select(0, rows), want.index_select(0, rows), rtol=1e-6, atol=1e-6)


def test_check_fails_a_planted_error_and_a_rank_without_b():
    A, B, C = _operands()

    def off_by_a_bit(A, B, C, alpha, beta):
        _fp64_op(A, B, C, alpha, beta)
        C.add_(1e-4)

    chk = bench.SampledCheck(torch, A.shape[0], B.shape[1], A.shape[1], C, rank=0)
    bad = chk.run(torch, off_by_a_bit, A, B, B.clone(), C, 0.5, 1.0, True, rank=0)
    assert bad[5] == 0.0
    # A rank other than the root whose operator read its own (NaN-filled) B fails the check.
    B_buf = B.clone()
    A2, _, C2 = _operands(seed=4)
    chk2 = bench.SampledCheck(torch, A2.shape[0], B.shape[1], A2.shape[1], C2, rank=1)
    res = chk2.run(torch, lambda A_, B_, C_, al, be: _fp64_op(A_, B_buf, C_, al, be), A2, B, B_buf, C2, 0.5, 1.0,
                   True, rank=1)
    assert res[5] == 0.0
    good = [1e-7, 1e-6, 1e-6, 1e-3, 5e-7, 1.0]
    s = bench.SampledCheck.summarize([good, res, good], True)
    assert not s["ok"] and s["worst_rank"] == 1 and s["ranks"] == 3
