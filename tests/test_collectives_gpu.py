"""GPU tier: collectives (mfb_all_reduce & co.) against the reference's host algorithms.

Replaces matrix_pro::all_reduce / broadcast / all_gather / reduce_scatter / scatter / gather
(src/hw/collectives.cpp:185-311) and hw::cuda_nccl_allreduce. The expected values restate the
reference's host code with numpy float32: Mean = Sum * float32(1/ranks); reduce_scatter puts rank
r's chunk in front of the all-reduced rest of its buffer (Mean scales that chunk only). Ranks on
one GPU take the device-local path (bit-exact: sums in rank order); ranks on distinct GPUs take
NCCL (skipped with fewer than 2 GPUs)."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
from matrixflash_pro_b200.collectives import ReduceOp

pytestmark = pytest.mark.gpu
C = mf.collectives


def _ranks(devices, count, seed):
    rng = np.random.default_rng(seed)
    host = [rng.standard_normal(count).astype(np.float32) for _ in devices]
    return host, [torch.from_numpy(h.copy()).to(f"cuda:{d}") for h, d in zip(host, devices)]


def _reduce(host, op):
    acc = host[0].copy()
    for h in host[1:]:
        acc = np.maximum(acc, h) if op == ReduceOp.Max else (acc + h).astype(np.float32)
    if op == ReduceOp.Mean:
        acc = (acc * np.float32(1.0 / np.float32(len(host)))).astype(np.float32)
    return acc


def _check_all(devices, exact):
    def same(got, want, what):
        got = got.cpu().numpy()
        if exact:
            assert np.array_equal(got, want), what
        else:
            assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), what

    n = len(devices)
    for op in ReduceOp:
        host, dev = _ranks(devices, 1000, int(op))
        C.all_reduce(dev, op)
        for t in dev:
            same(t, _reduce(host, op), f"all_reduce {op.name}")
    host, dev = _ranks(devices, 777, 7)
    C.broadcast(dev, n - 1)
    for t in dev:
        same(t, host[n - 1], "broadcast")
    host, dev = _ranks(devices, 3 * n + 5, 8)
    C.all_gather(dev, 3)
    gathered = np.concatenate([h[:3] for h in host])
    for h, t in zip(host, dev):
        same(t, np.concatenate([gathered, h[3 * n:]]), "all_gather")
    for op in ReduceOp:
        host, dev = _ranks(devices, 4 * n, 20 + int(op))
        C.reduce_scatter(dev, op)
        total = _reduce(host, ReduceOp.Sum if op == ReduceOp.Mean else op)
        for r, t in enumerate(dev):
            want = total.copy()
            want[:4] = total[4 * r:4 * r + 4]
            if op == ReduceOp.Mean:
                want[:4] = (want[:4] * np.float32(1.0 / np.float32(n))).astype(np.float32)
            same(t, want, f"reduce_scatter {op.name}")
    host, dev = _ranks(devices, 5 * n + 2, 9)
    C.scatter(dev, 0, 5)
    for r, (h, t) in enumerate(zip(host, dev)):
        want = h.copy()
        want[:5] = host[0][5 * r:5 * r + 5]
        same(t, want, "scatter")
    host, dev = _ranks(devices, 6 * n, 10)
    C.gather(dev, n - 1, 6)
    for r, (h, t) in enumerate(zip(host, dev)):
        want = np.concatenate([x[:6] for x in host]) if r == n - 1 else h
        same(t, want, "gather")
    host, dev = _ranks(devices, 513, 11)
    C.cuda_nccl_allreduce(dev, ReduceOp.Sum)
    for t in dev:
        same(t, _reduce(host, ReduceOp.Sum), "cuda_nccl_allreduce")


def test_ranks_on_one_gpu():
    _check_all([0, 0, 0], exact=True)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ranks_on_distinct_gpus_nccl():
    n = min(4, torch.cuda.device_count())
    _check_all(list(range(n)), exact=(n == 2))


def test_errors():
    a = torch.zeros(10, device="cuda")
    with pytest.raises(mf.InvalidArgumentError):
        C.all_reduce([a, torch.zeros(11, device="cuda")])
    with pytest.raises(mf.InvalidArgumentError):
        C.broadcast([a, torch.zeros(10, device="cuda")], 2)
    with pytest.raises(mf.InvalidArgumentError):
        C.all_gather([a, torch.zeros(10, device="cuda")], 6)
    with pytest.raises(mf.InvalidArgumentError):
        C.reduce_scatter([torch.zeros(9, device="cuda"), torch.zeros(9, device="cuda")])
