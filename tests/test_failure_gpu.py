"""GPU tier: failure detection without a GPU fault.

Every device-side wait in libmfb.so is bounded. A probe kernel waits on an mbarrier
that nothing arrives on, gives up after a short limit and records a status bit; the
host turns that into DeviceTimeoutError and the CUDA context stays usable."""
import numpy as np
import pytest
import torch

import matrixflash_pro_b200 as mf
from matrixflash_pro_b200 import _lib
from helpers import to_dev

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives():
    assert mf.device_status(0) == 0
    _lib.check(_lib.lib().mfb_probe_wait_timeout(0, torch.cuda.current_stream().cuda_stream, 2_000_000))
    with pytest.raises(mf.DeviceTimeoutError):
        mf.sync()
    assert mf.device_status(0) == 0  # read-and-clear
    # The context is still healthy: a GEMM right after runs and is correct.
    a = torch.ones(64, 64, device="cuda")
    out = mf.multiply(a, a)
    torch.cuda.synchronize()
    assert torch.all(out == 64)
    assert mf.device_status(0) == 0


def test_status_bits_reported_raw():
    _lib.check(_lib.lib().mfb_probe_wait_timeout(0, torch.cuda.current_stream().cuda_stream, 1_000_000))
    bits = mf.device_status(0)
    assert bits & (1 << 4)


def test_probe_rejects_unbounded_limits():
    with pytest.raises(mf.InvalidArgumentError):
        _lib.check(_lib.lib().mfb_probe_wait_timeout(0, None, 0))
    with pytest.raises(mf.InvalidArgumentError):
        _lib.check(_lib.lib().mfb_probe_wait_timeout(0, None, 20_000_000_000))


def test_short_wait_limit_does_not_break_normal_kernels():
    old = mf.get_wait_limit_ns()
    try:
        mf.set_wait_limit_ns(200_000_000)  # 0.2 s per wait: far above any legitimate wait here
        a = to_dev(np.eye(300, dtype=np.float32))
        out = mf.multiply(a, a)
        mf.sync()
        assert torch.equal(out, a)
    finally:
        mf.set_wait_limit_ns(old)
