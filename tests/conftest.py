import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")
    config.addinivalue_line("markers", "slow: full-size workloads (still bounded to tens of seconds)")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_gemm():
    import numpy as np
    data = np.load(os.path.join(ROOT, "tests", "golden", "gemm_golden.npz"))
    cases = {}
    for key in data.files:
        name, field = key.split("__", 1)
        if name == "meta":
            continue
        cases.setdefault(name, {})[field] = data[key]
    return cases


@pytest.fixture(scope="session")
def golden_conv():
    import numpy as np
    data = np.load(os.path.join(ROOT, "tests", "golden", "conv_golden.npz"))
    cases = {}
    for key in data.files:
        name, field = key.split("__", 1)
        cases.setdefault(name, {})[field] = data[key]
    return cases
