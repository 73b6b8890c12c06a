"""CPU tier: argument checks of mfb_sgemm_multi (the row split over the GPUs of one process),
with two row blocks. Every call here fails one of the checks that run before the library
touches a device (the placeholder pointers are never dereferenced), so the calls return their
status with or without GPUs; the GPU tier runs the split itself."""
import ctypes

import pytest

import matrixflash_pro_b200 as mf
from matrixflash_pro_b200 import _lib

FAKE = 1 << 32  # non-null placeholders: nothing is dereferenced before the checks pass


def _blocks(specs):
    arr = (_lib.RowBlock * len(specs))()
    for i, (dev, rows, a, c) in enumerate(specs):
        arr[i] = _lib.RowBlock(dev, rows, a, c)
    return arr


def _call(specs, desc, root=0, b=FAKE + 4096, bias=0, count=None):
    blocks = _blocks(specs) if specs else None
    n = len(specs) if count is None else count
    return _lib.lib().mfb_sgemm_multi(blocks, n, root, ctypes.byref(desc) if desc is not None else None, b, bias)


def _desc(m=100, n=64, k=32, **kw):
    return mf.make_desc(m, n, k, k, n, n, **kw)


TWO = [(0, 60, FAKE, FAKE + 1024), (1, 40, FAKE + 2048, FAKE + 3072)]


@pytest.mark.parametrize("specs,desc,root,b,bias,count,want", [
    ([], _desc(), 0, FAKE, 0, 0, _lib.MFB_EINVAL),                          # no blocks
    (TWO, _desc(), 2, FAKE, 0, None, _lib.MFB_EINVAL),                      # root out of range
    (TWO, _desc(), -1, FAKE, 0, None, _lib.MFB_EINVAL),
    (TWO, None, 0, FAKE, 0, None, _lib.MFB_EINVAL),                         # no descriptor
    ([(0, 60, FAKE, FAKE + 1024), (0, 40, FAKE + 2048, FAKE + 3072)], _desc(), 0, FAKE, 0, None,
     _lib.MFB_EINVAL),                                                      # two blocks on one GPU
    (TWO, _desc(m=101), 0, FAKE, 0, None, _lib.MFB_ESHAPE),                 # rows do not add up to m
    ([(0, 110, FAKE, FAKE + 1024), (1, -10, FAKE + 2048, FAKE + 3072)], _desc(), 0, FAKE, 0, None,
     _lib.MFB_EINVAL),                                                      # negative rows
    (TWO, mf.make_desc(100, 64, 32, 100, 64, 64, trans_a=1), 0, FAKE, 0, None,
     _lib.MFB_EUNSUPPORTED),                                                # row split of a transposed A
    (TWO, _desc(trans_b=1), 0, FAKE, 0, None, _lib.MFB_EUNSUPPORTED),
    ([(0, 60, FAKE, 0), (1, 40, FAKE + 2048, FAKE + 3072)], _desc(), 0, FAKE, 0, None, _lib.MFB_EINVAL),  # null C
    ([(0, 60, 0, FAKE), (1, 40, FAKE + 2048, FAKE + 3072)], _desc(), 0, FAKE, 0, None, _lib.MFB_EINVAL),  # null A
    ([(0, 60, FAKE, FAKE), (1, 40, FAKE + 2048, FAKE + 3072)], _desc(), 0, FAKE, 0, None,
     _lib.MFB_EINVAL),                                                      # C aliases A
    (TWO, _desc(), 0, 0, 0, None, _lib.MFB_EINVAL),                         # null B
    (TWO, _desc(epilogue=1), 0, FAKE, 0, None, _lib.MFB_ESHAPE),            # bias missing
    (TWO, mf.make_desc(100, 64, 32, 16, 64, 64), 0, FAKE, 0, None, _lib.MFB_EINVAL),  # lda < k
])
def test_mfb_sgemm_multi_rejects_bad_arguments(specs, desc, root, b, bias, count, want):
    assert _call(specs, desc, root, b, bias, count) == want
    assert _lib.last_error()
