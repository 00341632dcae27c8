"""DeviceTensor::randn's sequence (the C++ mirror, libaxon_cuda.so) against
the reference's Tensor::randn (tensor.cpp:36-47, compiled into oracle/_ref):
the same values, bit for bit, over a series of calls of different sizes
(each call a fresh normal distribution over one process-wide generator)."""
import ctypes
import os

import numpy as np
import pytest

from conftest import ROOT


def test_randn_sequence_matches_reference():
    import oracle
    ref = oracle.ref()
    if ref is None:
        pytest.skip("reference library not built here")
    mine = ctypes.CDLL(os.path.join(ROOT, "axon_b200", "libaxon_cuda.so"))
    mine.axon_cuda_randn_fill.argtypes = [ctypes.c_void_p, ctypes.c_size_t]
    ref.lib.ref_randn.argtypes = [ctypes.c_int64, ctypes.c_void_p]
    for n in (1000, 333, 1, 4097):
        a = np.zeros(n, dtype=np.float32)
        b = np.zeros(n, dtype=np.float32)
        mine.axon_cuda_randn_fill(a.ctypes.data, n)
        ref.lib.ref_randn(n, b.ctypes.data)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), n
