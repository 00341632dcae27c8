import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

FORMATS = ["Q8_0", "Q4_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.orc()


@pytest.fixture(scope="session")
def ref():
    import oracle
    return oracle.ref()


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    import axon_b200
    axon_b200.lib()
    return torch.device("cuda:0")


def gen(rng, shape, kind):
    """Seeded synthetic inputs with the workload distributions."""
    if kind == "sweep":  # N(0,1) mixed with 1% U(-50,50)
        x = rng.standard_normal(shape).astype(np.float32)
        m = rng.random(shape) < 0.01
        x[m] = rng.uniform(-50, 50, int(m.sum())).astype(np.float32)
        return x
    if kind == "w002":  # N(0, 0.02^2)
        return (rng.standard_normal(shape) * 0.02).astype(np.float32)
    if kind == "outlier":  # N(0,0.02^2) + 0.1% N(0,0.5^2)
        x = (rng.standard_normal(shape) * 0.02).astype(np.float32)
        m = rng.random(shape) < 0.001
        x[m] = (rng.standard_normal(int(m.sum())) * 0.5).astype(np.float32)
        return x
    if kind == "randn":
        return rng.standard_normal(shape).astype(np.float32)
    raise ValueError(kind)


def rel_err(y, y_ref):
    """max|y - y_ref| / max|y_ref| (0 when both are exactly zero)."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    den = np.abs(y_ref).max() if y_ref.size else 0.0
    num = np.abs(y - y_ref).max() if y_ref.size else 0.0
    if den == 0.0:
        return 0.0 if num == 0.0 else float("inf")
    return num / den
