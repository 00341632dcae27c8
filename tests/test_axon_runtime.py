"""The reference's own Runtime::matmul / cpu::quantize / cpu::dequantize on
Device::CUDA tensors, through its own KernelRegistry, into this library's
kernels: the reference compiled with axon_b200/integration/axon_device.patch
plus axon_b200/integration/cuda_backend.cpp (built where the reference's
sources are available, `make -C axon_b200/integration REF=...`), driven by
tests/cpp/axon_runtime_test.cpp against the same library's CPU path."""
import os
import subprocess

import pytest

from conftest import ROOT

EXE = os.path.join(ROOT, "axon_b200", "integration", "_build", "axon_runtime_test")


def _exe():
    if not os.path.exists(EXE):
        pytest.skip("integration build absent: the reference's sources were not available when building")
    return EXE


def test_registration_and_refusals_without_gpu():
    r = subprocess.run([_exe(), "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


@pytest.mark.gpu
def test_runtime_matmul_on_cuda_tensors(cuda):
    r = subprocess.run([_exe()], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout
