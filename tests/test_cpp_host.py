"""The C++ host mirror (axon_b200/host/axon_cuda.h): the reference's
KernelRegistry / KernelKey / KernelContext seam and cpu_backend.h front doors
restated for a Device::CUDA backend over the C ABI.

The C++ tests are built here with g++ (C++20, like the reference) and run as
executables: tests/cpp/registry_test.cpp needs no GPU (registration,
dispatch by key and by name, size pins, argument errors);
tests/cpp/quant_cuda_test.cpp runs every format through the mirror on the
GPU against the oracle.
"""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

CPP = os.path.join(ROOT, "tests", "cpp")
BUILD = os.path.join(CPP, "_build")
LIB = os.path.join(ROOT, "axon_b200")
ORC = os.path.join(ROOT, "oracle", "_build")
CUDA = "/usr/local/cuda"


def _cxx():
    return os.environ.get("CXX") or shutil.which("g++") or "g++"


def _build(name, with_oracle):
    src = os.path.join(CPP, name + ".cpp")
    exe = os.path.join(BUILD, name)
    deps = [src, os.path.join(CPP, "check.h"), os.path.join(LIB, "host", "axon_cuda.h"),
            os.path.join(LIB, "libaxon_cuda.so")]
    if os.path.exists(exe) and all(os.path.getmtime(exe) >= os.path.getmtime(d) for d in deps if os.path.exists(d)):
        return exe
    os.makedirs(BUILD, exist_ok=True)
    cmd = [_cxx(), "-std=c++20", "-O1", "-Wall", f"-I{ROOT}/include", f"-I{LIB}/host", f"-I{CUDA}/include",
           src, "-o", exe, f"-L{LIB}", "-laxon_cuda", "-laxq", "-Wl,-rpath,$ORIGIN/../../../axon_b200"]
    if with_oracle:
        cmd[6:6] = [f"-I{ROOT}/oracle"]
        cmd += [f"-L{ORC}", "-lorc", "-Wl,-rpath,$ORIGIN/../../../oracle/_build"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return exe


@pytest.fixture(scope="module")
def host_lib():
    path = os.path.join(LIB, "libaxon_cuda.so")
    assert os.path.exists(path), "build it with `make -C axon_b200`"
    return path


def test_registry_and_front_door_errors(host_lib):
    exe = _build("registry_test", with_oracle=False)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


@pytest.mark.gpu
def test_mirror_matches_oracle_on_gpu(host_lib, cuda):
    exe = _build("quant_cuda_test", with_oracle=True)
    r = subprocess.run([exe, os.path.join(ROOT, "tests", "golden")], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout
