"""axq_matmul_noalloc: the matmul entry point that allocates nothing.

Callers behind Axon's KernelRegistry receive only their tensors (no
allocator handle), and C hosts that own all device memory may forbid
cudaMalloc, so they cannot supply axq_matmul's workspace.  This entry point
runs the same kernels on a scratch array built into the library.  Here it is
called through the C ABI and compared with axq_matmul (caller workspace) and
with the CPU oracle on two consecutive calls each, for a GEMV-sized and a
GEMM-sized problem; its status word (axq_noalloc_status) reads success after
each call, and its size limit is checked.  This file is named so that pytest
collects it last.
"""
import ctypes

import numpy as np
import pytest

from conftest import gen, rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max-abs difference relative to max|reference output|, as in the matmul parity tests


def _run_both(orc, fmt, M, K, N, seed):
    import torch
    import axon_b200 as ax
    L = ax.lib()
    F = int(ax.QuantFormat[fmt])
    rng = np.random.default_rng(seed)
    q = torch.from_numpy(orc.quantize(fmt, gen(rng, (M, K), "randn"))).cuda()
    b = torch.from_numpy(rng.standard_normal((K, N)).astype(np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    need = L.axq_matmul_workspace_size(F, M, K, N)
    ws = torch.empty(need + 256, dtype=torch.uint8, device="cuda")
    wp = ws.data_ptr() + ((-ws.data_ptr()) % 256)
    ref_out = torch.full((M, N), float("nan"), device="cuda")
    assert L.axq_matmul(F, q.data_ptr(), b.data_ptr(), ref_out.data_ptr(), M, K, N, 0, wp, need, stream) == 0, \
        L.axq_last_error()
    outs = []
    for _ in range(2):  # two calls in a row on the shared scratch
        out = torch.full((M, N), float("nan"), device="cuda")
        st = L.axq_matmul_noalloc(F, q.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N, 0, stream)
        assert st == 0, L.axq_last_error()
        assert L.axq_noalloc_status(stream) == 0, L.axq_last_error()  # no bounded wait gave up
        outs.append(out)
    torch.cuda.synchronize()
    y_orc = orc.matmul(fmt, q.cpu().numpy(), b.cpu().numpy(), M, K)
    return ref_out.cpu().numpy(), [o.cpu().numpy() for o in outs], y_orc


@pytest.mark.parametrize("fmt", ["Q4_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("M,K,N", [(96, 4096, 1), (256, 2048, 64)])
def test_noalloc_matches_workspace_entry_point(cuda, orc, fmt, M, K, N):
    ref_out, outs, y_orc = _run_both(orc, fmt, M, K, N, seed=M + N)
    for y in outs:
        assert np.isfinite(y).all()
        assert rel_err(y, ref_out) <= TOL
        assert rel_err(y, y_orc) <= TOL


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda):
    import axon_b200 as ax
    L = ax.lib()
    F = int(ax.QuantFormat.Q4_K)
    M, K, N = 4096, 65536, 512  # needs far more than the built-in scratch
    assert L.axq_matmul_workspace_size(F, M, K, N) > (16 << 20)
    dummy = ctypes.c_void_p(1)  # never dereferenced: the size check comes first
    st = L.axq_matmul_noalloc(F, dummy, dummy, dummy, M, K, N, 0, None)
    assert st == ax.Status.ERR_WORKSPACE
    assert b"built-in scratch" in L.axq_last_error()
