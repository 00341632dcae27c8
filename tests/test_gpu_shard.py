"""Row-sharded matmul through the C ABI on the GPU.

One GPU: a one-rank communicator (axq_matmul_sharded then equals
axq_matmul), failure injection and error checks.  Two or more GPUs: the
parity run of tests/sharded_worker.py under torch.distributed.run, one
process per GPU, every rank's gathered output checked against the oracle.
"""
import json
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT, gen, rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max|y - y_ref| <= TOL * max|y_ref|, the matmul parity rule


@pytest.fixture(scope="module")
def comm1(cuda):
    import axon_b200 as ax
    c = ax.Communicator.create(ax.Communicator.unique_id(), 1, 0)
    yield c
    c.destroy()


@pytest.mark.parametrize("fmt,M,K,N", [("Q5_K", 256, 4096, 1), ("Q3_K", 128, 2048, 8), ("Q4_K", 256, 2048, 32)])
def test_one_rank_sharded_equals_matmul_and_oracle(orc, comm1, fmt, M, K, N):
    import torch
    import axon_b200 as ax
    rng = np.random.default_rng(M * N + K)
    q = orc.quantize(fmt, gen(rng, (M, K), "randn"))
    b = rng.standard_normal((K, N)).astype(np.float32)
    F = ax.QuantFormat[fmt]
    a = ax.QTensor(torch.from_numpy(q).cuda(), (M, K), F)
    bd = torch.from_numpy(b).cuda()
    out = torch.full((M, N), float("nan"), device="cuda")
    ax.matmul_sharded(out, a, bd, comm1, M)
    ref_out = torch.full((M, N), float("nan"), device="cuda")
    ax.matmul_q(ref_out, a, bd)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    assert rel_err(out.cpu().numpy(), orc.matmul(fmt, q, b, M, K)) <= TOL


def test_injected_failure_is_reported_and_comm_stays_usable(comm1):
    import torch
    import axon_b200 as ax
    buf = torch.arange(16, dtype=torch.float32, device="cuda")
    comm1.inject_failure(1)
    ax.allgather_(buf, comm1)  # collective 0 runs
    with pytest.raises(ax.AxqError) as e:
        ax.allgather_(buf, comm1)  # collective 1 fails on the host
    assert e.value.status == ax.Status.ERR_COMM and "injected" in str(e.value)
    ax.allgather_(buf, comm1)
    torch.cuda.synchronize()
    comm1.check()
    assert torch.equal(buf.cpu(), torch.arange(16, dtype=torch.float32))


def test_sharded_argument_errors(comm1):
    import torch
    import axon_b200 as ax
    L = ax.lib()
    st = L.axq_matmul_sharded(comm1.handle, 5, None, None, None, 8, 256, 1, ax.FLAG_OUT_TOKMAJOR, None, 0, None)
    assert st == ax.Status.ERR_UNSUPPORTED
    a = ax.QTensor.empty(8, 256, ax.QuantFormat.Q5_K, device="cuda")
    with pytest.raises(ax.AxqError, match="local shard"):
        ax.matmul_sharded(torch.empty(16, 1, device="cuda"), a, torch.empty(256, 1, device="cuda"), comm1, 16)


def test_one_rank_peer_store_async_and_wait(orc, comm1):
    """The peer-store path on one rank (its only peer is itself): calls on two
    buffers issued back to back, then both waits, three times over; a second
    call on a buffer whose wait is outstanding is refused on the host."""
    import torch
    import axon_b200 as ax
    rng = np.random.default_rng(5)
    cases = []
    for fmt, M, K, N in [("Q2_K", 272, 2048, 1), ("Q6_K", 96, 1024, 4)]:
        q = orc.quantize(fmt, gen(rng, (M, K), "randn"))
        b = rng.standard_normal((K, N)).astype(np.float32)
        a = ax.QTensor(torch.from_numpy(q).cuda(), (M, K), ax.QuantFormat[fmt])
        cases.append((a, torch.from_numpy(b).cuda(), M, N, orc.matmul(fmt, q, b, M, K)))
    bufs = [ax.SymmetricBuffer(comm1, 4 * M * N) for _, _, M, N, _ in cases]
    try:
        for it in range(3):
            for (a, bd, M, N, _), buf in zip(cases, bufs):
                buf.tensor((M, N)).fill_(float("nan"))
                ax.matmul_sharded_p2p(buf, a, bd, M, wait=False)
            a, bd, M, _, _ = cases[0]
            with pytest.raises(ax.AxqError, match="axq_symm_wait first") as e:
                ax.matmul_sharded_p2p(bufs[0], a, bd, M, wait=False)
            assert e.value.status == ax.Status.ERR_INVALID
            if it == 1:
                ax.wait_all(bufs)  # both waits in one launch
            else:
                for buf in bufs:
                    buf.wait()
            for buf in bufs:
                buf.wait()  # nothing outstanding: a no-op
            torch.cuda.synchronize()
            for (_, _, M, N, y_ref), buf in zip(cases, bufs):
                assert rel_err(buf.tensor((M, N)).cpu().numpy(), y_ref) <= TOL
    finally:
        torch.cuda.synchronize()
        for buf in bufs:
            buf.destroy()


def test_one_rank_peer_waits_run_out_and_context_survives(orc, comm1):
    """Failure detection without a GPU fault: between a call and its wait the
    buffer's call count is advanced by hand, so the wait (peer_wait_kernel)
    looks for landing slots tagged with a call number no rank ever stores,
    gives up on its own one-second bound and reports through the call's
    workspace status word.  The context stays usable: a plain matmul and a
    fresh symmetric buffer still give the oracle's result."""
    import time
    import torch
    import axon_b200 as ax
    from axon_b200.shard import _CudaArray
    fmt, M, K, N = "Q4_K", 64, 1024, 1
    rng = np.random.default_rng(17)
    q = orc.quantize(fmt, gen(rng, (M, K), "randn"))
    b = rng.standard_normal((K, N)).astype(np.float32)
    y_ref = orc.matmul(fmt, q, b, M, K)
    a = ax.QTensor(torch.from_numpy(q).cuda(), (M, K), ax.QuantFormat[fmt])
    bd = torch.from_numpy(b).cuda()
    ws = ax.Workspace()
    buf = ax.SymmetricBuffer(comm1, 4 * M * N)
    try:
        assert rel_err(ax.matmul_sharded_p2p(buf, a, bd, M, workspace=ws).cpu().numpy(), y_ref) <= TOL
        # control block after the output (rounded up to 256 bytes) and its two
        # landing copies (8 bytes per output value each), one 128-byte line
        # each: call count, finished wait blocks
        data_bytes = -(-buf.nbytes // 256) * 256
        calls = torch.as_tensor(_CudaArray(buf.ptr + 5 * data_bytes, (1,), "<i4"), device="cuda")
        ax.matmul_sharded_p2p(buf, a, bd, M, workspace=ws, wait=False)  # stores call 2's tags
        torch.cuda.synchronize()
        calls += 1  # the wait now expects call 3
        torch.cuda.synchronize()
        t0 = time.time()
        buf.wait()
        wp = ws.get(1, bd.device).data_ptr()
        wp += (-wp) % 256
        with pytest.raises(ax.AxqError) as e:
            ax.workspace_status(wp)
        elapsed = time.time() - t0
        assert e.value.status == ax.Status.ERR_TIMEOUT
        assert 1.0 <= elapsed < 60.0, elapsed
    finally:
        torch.cuda.synchronize()
        buf.destroy()
    out = torch.full((M, N), float("nan"), device="cuda")
    ax.matmul_q(out, a, bd)
    torch.cuda.synchronize()
    assert rel_err(out.cpu().numpy(), y_ref) <= TOL
    fresh = ax.SymmetricBuffer(comm1, 4 * M * N)
    try:
        assert rel_err(ax.matmul_sharded_p2p(fresh, a, bd, M, workspace=ws).cpu().numpy(), y_ref) <= TOL
        ax.workspace_status(wp)
    finally:
        torch.cuda.synchronize()
        fresh.destroy()


def test_destroyed_communicator_is_refused(cuda):
    import axon_b200 as ax
    c = ax.Communicator.create(ax.Communicator.unique_id(), 1, 0)
    c.destroy()
    with pytest.raises(ax.AxqError, match="destroyed"):
        c.check()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_multi_gpu_sharded_parity(cuda, tmp_path, ranks):
    import torch
    if torch.cuda.device_count() < ranks:
        pytest.skip(f"needs {ranks} GPUs, have {torch.cuda.device_count()}")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={ranks}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "sharded_worker.py"), str(tmp_path)]
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    import axon_b200 as ax
    for rank in range(ranks):
        rep = json.load(open(tmp_path / f"rank{rank}.json"))
        for c in rep["cases"]:
            assert c["err"] <= TOL and c["err_tokmajor"] <= TOL, c
        assert len(rep["p2p"]) == 7
        for c in rep["p2p"]:
            assert all(e <= TOL for e in c["errs"]), c
        assert len(rep["p2p_async"]) == 2 and all(e <= TOL for errs in rep["p2p_async"] for e in errs), rep
        assert rep["p2p_refused"] == ax.Status.ERR_INVALID
        assert rep["injected"][0] == ax.Status.ERR_COMM, rep["injected"]
        assert rep["allgather_ok"] and rep["check_ok"]
        assert rep.get("wrong_device_status") == ax.Status.ERR_INVALID
