"""Host threads calling the library at once: each thread runs matmuls with
a different token count (so a different kernel and shared-memory plan) on
its own stream and workspace; every result matches the oracle.  ctypes
releases the GIL during the calls, so the library's host code (launch
set-up, per-device caches) really runs concurrently."""
import threading

import numpy as np
import pytest
import torch

from conftest import gen, rel_err

pytestmark = pytest.mark.gpu


def test_concurrent_host_threads(cuda, orc):
    import axon_b200 as ax
    rng = np.random.default_rng(31)
    cases = []
    for fmt, N in (("Q4_K", 1), ("Q6_K", 2), ("Q2_K", 4), ("Q5_K", 16)):
        q = orc.quantize(fmt, gen(rng, (256, 2048), "randn"))
        x = rng.standard_normal((N, 2048)).astype(np.float32)
        cases.append((fmt, q, x, orc.matmul(fmt, q, np.ascontiguousarray(x.T), 256, 2048).T))
    errs = [None] * len(cases)
    barrier = threading.Barrier(len(cases))

    def work(i):
        fmt, q, x, y_ref = cases[i]
        stream = torch.cuda.Stream()
        ws = ax.Workspace()
        with torch.cuda.stream(stream):
            w = ax.QTensor(torch.from_numpy(q).cuda(), (256, 2048), ax.QuantFormat[fmt])
            xd = torch.from_numpy(x).cuda()
            barrier.wait()
            worst = 0.0
            for _ in range(20):
                y = ax.linear_q(xd, w, workspace=ws, stream=stream)
                stream.synchronize()
                worst = max(worst, rel_err(y.cpu().numpy(), y_ref))
        errs[i] = worst

    threads = [threading.Thread(target=work, args=(i,)) for i in range(len(cases))]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert all(e is not None and e <= 1e-3 for e in errs), errs
