"""One rank of the multi-GPU sharded-matmul test (launched by
tests/test_gpu_shard.py under torch.distributed.run, one process per GPU).

Every rank builds the same seeded operands, keeps only its row shard of the
packed weights, runs axq_matmul_sharded through the Python API and checks
the full gathered output against the oracle.  Failure injection is armed on
every rank for the same collective, so no rank is left waiting in NCCL for a
peer.  Results go to <outdir>/rank<r>.json.
"""
import datetime
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

TOL = 1e-3  # max|y - y_ref| <= TOL * max|y_ref|, the matmul parity rule

CASES = [("Q5_K", 1024, 4096, 1), ("Q4_0", 512, 2048, 3), ("Q6_K", 512, 1024, 64), ("Q2_K", 1024, 2048, 16)]
# peer-store GEMV cases (N <= 4), including a row count that is not a
# multiple of the 16-row unit per rank
P2P_CASES = [("Q3_K", 2048, 2048, 1), ("Q4_K", 1040, 1024, 4), ("Q8_0", 96, 512, 2)]


def main(outdir):
    import torch
    import torch.distributed as dist
    import oracle
    import axon_b200 as ax
    from conftest import gen, rel_err

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    report = {"rank": rank, "world": world, "cases": []}
    comm = ax.Communicator.from_process_group()
    try:
        orc = oracle.orc()
        for fmt, M, K, N in CASES:
            rng = np.random.default_rng(M + K + N)  # same on every rank
            q_full = orc.quantize(fmt, gen(rng, (M, K), "randn"))
            b = rng.standard_normal((K, N)).astype(np.float32)
            F = ax.QuantFormat[fmt]
            local_q = ax.shard_rows(q_full, M, K, F, world, rank)
            a = ax.QTensor(torch.from_numpy(np.ascontiguousarray(local_q)).to(dev), (M // world, K), F)
            bd = torch.from_numpy(b).to(dev)
            out = torch.full((M, N), float("nan"), device=dev)
            ax.matmul_sharded(out, a, bd, comm, M)
            # token-major activations give the same product
            out_t = torch.full((M, N), float("nan"), device=dev)
            ax.matmul_sharded(out_t, a, bd.t().contiguous(), comm, M, b_tokmajor=True)
            torch.cuda.synchronize()
            y_ref = orc.matmul(fmt, q_full, b, M, K)
            report["cases"].append({"case": [fmt, M, K, N], "err": rel_err(out.cpu().numpy(), y_ref),
                                    "err_tokmajor": rel_err(out_t.cpu().numpy(), y_ref)})

        # peer-store path: outputs written straight into every rank's copy of
        # a symmetric buffer by the GEMV epilogue (N <= 4), NCCL otherwise;
        # two calls back to back, then one captured in a CUDA graph and replayed
        buf = ax.SymmetricBuffer(comm, 4 * max(M * N for _, M, _, N in CASES + P2P_CASES))
        report["p2p"] = []
        for fmt, M, K, N in P2P_CASES + CASES:
            rng = np.random.default_rng(M + K + N + 1)
            q_full = orc.quantize(fmt, gen(rng, (M, K), "randn"))
            b = rng.standard_normal((K, N)).astype(np.float32)
            F = ax.QuantFormat[fmt]
            a = ax.QTensor(torch.from_numpy(np.ascontiguousarray(ax.shard_rows(q_full, M, K, F, world, rank))).to(dev),
                           (M // world, K), F)
            bd = torch.from_numpy(b).to(dev)
            y_ref = orc.matmul(fmt, q_full, b, M, K)
            errs = []
            y = ax.matmul_sharded_p2p(buf, a, bd, M)
            torch.cuda.synchronize()
            errs.append(rel_err(y.cpu().numpy(), y_ref))
            buf.tensor((M, N)).fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()  # every rank cleared before the next call writes
            for _ in range(2):  # back to back: the entry handshake orders the writes
                y = ax.matmul_sharded_p2p(buf, a, bd, M)
            torch.cuda.synchronize()
            errs.append(rel_err(y.cpu().numpy(), y_ref))
            dist.barrier()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                ax.matmul_sharded_p2p(buf, a, bd, M)
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            errs.append(rel_err(buf.tensor((M, N)).cpu().numpy(), y_ref))
            del g
            report["p2p"].append({"case": [fmt, M, K, N], "errs": errs})
        torch.cuda.synchronize()
        dist.barrier()

        # split issue and wait: two buffers' calls back to back, then both
        # waits; a second call on a buffer with one outstanding is refused
        buf2 = ax.SymmetricBuffer(comm, buf.nbytes)
        report["p2p_async"] = []
        ops = []
        for fmt, M, K, N in P2P_CASES[:2]:
            rng = np.random.default_rng(M + K + N + 2)
            q_full = orc.quantize(fmt, gen(rng, (M, K), "randn"))
            b = rng.standard_normal((N, K)).astype(np.float32)  # token-major
            F = ax.QuantFormat[fmt]
            a = ax.QTensor(torch.from_numpy(np.ascontiguousarray(ax.shard_rows(q_full, M, K, F, world, rank))).to(dev),
                           (M // world, K), F)
            ops.append((a, torch.from_numpy(b).to(dev), M, N, orc.matmul(fmt, q_full, np.ascontiguousarray(b.T), M, K)))
        for it in range(2):
            for (a, bd, M, N, _), bb in zip(ops, (buf, buf2)):
                ax.matmul_sharded_p2p(bb, a, bd, M, b_tokmajor=True, wait=False)
            try:
                ax.matmul_sharded_p2p(buf, ops[0][0], ops[0][1], ops[0][2], b_tokmajor=True, wait=False)
                report["p2p_refused"] = None
            except ax.AxqError as e:
                report["p2p_refused"] = int(e.status)
            if it == 0:
                buf.wait()
                buf2.wait()
            else:
                ax.wait_all([buf, buf2])  # both waits in one launch
            torch.cuda.synchronize()
            report["p2p_async"].append([rel_err(bb.tensor((M, N)).cpu().numpy(), y_ref)
                                        for (_, _, M, N, y_ref), bb in zip(ops, (buf, buf2))])
            dist.barrier()
        torch.cuda.synchronize()
        dist.barrier()
        buf.destroy()
        buf2.destroy()

        # host-side failure injection, armed on every rank for the next collective
        comm.inject_failure(0)
        fmt, M, K, N = CASES[0]
        a = ax.QTensor(torch.zeros(ax.quantized_size_2d(M // world, K, ax.QuantFormat[fmt]), dtype=torch.uint8,
                                   device=dev), (M // world, K), ax.QuantFormat[fmt])
        out = torch.zeros(M, N, device=dev)
        try:
            ax.matmul_sharded(out, a, torch.zeros(K, N, device=dev), comm, M)
            report["injected"] = "no error"
        except ax.AxqError as e:
            report["injected"] = [int(e.status), str(e)]
        # the communicator stays usable after an injected failure
        buf = torch.arange(world * 8, dtype=torch.float32, device=dev)
        mine = buf[rank * 8:(rank + 1) * 8].clone()
        buf.zero_()
        buf[rank * 8:(rank + 1) * 8] = mine
        ax.allgather_(buf, comm)
        torch.cuda.synchronize()
        report["allgather_ok"] = bool(torch.equal(buf.cpu(), torch.arange(world * 8, dtype=torch.float32)))
        comm.check()
        report["check_ok"] = True

        # a call from the wrong device is refused before any launch
        if torch.cuda.device_count() > 1:
            other = (local + 1) % torch.cuda.device_count()
            with torch.cuda.device(other):
                st = ax.lib().axq_matmul_sharded(comm.handle, 5, None, None, None, M, K, N, 0, None, 0, None)
            report["wrong_device_status"] = int(st)
    finally:
        torch.cuda.synchronize()
        comm.destroy()
        dist.barrier()
        dist.destroy_process_group()
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(report, f)


if __name__ == "__main__":
    main(sys.argv[1])
