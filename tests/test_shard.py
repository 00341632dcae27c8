"""Row-sharded multi-GPU path, host side (CPU only: no kernel is launched).

The sharded matmul splits the packed operand by contiguous row ranges and
all-gathers the output rows.  These tests check the partition arithmetic
against the packed layout, and — with two `gloo` ranks on the CPU standing
in for two GPUs, the oracle standing in for the kernels — that shard slices
placed by shard_bounds and all-gathered reproduce the unsharded product
byte for byte, and that the communicator id reaches every rank intact.
"""
import os
import socket

import numpy as np
import pytest

from conftest import FORMATS, gen


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("fmt", FORMATS)
def test_row_bytes_match_packed_layout(fmt):
    import oracle
    import axon_b200 as ax
    F = ax.QuantFormat[fmt]
    for K in (1, 32, 33, 256, 300, 4096, 11008):
        assert ax.row_bytes(K, F) * 7 == oracle.packed_size_2d(fmt, 7, K)


def test_shard_bounds_cover_rows_exactly():
    import axon_b200 as ax
    for M, world in ((28672, 8), (4096, 2), (12, 3), (5, 1)):
        spans = [ax.shard_bounds(M, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == M
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert len({r1 - r0 for r0, r1 in spans}) == 1


def test_shard_bounds_reject_bad_partitions():
    import axon_b200 as ax
    with pytest.raises(ax.AxqError, match="not divisible"):
        ax.shard_bounds(10, 4, 0)
    with pytest.raises(ax.AxqError, match="not in a world"):
        ax.shard_bounds(8, 2, 2)
    with pytest.raises(ax.AxqError, match="expected"):
        ax.shard_rows(np.zeros(10, np.uint8), 4, 32, ax.QuantFormat.Q8_0, 2, 0)


def test_comm_entry_points_reject_bad_arguments_without_a_gpu():
    import ctypes
    import axon_b200 as ax
    L = ax.lib()
    h = ctypes.c_void_p()
    id_buf = ctypes.create_string_buffer(128)
    assert L.axq_comm_unique_id(id_buf, 16) == ax.Status.ERR_INVALID
    assert L.axq_comm_init(ctypes.byref(h), id_buf, 128, 2, 2) == ax.Status.ERR_INVALID
    assert L.axq_comm_init(ctypes.byref(h), id_buf, 64, 2, 0) == ax.Status.ERR_INVALID
    assert L.axq_matmul_sharded(None, 5, None, None, None, 8, 256, 1, 0, None, 0, None) == ax.Status.ERR_INVALID
    assert b"communicator" in L.axq_last_error()
    assert L.axq_allgather(None, None, 4, None) == ax.Status.ERR_INVALID
    assert L.axq_comm_inject_failure(None, 0) == ax.Status.ERR_INVALID
    assert L.axq_comm_check(None) == ax.Status.ERR_INVALID
    assert L.axq_comm_destroy(None) == 0 and L.axq_comm_abort(None) == 0


def test_unique_ids_are_fresh():
    import axon_b200 as ax
    a, b = ax.Communicator.unique_id(), ax.Communicator.unique_id()
    assert len(a) == len(b) == 128 and a != b


# ---- two gloo ranks -------------------------------------------------------

def _sharded_worker(rank, world, port, fmt, M, K, N, q_full, b, result_dir):
    import torch
    import torch.distributed as dist
    import oracle
    import axon_b200 as ax
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # the id exchange the GPU path uses, over this process group
        comm_id = ax.shard.exchange_comm_id()
        ids = [None] * world
        dist.all_gather_object(ids, comm_id)
        assert all(i == comm_id for i in ids)

        F = ax.QuantFormat[fmt]
        local = ax.shard_rows(q_full, M, K, F, world, rank)
        r0, r1 = ax.shard_bounds(M, world, rank)
        out = torch.zeros(M * N, dtype=torch.float32)
        y_local = oracle.orc().matmul(fmt, np.ascontiguousarray(local), b, r1 - r0, K)
        out[r0 * N:r1 * N] = torch.from_numpy(y_local.reshape(-1))
        # in-place all-gather, as axq_allgather does: rank r's part at r*count
        parts = list(out.view(world, -1).unbind(0))
        dist.all_gather(parts, parts[rank].clone())
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.view(M, N).numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt,M,K,N", [("Q5_K", 64, 512, 3), ("Q4_0", 48, 96, 1), ("Q2_K", 32, 300, 17)])
def test_two_rank_sharded_product_equals_unsharded(orc, tmp_path, fmt, M, K, N):
    import torch.multiprocessing as mp
    rng = np.random.default_rng(M + K + N)
    q_full = orc.quantize(fmt, gen(rng, (M, K), "outlier"))
    b = rng.standard_normal((K, N)).astype(np.float32)
    world = 2
    mp.start_processes(_sharded_worker, args=(world, _free_port(), fmt, M, K, N, q_full, b, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    y_ref = orc.matmul(fmt, q_full, b, M, K)
    for r in range(world):
        y = np.load(tmp_path / f"out{r}.npy")
        # rows are independent in every format, so sharding changes no bit
        assert np.array_equal(y.view(np.uint32), y_ref.view(np.uint32))
