"""Row-sharded multi-GPU quantized matmul over the C ABI.

The reference is a single-process CPU library, so nothing here replaces a
reference function; it extends ``matmul_q*`` (cpu_backend.cpp:1674-2066)
across GPUs the way the format allows.  Each packed row is self-contained —
``cpu::quantize`` packs row by row and blocks never span rows
(cpu_backend.cpp:1174-1185) — so the quantized operand A_q[M x K] shards by
contiguous row ranges with no reduction: rank r of G owns rows
``[r*M/G, (r+1)*M/G)``, holds a full copy of B, computes its rows of the
output in place, and one in-place all-gather (NCCL, inside the library)
completes ``out[M x N]`` on every rank.

One process per GPU: the communicator id travels over an existing
``torch.distributed`` process group (any backend), then the library creates
its own NCCL communicator on the current device.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from ._capi import (
    BLOCK_BYTES,
    BLOCK_ELEMS,
    COMM_ID_BYTES,
    FLAG_B_TOKMAJOR,
    AxqError,
    QuantFormat,
    Status,
    check,
    lib,
)
from .ops import QTensor, Workspace, _aligned_ptr, _default_ws, _req_cuda, _stream_handle


def row_bytes(K: int, fmt: QuantFormat) -> int:
    """Packed bytes of one row of K elements (cpu_backend.cpp:713-735)."""
    fmt = QuantFormat(fmt)
    return -(-K // BLOCK_ELEMS[fmt]) * BLOCK_BYTES[fmt]


def shard_bounds(M: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [r0, r1) of an M-row operand owned by `rank` of `world`; M must
    divide evenly, as axq_matmul_sharded requires."""
    if world < 1 or not 0 <= rank < world:
        raise AxqError(Status.ERR_INVALID, f"rank {rank} is not in a world of {world}")
    if M % world:
        raise AxqError(Status.ERR_INVALID, f"M={M} is not divisible by {world} ranks")
    rows = M // world
    return rank * rows, (rank + 1) * rows


def shard_rows(packed, M: int, K: int, fmt: QuantFormat, world: int, rank: int):
    """This rank's slice of a packed [M x K] operand: a view of the bytes of
    rows shard_bounds(M, world, rank) (works on any 1-D byte buffer that
    slices: torch tensor or numpy array)."""
    r0, r1 = shard_bounds(M, world, rank)
    rb = row_bytes(K, fmt)
    if len(packed) != M * rb:
        raise AxqError(Status.ERR_INVALID, f"packed buffer has {len(packed)} bytes, expected {M * rb}")
    return packed[r0 * rb:r1 * rb]


class Communicator:
    """A library-owned NCCL communicator bound to the current CUDA device."""

    def __init__(self, handle: int, world: int, rank: int):
        self._h = ctypes.c_void_p(handle)
        self.world = world
        self.rank = rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(COMM_ID_BYTES)
        check(lib().axq_comm_unique_id(buf, COMM_ID_BYTES))
        return buf.raw

    @classmethod
    def create(cls, comm_id: bytes, world: int, rank: int) -> "Communicator":
        if len(comm_id) != COMM_ID_BYTES:
            raise AxqError(Status.ERR_INVALID, f"communicator id must be {COMM_ID_BYTES} bytes")
        h = ctypes.c_void_p()
        check(lib().axq_comm_init(ctypes.byref(h), comm_id, COMM_ID_BYTES, world, rank))
        return cls(h.value, world, rank)

    @classmethod
    def from_process_group(cls, group=None) -> "Communicator":
        """Collective over `group`: rank 0 makes the id, every rank joins."""
        comm_id = exchange_comm_id(group)
        import torch.distributed as dist
        return cls.create(comm_id, dist.get_world_size(group), dist.get_rank(group))

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h.value:
            raise AxqError(Status.ERR_INVALID, "communicator was destroyed")
        return self._h

    def check(self) -> None:
        """Raises AxqError(ERR_COMM) if NCCL recorded an asynchronous error."""
        check(lib().axq_comm_check(self.handle))

    def inject_failure(self, collective_index: int = 0) -> None:
        """Make the collective_index-th collective from now fail on the host."""
        check(lib().axq_comm_inject_failure(self.handle, collective_index))

    def destroy(self) -> None:
        if self._h.value:
            h, self._h = self._h, ctypes.c_void_p()
            check(lib().axq_comm_destroy(h))

    def abort(self) -> None:
        if self._h.value:
            h, self._h = self._h, ctypes.c_void_p()
            check(lib().axq_comm_abort(h))

    def __enter__(self):
        return self

    def __exit__(self, exc_type, *_):
        if exc_type is None:
            self.destroy()
        else:
            self.abort()


def exchange_comm_id(group=None) -> bytes:
    """Rank 0 of `group` creates a communicator id and broadcasts it over the
    process group; every rank returns the same bytes."""
    import torch.distributed as dist
    holder = [Communicator.unique_id() if dist.get_rank(group) == 0 else None]
    src = dist.get_global_rank(group, 0) if group is not None else 0
    dist.broadcast_object_list(holder, src=src, group=group)
    comm_id = holder[0]
    if not isinstance(comm_id, bytes) or len(comm_id) != COMM_ID_BYTES:
        raise AxqError(Status.ERR_COMM, "communicator id exchange returned a malformed id")
    return comm_id


def allgather_(buf: torch.Tensor, comm: Communicator, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """In place: rank r's numel/world floats at buf[r*n:(r+1)*n] reach every rank."""
    _req_cuda(buf, "buf", torch.float32)
    if buf.numel() % comm.world:
        raise AxqError(Status.ERR_INVALID, f"buffer of {buf.numel()} floats does not split over {comm.world} ranks")
    check(lib().axq_allgather(comm.handle, buf.data_ptr(), buf.numel() // comm.world, _stream_handle(stream)))
    return buf


def matmul_sharded(out: torch.Tensor, a_local: QTensor, b: torch.Tensor, comm: Communicator, M: int,
                   b_tokmajor: bool = False, workspace: Optional[Workspace] = None,
                   stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """out[M x N] = A_q . B on every rank, where this rank holds rows
    shard_bounds(M, world, rank) of A_q as `a_local` ([M/world x K])."""
    _req_cuda(a_local.data, "a_local.data", torch.uint8)
    _req_cuda(b, "b", torch.float32)
    _req_cuda(out, "out", torch.float32)
    rows, K = a_local.shape
    if rows * comm.world != M:
        raise AxqError(Status.ERR_INVALID, f"local shard has {rows} rows; {comm.world} ranks need M/{comm.world}")
    if b.dim() != 2:
        raise AxqError(Status.ERR_INVALID, "b must be 2-D")
    N = b.shape[0] if b_tokmajor else b.shape[1]
    if (b.shape[1] if b_tokmajor else b.shape[0]) != K:
        raise AxqError(Status.ERR_INVALID, f"b does not have K={K}")
    if tuple(out.shape) != (M, N):
        raise AxqError(Status.ERR_INVALID, f"out must be [{M} x {N}]")
    fmt = int(a_local.fmt)
    need = int(lib().axq_matmul_workspace_size(fmt, rows, K, N))
    ptr, nbytes = _aligned_ptr((workspace or _default_ws).get(need + 256, out.device))
    flags = FLAG_B_TOKMAJOR if b_tokmajor else 0
    check(lib().axq_matmul_sharded(comm.handle, fmt, a_local.data.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N,
                                   flags, ptr, nbytes, _stream_handle(stream)))
    return out


class _CudaArray:
    """__cuda_array_interface__ view of library-owned device memory."""

    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 2, "strides": None}


class SymmetricBuffer:
    """Device memory that every rank of a communicator allocates and maps
    from every other rank (CUDA IPC over NVLink).  Collective to create and
    to destroy; `tensor(shape)` views this rank's copy as fp32."""

    def __init__(self, comm: Communicator, nbytes: int):
        h, p = ctypes.c_void_p(), ctypes.c_void_p()
        check(lib().axq_symm_create(comm.handle, nbytes, ctypes.byref(h), ctypes.byref(p)))
        self._h, self.ptr, self.nbytes, self.comm = h, p.value, nbytes, comm

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h.value:
            raise AxqError(Status.ERR_INVALID, "symmetric buffer was destroyed")
        return self._h

    def tensor(self, shape) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= int(d)
        if 4 * n > self.nbytes:
            raise AxqError(Status.ERR_INVALID, f"view of {n} floats exceeds the buffer's {self.nbytes} bytes")
        return torch.as_tensor(_CudaArray(self.ptr, shape), device=f"cuda:{torch.cuda.current_device()}")

    def wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Enqueue the wait for this buffer's outstanding peer-store call."""
        check(lib().axq_symm_wait(self.handle, _stream_handle(stream)))

    def destroy(self) -> None:
        if self._h.value:
            h, self._h = self._h, ctypes.c_void_p()
            check(lib().axq_symm_destroy(h))


def wait_all(buffers, stream: Optional[torch.cuda.Stream] = None) -> None:
    """Enqueue the waits of several symmetric buffers' outstanding peer-store
    calls as one kernel (axq_symm_wait_many)."""
    bufs = list(buffers)
    if not bufs:
        return
    arr = (ctypes.c_void_p * len(bufs))(*[b.handle.value for b in bufs])
    dev = torch.device("cuda", torch.cuda.current_device())
    check(lib().axq_symm_wait_many(ctypes.cast(arr, ctypes.c_void_p), len(bufs), _stream_handle(stream, dev)))


def matmul_sharded_p2p(out: SymmetricBuffer, a_local: QTensor, b: torch.Tensor, M: int, b_tokmajor: bool = False,
                       workspace: Optional[Workspace] = None, stream: Optional[torch.cuda.Stream] = None,
                       wait: bool = True) -> torch.Tensor:
    """As matmul_sharded, into a symmetric buffer: up to 4 columns store every
    output value into each rank's landing copy from the GEMV epilogue, as a
    slot tagged with the call's number (no separate collective).  Returns this rank's full [M x N] copy.  wait=False
    leaves the completion wait to `out.wait()`, so calls on several buffers
    can be issued back to back."""
    _req_cuda(a_local.data, "a_local.data", torch.uint8)
    _req_cuda(b, "b", torch.float32)
    comm = out.comm
    rows, K = a_local.shape
    if rows * comm.world != M:
        raise AxqError(Status.ERR_INVALID, f"local shard has {rows} rows; {comm.world} ranks need M/{comm.world}")
    if b.dim() != 2 or (b.shape[1] if b_tokmajor else b.shape[0]) != K:
        raise AxqError(Status.ERR_INVALID, f"b must be 2-D with K={K}")
    N = b.shape[0] if b_tokmajor else b.shape[1]
    fmt = int(a_local.fmt)
    need = int(lib().axq_matmul_workspace_size(fmt, rows, K, N))
    ptr, nbytes = _aligned_ptr((workspace or _default_ws).get(need + 256, b.device))
    flags = FLAG_B_TOKMAJOR if b_tokmajor else 0
    fn = lib().axq_matmul_sharded_p2p if wait else lib().axq_matmul_sharded_p2p_async
    check(fn(out.handle, fmt, a_local.data.data_ptr(), b.data_ptr(), M, K, N, flags, ptr, nbytes,
             _stream_handle(stream, b.device)))
    return out.tensor((M, N))
