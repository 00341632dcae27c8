"""B200 (sm_100a) implementation of Axon's block-quantized matmul path.

This package is the Python host side of ``libaxq.so`` (C ABI declared in
``include/axq.h``).  Its functions mirror the reference's CPU backend entry
points (ruwwww/Axon ``include/axon/backend/cpu_backend.h:36-46``) with the
same names, argument meaning and error behaviour: ``quantize``,
``dequantize``, ``matmul_q4`` / ``matmul_q2_K`` / ... plus the generic
``matmul_q`` and the size helpers.  Tensors are torch CUDA tensors used as
plain device buffers; every call goes to the CUDA kernels — there is no CPU
path, and importing fails loudly when the library is missing.

Errors: the reference returns ``Expected<void>`` holding ``Error{message}``;
here a failed call raises :class:`AxqError` carrying the library's status
code and message.
"""
from __future__ import annotations

from ._capi import (  # noqa: F401
    AxqError,
    FLAG_B_TOKMAJOR,
    FLAG_OUT_TOKMAJOR,
    QuantFormat,
    BLOCK_ELEMS,
    BLOCK_BYTES,
    Status,
    lib,
    lib_path,
    quantized_size,
    quantized_size_2d,
    matmul_workspace_size,
    workspace_status,
)
from .ops import (  # noqa: F401
    QTensor,
    Workspace,
    quantize,
    dequantize,
    matmul,
    matmul_q,
    matmul_q8_0,
    matmul_q4,
    matmul_q2_K,
    matmul_q3_K,
    matmul_q4_K,
    matmul_q5_K,
    matmul_q6_K,
    linear_q,
    gate_up_silu,
    mlp_q,
)
from .axon_file import (  # noqa: F401
    AxonRecord,
    axon_records,
    load_axon,
    load_tensor,
    save_axon,
    save_tensor,
)
from .shard import (  # noqa: F401
    Communicator,
    SymmetricBuffer,
    matmul_sharded_p2p,
    wait_all,
    allgather_,
    matmul_sharded,
    row_bytes,
    shard_bounds,
    shard_rows,
)

__all__ = [
    "AxqError", "QuantFormat", "QTensor", "Status", "Workspace", "quantize", "dequantize", "matmul_q",
    "matmul_q8_0", "matmul_q4", "matmul_q2_K", "matmul_q3_K", "matmul_q4_K", "matmul_q5_K", "matmul_q6_K",
    "linear_q", "gate_up_silu", "mlp_q", "quantized_size", "quantized_size_2d", "matmul_workspace_size", "lib", "lib_path",
    "Communicator", "SymmetricBuffer", "matmul_sharded_p2p", "wait_all", "allgather_", "matmul_sharded", "row_bytes", "shard_bounds", "shard_rows",
]
