"""ctypes binding of ``libaxq.so`` (the C ABI in ``include/axq.h``).

The library is built in-tree (``make -C axon_b200``) and loaded from this
package directory only; a missing library is an ImportError-class failure,
never a silent fallback.
"""
from __future__ import annotations

import ctypes
import enum
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_NAME = "libaxq.so"

FLAG_B_TOKMAJOR = 1
FLAG_OUT_TOKMAJOR = 2


class QuantFormat(enum.IntEnum):
    """The reference's QuantFormat (include/axon/core/types.h:36-45); the
    ordinals are the C ABI's format ids."""

    NONE = 0
    Q8_0 = 1
    Q6_K = 2
    Q5_K = 3
    Q4_0 = 4
    Q4_K = 5
    Q3_K = 6
    Q2_K = 7


BLOCK_ELEMS = {QuantFormat.Q8_0: 32, QuantFormat.Q4_0: 32, QuantFormat.Q2_K: 256, QuantFormat.Q3_K: 256,
               QuantFormat.Q4_K: 256, QuantFormat.Q5_K: 256, QuantFormat.Q6_K: 256}
BLOCK_BYTES = {QuantFormat.Q8_0: 34, QuantFormat.Q4_0: 18, QuantFormat.Q2_K: 84, QuantFormat.Q3_K: 110,
               QuantFormat.Q4_K: 144, QuantFormat.Q5_K: 176, QuantFormat.Q6_K: 210}


class Status(enum.IntEnum):
    OK = 0
    ERR_INVALID = 1
    ERR_UNSUPPORTED = 2
    ERR_CUDA = 3
    ERR_WORKSPACE = 4
    ERR_TIMEOUT = 5
    ERR_COMM = 6


class AxqError(RuntimeError):
    """A failed library call: ``status`` is the C ABI code, the message is
    the library's (the reference's ``Error{message}``)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = Status(status) if status in Status._value2member_map_ else status


# Every symbol include/axq.h declares, with its ctypes signature.
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
SIGNATURES = {
    "axq_last_error": (ctypes.c_char_p, []),
    "axq_version": (ctypes.c_int, []),
    "axq_quantized_size": (_sz, [_sz, ctypes.c_int]),
    "axq_quantized_size_2d": (_sz, [_i64, _i64, ctypes.c_int]),
    "axq_quantize": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _i64, _i64, _vp]),
    "axq_dequantize": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _i64, _i64, _vp]),
    "axq_matmul_workspace_size": (_sz, [ctypes.c_int, _i64, _i64, _i64]),
    "axq_matmul": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_uint, _vp, _sz, _vp]),
    "axq_workspace_status": (ctypes.c_int, [_vp, _vp]),
    "axq_linear": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, ctypes.c_size_t, _vp]),
    "axq_matmul_noalloc": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_uint, _vp]),
    "axq_noalloc_status": (ctypes.c_int, [_vp]),
    "axq_gate_up_workspace_size": (_sz, [ctypes.c_int, _i64, _i64, _i64]),
    "axq_gate_up_silu": (ctypes.c_int, [ctypes.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_uint, _vp, _sz,
                                        _vp]),
    "axq_comm_unique_id": (ctypes.c_int, [_vp, _sz]),
    "axq_comm_init": (ctypes.c_int, [ctypes.POINTER(_vp), _vp, _sz, ctypes.c_int, ctypes.c_int]),
    "axq_comm_init_all": (ctypes.c_int, [ctypes.POINTER(_vp), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]),
    "axq_group_start": (ctypes.c_int, []),
    "axq_group_end": (ctypes.c_int, []),
    "axq_comm_destroy": (ctypes.c_int, [_vp]),
    "axq_comm_abort": (ctypes.c_int, [_vp]),
    "axq_comm_check": (ctypes.c_int, [_vp]),
    "axq_comm_inject_failure": (ctypes.c_int, [_vp, _i64]),
    "axq_allgather": (ctypes.c_int, [_vp, _vp, _sz, _vp]),
    "axq_matmul_sharded": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_uint, _vp,
                                          _sz, _vp]),
    "axq_symm_create": (ctypes.c_int, [_vp, _sz, ctypes.POINTER(_vp), ctypes.POINTER(_vp)]),
    "axq_symm_destroy": (ctypes.c_int, [_vp]),
    "axq_matmul_sharded_p2p": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _i64, _i64, _i64, ctypes.c_uint, _vp, _sz,
                                              _vp]),
    "axq_matmul_sharded_p2p_async": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _i64, _i64, _i64, ctypes.c_uint, _vp,
                                                    _sz, _vp]),
    "axq_symm_wait_many": (ctypes.c_int, [_vp, ctypes.c_int, _vp]),
    "axq_symm_wait": (ctypes.c_int, [_vp, _vp]),
    "axq_matmul_f32": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "axq_axon_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(_vp), ctypes.POINTER(ctypes.c_uint32)]),
    "axq_axon_info": (ctypes.c_int, [_vp, ctypes.c_uint32, _vp]),
    "axq_axon_read": (ctypes.c_int, [_vp, ctypes.c_uint32, _vp, _sz, _vp]),
    "axq_axon_close": (ctypes.c_int, [_vp]),
    "axq_axon_save": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_uint32, _vp, _vp, _vp]),
}

AXON_MAX_DIMS = 8
AXON_NAME_BYTES = 256
AXON_PLAIN, AXON_ROWS, AXON_FLAT = 0, 1, 2


class AxonTensorInfo(ctypes.Structure):
    """axq_axon_tensor (include/axq.h): one record of an .axon file."""

    _fields_ = [("name", ctypes.c_char * AXON_NAME_BYTES), ("dtype", ctypes.c_uint32), ("quant", ctypes.c_uint32),
                ("ndims", ctypes.c_uint32), ("layout", ctypes.c_uint32), ("shape", ctypes.c_int64 * AXON_MAX_DIMS),
                ("data_bytes", ctypes.c_uint64), ("offset", ctypes.c_uint64)]

COMM_ID_BYTES = 128  # AXQ_COMM_ID_BYTES

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return os.path.join(_HERE, _LIB_NAME)


def lib() -> ctypes.CDLL:
    """The loaded C library (raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                path = lib_path()
                if not os.path.exists(path):
                    raise ImportError(f"{path} is missing: build it with `make -C axon_b200` "
                                      "(there is no CPU fallback)")
                L = ctypes.CDLL(path)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(L, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = lib().axq_last_error().decode("utf-8", "replace")
        raise AxqError(status, msg or f"axq status {status}")


def quantized_size(numel: int, fmt: QuantFormat) -> int:
    """Replaces cpu::quantized_size (src/backend/cpu_backend.cpp:693-711)."""
    return int(lib().axq_quantized_size(numel, int(fmt)))


def quantized_size_2d(rows: int, cols: int, fmt: QuantFormat) -> int:
    """Replaces cpu::quantized_size_2d (src/backend/cpu_backend.cpp:713-735)."""
    return int(lib().axq_quantized_size_2d(rows, cols, int(fmt)))


def matmul_workspace_size(fmt: QuantFormat, M: int, K: int, N: int) -> int:
    return int(lib().axq_matmul_workspace_size(int(fmt), M, K, N))


def workspace_status(ws_ptr: int, stream: int = 0) -> None:
    check(lib().axq_workspace_status(ws_ptr, stream))
