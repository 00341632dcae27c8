"""CPU oracle for the block-quantized matmul path — TEST INFRASTRUCTURE ONLY.

Two checkers live here:

* ``orc``: the plain-C restatement (``axq_oracle.c``) of the reference's CPU
  quantize / dequantize / quantized-matmul loops, built by ``make -C oracle``
  into ``oracle/_build/liborc.so``.
* ``ref``: the reference's own CPU code compiled from its sources by the same
  Makefile into ``oracle/_ref/libaxon_ref.so`` (present only where the
  reference sources were available at build time).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this package; the product (``axon_b200``) never does.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
ORC_PATH = os.path.join(_HERE, "_build", "liborc.so")
REF_PATH = os.path.join(_HERE, "_ref", "libaxon_ref.so")

# Reference QuantFormat ordinals (include/axon/core/types.h:36-45).
FORMATS = {"Q8_0": 1, "Q6_K": 2, "Q5_K": 3, "Q4_0": 4, "Q4_K": 5, "Q3_K": 6, "Q2_K": 7}
BLOCK_ELEMS = {"Q8_0": 32, "Q4_0": 32, "Q2_K": 256, "Q3_K": 256, "Q4_K": 256, "Q5_K": 256, "Q6_K": 256}
BLOCK_BYTES = {"Q8_0": 34, "Q4_0": 18, "Q2_K": 84, "Q3_K": 110, "Q4_K": 144, "Q5_K": 176, "Q6_K": 210}

_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p


def packed_size_2d(fmt: str, rows: int, cols: int) -> int:
    be = BLOCK_ELEMS[fmt]
    return rows * ((cols + be - 1) // be) * BLOCK_BYTES[fmt]


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class _Lib:
    def __init__(self, path: str, prefix: str):
        self.path = path
        self.lib = ctypes.CDLL(path)
        self.prefix = prefix
        for name in ("quantize", "dequantize"):
            fn = getattr(self.lib, f"{prefix}_{name}")
            fn.restype = ctypes.c_int
            fn.argtypes = [ctypes.c_int, _vp, _c_i64, _c_i64, _vp]
        fn = getattr(self.lib, f"{prefix}_matmul")
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_int, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64]

    def quantize(self, fmt: str, x: np.ndarray) -> np.ndarray:
        """Pack a 2-D fp32 array row by row (or a 1-D array as one row)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, cols = (1, x.shape[0]) if x.ndim == 1 else x.shape
        out = np.zeros(packed_size_2d(fmt, rows, cols), dtype=np.uint8)
        rc = getattr(self.lib, f"{self.prefix}_quantize")(FORMATS[fmt], _ptr(x), rows, cols, _ptr(out))
        if rc != 0:
            raise RuntimeError(f"{self.prefix}_quantize failed ({rc})")
        return out

    def dequantize(self, fmt: str, q: np.ndarray, rows: int, cols: int) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.uint8)
        assert q.size >= packed_size_2d(fmt, rows, cols)
        out = np.zeros((rows, cols), dtype=np.float32)
        rc = getattr(self.lib, f"{self.prefix}_dequantize")(FORMATS[fmt], _ptr(q), rows, cols, _ptr(out))
        if rc != 0:
            raise RuntimeError(f"{self.prefix}_dequantize failed ({rc})")
        return out

    def matmul(self, fmt: str, a_q: np.ndarray, b: np.ndarray, M: int, K: int) -> np.ndarray:
        """out[M x N] = A_q[M x K] . B[K x N] (reference orientation)."""
        a_q = np.ascontiguousarray(a_q, dtype=np.uint8)
        b = np.ascontiguousarray(b, dtype=np.float32)
        assert b.shape[0] == K
        N = b.shape[1]
        out = np.zeros((M, N), dtype=np.float32)
        rc = getattr(self.lib, f"{self.prefix}_matmul")(FORMATS[fmt], _ptr(a_q), _ptr(b), _ptr(out), M, K, N)
        if rc != 0:
            raise RuntimeError(f"{self.prefix}_matmul failed ({rc})")
        return out


class Oracle(_Lib):
    """The C restatement."""

    def __init__(self, path: str = ORC_PATH):
        super().__init__(path, "orc")
        self.lib.orc_matmul_f64.restype = ctypes.c_int
        self.lib.orc_matmul_f64.argtypes = [ctypes.c_int, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64]
        self.lib.orc_matmul_rows.restype = ctypes.c_int
        self.lib.orc_matmul_rows.argtypes = [ctypes.c_int, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64,
                                             _c_i64, _c_i64]
        self.lib.orc_float_to_half.restype = ctypes.c_uint16
        self.lib.orc_float_to_half.argtypes = [ctypes.c_float]
        self.lib.orc_half_to_float.restype = ctypes.c_float
        self.lib.orc_half_to_float.argtypes = [ctypes.c_uint16]

    def matmul_f64(self, fmt: str, a_q: np.ndarray, b: np.ndarray, M: int, K: int) -> np.ndarray:
        a_q = np.ascontiguousarray(a_q, dtype=np.uint8)
        b = np.ascontiguousarray(b, dtype=np.float32)
        N = b.shape[1]
        out = np.zeros((M, N), dtype=np.float64)
        rc = self.lib.orc_matmul_f64(FORMATS[fmt], _ptr(a_q), _ptr(b), _ptr(out), M, K, N)
        if rc != 0:
            raise RuntimeError("orc_matmul_f64 failed")
        return out

    def matmul_rows(self, fmt: str, a_q: np.ndarray, b: np.ndarray, out: np.ndarray,
                    M: int, K: int, row0: int, row1: int) -> None:
        """Rows [row0,row1) of the product into `out` (M x N); for threaded timing."""
        rc = self.lib.orc_matmul_rows(FORMATS[fmt], _ptr(a_q), _ptr(b), _ptr(out), M, K,
                                      b.shape[1], row0, row1)
        if rc != 0:
            raise RuntimeError("orc_matmul_rows failed")


class Reference(_Lib):
    """The reference's own CPU code, compiled from its sources."""

    def __init__(self, path: str = REF_PATH):
        super().__init__(path, "ref")
        L = self.lib
        L.ref_has_avx2.restype = ctypes.c_int
        L.ref_job_create.restype = _vp
        L.ref_job_create.argtypes = [ctypes.c_int, _vp, _vp, _c_i64, _c_i64, _c_i64, ctypes.c_int]
        L.ref_job_run.restype = ctypes.c_int
        L.ref_job_run.argtypes = [_vp, _vp]
        L.ref_job_destroy.restype = None
        L.ref_job_destroy.argtypes = [_vp]
        L.ref_quantize_threads.restype = ctypes.c_int
        L.ref_quantize_threads.argtypes = [ctypes.c_int, _vp, _c_i64, _c_i64, _vp, ctypes.c_int]
        L.ref_quantized_size.restype = ctypes.c_size_t
        L.ref_quantized_size.argtypes = [ctypes.c_size_t, ctypes.c_int]
        L.ref_quantized_size_2d.restype = ctypes.c_size_t
        L.ref_quantized_size_2d.argtypes = [_c_i64, _c_i64, ctypes.c_int]

    def has_avx2(self) -> bool:
        return bool(self.lib.ref_has_avx2())

    def matmul_f32(self, a: np.ndarray, b: np.ndarray) -> np.ndarray:
        """cpu::matmul (cpu_backend.cpp:116-173) of fp32 [M x K] . [K x N]."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        b = np.ascontiguousarray(b, dtype=np.float32)
        M, K = a.shape
        N = b.shape[1]
        out = np.zeros((M, N), dtype=np.float32)
        L = self.lib
        L.ref_matmul_f32.argtypes = [_vp, _vp, _vp, _c_i64, _c_i64, _c_i64]
        if L.ref_matmul_f32(_ptr(a), _ptr(b), _ptr(out), M, K, N) != 0:
            raise RuntimeError("ref_matmul_f32 failed")
        return out

    # ---- .axon files through the reference's serializer (src/core/serialize.cpp)

    def save_tensor(self, path: str, shape, dtype: int, quant: int, data: np.ndarray) -> None:
        """save_tensor (serialize.cpp:84-96) of one tensor named "data"."""
        sh = np.ascontiguousarray(shape, dtype=np.int64)
        d = np.ascontiguousarray(data).view(np.uint8).ravel()
        L = self.lib
        L.ref_save_tensor.argtypes = [ctypes.c_char_p, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp,
                                      ctypes.c_size_t]
        if L.ref_save_tensor(path.encode(), _ptr(sh), len(shape), dtype, quant, _ptr(d), d.size) != 0:
            raise RuntimeError("ref_save_tensor failed")

    def save_checkpoint(self, path: str, tensors) -> None:
        """save_checkpoint (serialize.cpp:125-148); tensors: list of
        (name, shape, dtype, quant, data)."""
        n = len(tensors)
        names = (ctypes.c_char_p * n)(*[t[0].encode() for t in tensors])
        shapes = np.concatenate([np.asarray(t[1], dtype=np.int64) for t in tensors])
        ndims = np.asarray([len(t[1]) for t in tensors], dtype=np.int32)
        dtypes = np.asarray([t[2] for t in tensors], dtype=np.int32)
        quants = np.asarray([t[3] for t in tensors], dtype=np.int32)
        datas = [np.ascontiguousarray(t[4]).view(np.uint8).ravel() for t in tensors]
        ptrs = (_vp * n)(*[_ptr(d) for d in datas])
        sizes = (ctypes.c_size_t * n)(*[d.size for d in datas])
        L = self.lib
        L.ref_save_checkpoint.argtypes = [ctypes.c_char_p, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp]
        rc = L.ref_save_checkpoint(path.encode(), n, ctypes.cast(names, _vp), _ptr(shapes), _ptr(ndims),
                                   _ptr(dtypes), _ptr(quants), ctypes.cast(ptrs, _vp), ctypes.cast(sizes, _vp))
        if rc != 0:
            raise RuntimeError("ref_save_checkpoint failed")

    def load_tensor(self, path: str, cap: int = 1 << 20):
        """load_tensor (serialize.cpp:98-123): (data bytes, None) or (None, error)."""
        out = np.zeros(cap, dtype=np.uint8)
        got = ctypes.c_size_t(0)
        err = ctypes.create_string_buffer(512)
        L = self.lib
        L.ref_load_tensor.argtypes = [ctypes.c_char_p, _vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t),
                                      ctypes.c_char_p, ctypes.c_size_t]
        if L.ref_load_tensor(path.encode(), _ptr(out), cap, ctypes.byref(got), err, 512) != 0:
            return None, err.value.decode()
        return out[:got.value].copy(), None

    def quantize_1d(self, fmt: str, x: np.ndarray) -> np.ndarray:
        """The reference's flat (1-D tensor) pack path."""
        x = np.ascontiguousarray(x, dtype=np.float32).ravel()
        n = int(self.lib.ref_quantized_size(x.size, FORMATS[fmt]))
        out = np.zeros(n, dtype=np.uint8)
        rc = self.lib.ref_quantize(FORMATS[fmt], _ptr(x), -1, x.size, _ptr(out))
        if rc != 0:
            raise RuntimeError("ref_quantize (1-D) failed")
        return out


class MatmulJob:
    """Threaded reference matmul (rows of A_q split across host threads)."""

    def __init__(self, ref: Reference, fmt: str, a_q: np.ndarray, b: np.ndarray, M: int, K: int,
                 threads: int):
        self._keep = (np.ascontiguousarray(a_q, dtype=np.uint8), np.ascontiguousarray(b, dtype=np.float32))
        self.ref = ref
        self.N = b.shape[1]
        self.M = M
        self.h = ref.lib.ref_job_create(FORMATS[fmt], _ptr(self._keep[0]), _ptr(self._keep[1]), M, K,
                                        self.N, threads)

    def run(self, out: Optional[np.ndarray] = None) -> None:
        rc = self.ref.lib.ref_job_run(self.h, _ptr(out) if out is not None else None)
        if rc != 0:
            raise RuntimeError("ref_job_run failed")

    def close(self) -> None:
        if self.h:
            self.ref.lib.ref_job_destroy(self.h)
            self.h = None


_orc: Optional[Oracle] = None
_ref: Optional[Reference] = None


def orc() -> Oracle:
    global _orc
    if _orc is None:
        if not os.path.exists(ORC_PATH):
            raise FileNotFoundError(f"{ORC_PATH} missing: run `make -C oracle`")
        _orc = Oracle()
    return _orc


def ref() -> Optional[Reference]:
    """The compiled reference, or None where it was not built."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        _ref = Reference()
    return _ref
