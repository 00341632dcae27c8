"""Tensor-level entry points over the C ABI.

Each function mirrors one reference CPU-backend function (ruwwww/Axon
``include/axon/backend/cpu_backend.h:36-46``): same name, same argument
order (output first), same meaning.  The quantized operand is carried by
:class:`QTensor`, the counterpart of a reference ``Tensor`` whose metadata has
``quant != None`` and whose ``Storage`` holds the raw blocks
(``tensor_metadata.h:14-24``, ``storage.h:21-25``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch

from ._capi import (
    BLOCK_BYTES,
    BLOCK_ELEMS,
    FLAG_B_TOKMAJOR,
    FLAG_OUT_TOKMAJOR,
    AxqError,
    QuantFormat,
    Status,
    check,
    lib,
    quantized_size_2d,
)


def _stream_handle(stream: Optional[torch.cuda.Stream], device: Optional[torch.device] = None) -> int:
    if stream is not None:
        return int(stream.cuda_stream)
    idx = device.index if device is not None and device.index is not None else torch.cuda.current_device()
    return int(torch._C._cuda_getCurrentRawStream(idx))  # the current stream, without a Stream object


_ws_size_cache: Dict[Tuple[int, int, int, int], int] = {}


def _ws_size(fmt: int, M: int, K: int, N: int) -> int:
    key = (fmt, M, K, N)
    v = _ws_size_cache.get(key)
    if v is None:
        v = int(lib().axq_matmul_workspace_size(fmt, M, K, N))
        if len(_ws_size_cache) < 4096:
            _ws_size_cache[key] = v
    return v


def _packed_bytes(M: int, K: int, fmt: QuantFormat) -> int:
    be = BLOCK_ELEMS[fmt]
    return M * ((K + be - 1) // be) * BLOCK_BYTES[fmt]


def _req_cuda(t: torch.Tensor, name: str, dtype: torch.dtype) -> None:
    if not isinstance(t, torch.Tensor):
        raise AxqError(Status.ERR_INVALID, f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise AxqError(Status.ERR_INVALID, f"{name} must be a CUDA tensor (got {t.device})")
    if t.dtype != dtype:
        raise AxqError(Status.ERR_INVALID, f"{name} must be {dtype} (got {t.dtype})")
    if not t.is_contiguous():
        raise AxqError(Status.ERR_INVALID, f"{name} must be contiguous")


@dataclass
class QTensor:
    """Packed blocks of a [rows x cols] matrix (uint8 CUDA buffer) plus its
    QuantizationDescriptor (format, block size)."""

    data: torch.Tensor
    shape: Tuple[int, int]
    fmt: QuantFormat

    @property
    def block_size(self) -> int:
        return BLOCK_ELEMS[self.fmt]

    @staticmethod
    def empty(rows: int, cols: int, fmt: QuantFormat, device="cuda") -> "QTensor":
        n = quantized_size_2d(rows, cols, fmt)
        return QTensor(torch.empty(max(n, 1), dtype=torch.uint8, device=device), (rows, cols), QuantFormat(fmt))


def quantize(dst, src: torch.Tensor, fmt: QuantFormat, stream: Optional[torch.cuda.Stream] = None):
    """Pack ``src`` (fp32, 1-D or 2-D, row-major) into ``dst``.

    Replaces ``cpu::quantize(dst, src, format)`` (src/backend/cpu_backend.cpp:1160).
    ``dst`` is a :class:`QTensor` or a uint8 CUDA tensor of at least
    ``quantized_size_2d`` bytes.  Output bytes equal the reference's."""
    fmt = QuantFormat(fmt)
    _req_cuda(src, "src", torch.float32)
    if src.dim() == 1:
        rows, cols = 1, src.shape[0]
    elif src.dim() == 2:
        rows, cols = src.shape
    else:
        raise AxqError(Status.ERR_INVALID, "quantize: src must be 1-D or 2-D")
    buf = dst.data if isinstance(dst, QTensor) else dst
    _req_cuda(buf, "dst", torch.uint8)
    need = quantized_size_2d(rows, cols, fmt)
    if buf.numel() < need:
        raise AxqError(Status.ERR_INVALID, f"quantize: dst holds {buf.numel()} bytes, {need} needed")
    check(lib().axq_quantize(int(fmt), src.data_ptr(), buf.data_ptr(), rows, cols, _stream_handle(stream)))
    if isinstance(dst, QTensor):
        dst.shape, dst.fmt = (rows, cols), fmt
    return dst


def dequantize(dst: torch.Tensor, src, fmt: Optional[QuantFormat] = None,
               stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Decode packed ``src`` into ``dst`` (fp32, its shape gives rows/cols).

    Replaces ``cpu::dequantize(dst, src)`` (src/backend/cpu_backend.cpp:1334);
    like the reference, the format comes from the quantized operand (a
    :class:`QTensor`) unless given explicitly for a raw byte buffer."""
    buf = src.data if isinstance(src, QTensor) else src
    if fmt is None:
        if not isinstance(src, QTensor):
            raise AxqError(Status.ERR_INVALID, "dequantize: format unknown for a raw buffer")
        fmt = src.fmt
    fmt = QuantFormat(fmt)
    _req_cuda(dst, "dst", torch.float32)
    _req_cuda(buf, "src", torch.uint8)
    rows, cols = (1, dst.shape[0]) if dst.dim() == 1 else tuple(dst.shape)
    need = quantized_size_2d(rows, cols, fmt)
    if buf.numel() < need:
        raise AxqError(Status.ERR_INVALID, f"dequantize: src holds {buf.numel()} bytes, {need} needed")
    check(lib().axq_dequantize(int(fmt), buf.data_ptr(), dst.data_ptr(), rows, cols, _stream_handle(stream)))
    return dst


class Workspace:
    """Device scratch for ``axq_matmul``, one growing buffer per device.

    Allocation happens here (torch's caching allocator), outside the C ABI,
    whose matmul call allocates nothing."""

    def __init__(self):
        self._bufs: Dict[int, torch.Tensor] = {}

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        idx = device.index if device.index is not None else torch.cuda.current_device()
        buf = self._bufs.get(idx)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 256) + 256, dtype=torch.uint8, device=f"cuda:{idx}")
            self._bufs[idx] = buf
        return buf


_default_ws = Workspace()


def _aligned_ptr(buf: torch.Tensor) -> Tuple[int, int]:
    p = buf.data_ptr()
    off = (-p) % 256
    return p + off, buf.numel() - off


def matmul_q(out: torch.Tensor, a, b: torch.Tensor, fmt: Optional[QuantFormat] = None,
             M: Optional[int] = None, K: Optional[int] = None, *, b_tokmajor: bool = False,
             out_tokmajor: bool = False, workspace: Optional[Workspace] = None,
             stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """``out = A_q . B`` in the reference's orientation (quantized LEFT operand).

    ``a`` is a :class:`QTensor` of shape [M, K] (or a raw uint8 buffer with
    ``fmt``/``M``/``K``).  ``b`` is fp32 [K, N] (``b_tokmajor``: [N, K]);
    ``out`` is fp32 [M, N] (``out_tokmajor``: [N, M])."""
    if isinstance(a, QTensor):
        buf, fmt, (M, K) = a.data, a.fmt, a.shape
    else:
        buf = a
        if fmt is None or M is None or K is None:
            raise AxqError(Status.ERR_INVALID, "matmul_q: fmt, M and K are required for a raw buffer")
    fmt = QuantFormat(fmt)
    _req_cuda(buf, "a", torch.uint8)
    _req_cuda(b, "b", torch.float32)
    _req_cuda(out, "out", torch.float32)
    if b.dim() != 2 or out.dim() != 2:
        raise AxqError(Status.ERR_INVALID, "matmul_q: inputs must be 2D")
    kb, N = (b.shape[1], b.shape[0]) if b_tokmajor else (b.shape[0], b.shape[1])
    if kb != K:
        raise AxqError(Status.ERR_INVALID, "matmul_q: inner dimension mismatch")
    want = (N, M) if out_tokmajor else (M, N)
    if tuple(out.shape) != want:
        raise AxqError(Status.ERR_INVALID, f"matmul_q: output shape {tuple(out.shape)} != {want}")
    if buf.numel() < _packed_bytes(M, K, fmt):
        raise AxqError(Status.ERR_INVALID, "matmul_q: quantized operand is smaller than its shape")
    flags = (FLAG_B_TOKMAJOR if b_tokmajor else 0) | (FLAG_OUT_TOKMAJOR if out_tokmajor else 0)
    need = _ws_size(int(fmt), M, K, N)
    ws = (workspace or _default_ws).get(need + 256, out.device)
    wp, wbytes = _aligned_ptr(ws)
    check(lib().axq_matmul(int(fmt), buf.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N, flags, wp, wbytes,
                           _stream_handle(stream, out.device)))
    return out


def _fixed(fmt: QuantFormat, name: str):
    def fn(out: torch.Tensor, a: QTensor, b: torch.Tensor, **kw) -> torch.Tensor:
        if a.fmt != fmt:
            raise AxqError(Status.ERR_INVALID, f"{name}: operand is {a.fmt.name}, not {fmt.name}")
        return matmul_q(out, a, b, **kw)

    fn.__name__ = name
    fn.__doc__ = f"{fmt.name} quantized matmul; replaces cpu::{name} of the reference."
    return fn


matmul_q8_0 = _fixed(QuantFormat.Q8_0, "matmul_q8_0")
matmul_q4 = _fixed(QuantFormat.Q4_0, "matmul_q4")
matmul_q2_K = _fixed(QuantFormat.Q2_K, "matmul_q2_K")
matmul_q3_K = _fixed(QuantFormat.Q3_K, "matmul_q3_K")
matmul_q4_K = _fixed(QuantFormat.Q4_K, "matmul_q4_K")
matmul_q5_K = _fixed(QuantFormat.Q5_K, "matmul_q5_K")
matmul_q6_K = _fixed(QuantFormat.Q6_K, "matmul_q6_K")


def matmul(out: torch.Tensor, a, b: torch.Tensor, stream: Optional[torch.cuda.Stream] = None, **kw) -> torch.Tensor:
    """``out = a . b`` routed like the reference's ``cpu::matmul``
    (src/backend/cpu_backend.cpp:116-173 with choose_gemm_strategy,
    src/backend/cpu/strategy.cpp:5-65): a packed :class:`QTensor` A goes to
    its format's quantized matmul, an fp32 A (all row-major [M x K] . [K x N])
    to the fp32 GEMM (``axq_matmul_f32``, fp32 multiply-adds, no TF32)."""
    if isinstance(a, QTensor):
        return matmul_q(out, a, b, stream=stream, **kw)
    for t, name in ((a, "a"), (b, "b"), (out, "out")):
        _req_cuda(t, name, torch.float32)
        if t.dim() != 2:
            raise AxqError(Status.ERR_INVALID, "cpu::matmul: all inputs must be 2D")
    M, K = a.shape
    if b.shape[0] != K:
        raise AxqError(Status.ERR_INVALID, "cpu::matmul: inner dimensions must match")
    N = b.shape[1]
    if tuple(out.shape) != (M, N):
        raise AxqError(Status.ERR_INVALID, "cpu::matmul: output shape mismatch")
    check(lib().axq_matmul_f32(a.data_ptr(), b.data_ptr(), out.data_ptr(), M, K, N, _stream_handle(stream, out.device)))
    return out


def linear_q(x: torch.Tensor, w: QTensor, out: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None,
             workspace: Optional[Workspace] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Quantized Linear: y[N, M] = x[N, K] . W[M, K]^T (+ bias[M]) with W
    packed row-wise (C ABI axq_linear).

    The reference's Linear (src/nn/linear.cpp:19-27) keeps an fp32 weight
    [in, out] on the right of rt.matmul and adds the bias with AddOp; a
    packed weight sits on the left, so this is y = (W_q . x^T)^T + bias."""
    M, K = w.shape
    _req_cuda(x, "x", torch.float32)
    _req_cuda(w.data, "w", torch.uint8)
    if x.dim() != 2 or x.shape[1] != K:
        raise AxqError(Status.ERR_INVALID, f"linear_q: x must be [N x {K}]")
    N = x.shape[0]
    if out is None:
        out = torch.empty((N, M), dtype=torch.float32, device=x.device)
    _req_cuda(out, "out", torch.float32)
    if tuple(out.shape) != (N, M):
        raise AxqError(Status.ERR_INVALID, f"linear_q: out must be [{N} x {M}]")
    if w.data.numel() < _packed_bytes(M, K, w.fmt):
        raise AxqError(Status.ERR_INVALID, "linear_q: quantized weight is smaller than its shape")
    bptr = None
    if bias is not None:
        _req_cuda(bias, "bias", torch.float32)
        if bias.numel() != M:
            raise AxqError(Status.ERR_INVALID, f"linear_q: bias must have {M} elements")
        bptr = bias.data_ptr()
    need = _ws_size(int(w.fmt), M, K, N)
    wp, wbytes = _aligned_ptr((workspace or _default_ws).get(need + 256, out.device))
    check(lib().axq_linear(int(w.fmt), w.data.data_ptr(), x.data_ptr(), bptr, out.data_ptr(), M, K, N, wp, wbytes,
                           _stream_handle(stream, out.device)))
    return out


def gate_up_silu(x: torch.Tensor, w_gate: QTensor, w_up: QTensor, out: Optional[torch.Tensor] = None,
                 workspace: Optional[Workspace] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Fused front half of a gated MLP: h[N, M] = silu(x . W_gate^T) * (x . W_up^T),
    silu(v) = v / (1 + e^-v).  The reference has neither SiLU nor a quantized
    Linear (its Linear, src/nn/linear.cpp:19-27, is fp32); this composes its
    quantized matmul.  Up to 8 rows of x (4 for Q8_0 / Q4_0) run as a single
    GEMV pass over both packed matrices (one activation prep, SiLU and product
    in the epilogue)."""
    if w_gate.fmt != w_up.fmt or tuple(w_gate.shape) != tuple(w_up.shape):
        raise AxqError(Status.ERR_INVALID, "gate_up_silu: W_gate and W_up must have the same shape and format")
    M, K = w_gate.shape
    fmt = int(w_gate.fmt)
    _req_cuda(x, "x", torch.float32)
    _req_cuda(w_gate.data, "w_gate", torch.uint8)
    _req_cuda(w_up.data, "w_up", torch.uint8)
    if x.dim() != 2 or x.shape[1] != K:
        raise AxqError(Status.ERR_INVALID, f"gate_up_silu: x must be [N x {K}]")
    N = x.shape[0]
    if out is None:
        out = torch.empty((N, M), dtype=torch.float32, device=x.device)
    _req_cuda(out, "out", torch.float32)
    if tuple(out.shape) != (N, M):
        raise AxqError(Status.ERR_INVALID, f"gate_up_silu: out must be [{N} x {M}]")
    need = int(lib().axq_gate_up_workspace_size(fmt, M, K, N))
    wp, wbytes = _aligned_ptr((workspace or _default_ws).get(need + 256, out.device))
    check(lib().axq_gate_up_silu(fmt, w_gate.data.data_ptr(), w_up.data.data_ptr(), x.data_ptr(), out.data_ptr(), M, K,
                                 N, FLAG_B_TOKMAJOR | FLAG_OUT_TOKMAJOR, wp, wbytes, _stream_handle(stream, out.device)))
    return out


def mlp_q(x: torch.Tensor, w_gate: QTensor, w_up: QTensor, w_down: QTensor, out: Optional[torch.Tensor] = None,
          workspace: Optional[Workspace] = None, stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
    """Gated MLP block y = (silu(x W_gate^T) * (x W_up^T)) W_down^T with packed
    weights: the fused gate/up pass, then the down projection."""
    h = gate_up_silu(x, w_gate, w_up, workspace=workspace, stream=stream)
    return linear_q(h, w_down, out=out, workspace=workspace, stream=stream)
