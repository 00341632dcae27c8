""".axon tensor files straight to and from device memory.

Replaces the reference's ``save_tensor`` / ``load_tensor`` /
``save_checkpoint`` / ``load_checkpoint`` (src/core/serialize.cpp:84-203)
for CUDA tensors, through ``axq_axon_*`` of ``include/axq.h``.  The bytes on
disk are the reference's, so files move between the two.  The reference's
loaders ignore the recorded quant_type and fail on packed tensors ("Tensor
data size mismatch"); here a packed record comes back as a :class:`QTensor`
in its format, ready for ``linear_q`` / ``matmul_q``.

Destinations may also be CPU tensors (``device="cpu"``): the file is then
read straight into host memory, which needs no GPU.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Mapping, Optional, Tuple, Union

import torch

from ._capi import (AXON_FLAT, AXON_MAX_DIMS, AXON_NAME_BYTES, AXON_PLAIN, AXON_ROWS, AxonTensorInfo, AxqError,
                    QuantFormat, Status, check, lib, quantized_size_2d)
from .ops import QTensor, _stream_handle

# The reference's DType ordinals (include/axon/core/types.h:9-17).
DTYPES = {0: torch.float32, 1: torch.float64, 2: torch.int32, 3: torch.int64, 4: torch.int16, 5: torch.int8,
          6: torch.uint8}
DTYPE_IDS = {v: k for k, v in DTYPES.items()}
LAYOUTS = {AXON_PLAIN: "plain", AXON_ROWS: "rows", AXON_FLAT: "flat"}


@dataclass
class AxonRecord:
    """Metadata of one tensor of an .axon file."""

    name: str
    dtype: int
    quant: QuantFormat
    shape: Tuple[int, ...]
    layout: str          # "plain", "rows" (packed rows of whole blocks) or "flat" (packed flattened tensor)
    data_bytes: int
    offset: int


class _File:
    def __init__(self, path: str):
        h = ctypes.c_void_p()
        n = ctypes.c_uint32()
        check(lib().axq_axon_open(path.encode(), ctypes.byref(h), ctypes.byref(n)))
        self.h, self.count = h, n.value

    def info(self, i: int) -> Tuple[AxonRecord, AxonTensorInfo]:
        raw = AxonTensorInfo()
        check(lib().axq_axon_info(self.h, i, ctypes.byref(raw)))
        rec = AxonRecord(raw.name.decode("utf-8", "replace"), raw.dtype, QuantFormat(raw.quant),
                         tuple(raw.shape[d] for d in range(raw.ndims)), LAYOUTS[raw.layout], raw.data_bytes,
                         raw.offset)
        return rec, raw

    def close(self):
        if self.h:
            lib().axq_axon_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def axon_records(path: str) -> List[AxonRecord]:
    """Every record of an .axon file (the file is checked as a whole first)."""
    with _File(path) as f:
        return [f.info(i)[0] for i in range(f.count)]


def _rows_cols(shape: Tuple[int, ...]) -> Tuple[int, int]:
    cols = shape[-1] if shape else 1
    numel = 1
    for s in shape:
        numel *= s
    return (numel // cols if cols else 0), cols


def load_axon(path: str, device: Union[str, torch.device, None] = None,
              stream: Optional[torch.cuda.Stream] = None) -> Dict[str, Union[QTensor, torch.Tensor]]:
    """All tensors of an .axon file, by name, in file order (what
    load_checkpoint reads, serialize.cpp:151-201).  Packed records become
    :class:`QTensor`: rows-layout tensors keep their [rows x last dim]
    matrix shape (rows = product of the other dimensions); flat-layout ones
    (rows not whole blocks) are one row of all their elements.  Plain
    records become tensors of their dtype and shape."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    out: Dict[str, Union[QTensor, torch.Tensor]] = {}
    with _File(path) as f:
        for i in range(f.count):
            rec, _ = f.info(i)
            if rec.quant != QuantFormat.NONE:
                buf = torch.empty(max(rec.data_bytes, 1), dtype=torch.uint8, device=dev)
                if rec.layout == "rows":
                    shape = _rows_cols(rec.shape)
                else:
                    numel = 1
                    for s in rec.shape:
                        numel *= s
                    shape = (1, numel)
                val: Union[QTensor, torch.Tensor] = QTensor(buf, shape, rec.quant)
            else:
                if rec.dtype not in DTYPES:
                    raise AxqError(Status.ERR_UNSUPPORTED, f"load_axon: dtype {rec.dtype} has no torch type")
                buf = torch.empty(rec.shape, dtype=DTYPES[rec.dtype], device=dev)
                val = buf
            sh = _stream_handle(stream, dev) if dev.type == "cuda" else 0
            check(lib().axq_axon_read(f.h, i, buf.data_ptr(), buf.numel() * buf.element_size(), sh))
            out[rec.name] = val
    return out


def load_tensor(path: str, device: Union[str, torch.device, None] = None) -> Union[QTensor, torch.Tensor]:
    """The first tensor of an .axon file (the reference's load_tensor,
    serialize.cpp:98-123, which also reads only the first record)."""
    tensors = load_axon(path, device)
    if not tensors:
        raise AxqError(Status.ERR_INVALID, "load_tensor: no tensors in file")
    return next(iter(tensors.values()))


def save_axon(path: str, tensors: Mapping[str, Union[QTensor, torch.Tensor]],
              stream: Optional[torch.cuda.Stream] = None) -> None:
    """Write tensors (CUDA or CPU) in the reference's format, in the
    mapping's order (what save_checkpoint writes for a module's parameters,
    serialize.cpp:125-148).  A QTensor is written as a packed [rows x cols]
    record of its format (quant_type set, rows layout); a tensor with its
    dtype and shape."""
    infos = (AxonTensorInfo * max(len(tensors), 1))()
    ptrs = (ctypes.c_void_p * max(len(tensors), 1))()
    keep = []
    dev = None
    for i, (name, t) in enumerate(tensors.items()):
        nb = name.encode()
        if len(nb) >= AXON_NAME_BYTES:
            raise AxqError(Status.ERR_INVALID, f"save_axon: name '{name}' too long")
        info = infos[i]
        info.name = nb
        if isinstance(t, QTensor):
            rows, cols = t.shape
            info.dtype, info.quant, info.ndims = 0, int(t.fmt), 2
            info.shape[0], info.shape[1] = rows, cols
            info.data_bytes = quantized_size_2d(rows, cols, t.fmt)
            buf = t.data
        else:
            if t.dtype not in DTYPE_IDS:
                raise AxqError(Status.ERR_UNSUPPORTED, f"save_axon: dtype {t.dtype} has no .axon id")
            if t.dim() > AXON_MAX_DIMS:
                raise AxqError(Status.ERR_INVALID, f"save_axon: '{name}' has more than {AXON_MAX_DIMS} dimensions")
            buf = t.contiguous()
            info.dtype, info.quant, info.ndims = DTYPE_IDS[t.dtype], 0, buf.dim()
            for d in range(buf.dim()):
                info.shape[d] = buf.shape[d]
            info.data_bytes = buf.numel() * buf.element_size()
        if buf.numel() * buf.element_size() < info.data_bytes:
            raise AxqError(Status.ERR_INVALID, f"save_axon: '{name}' buffer is smaller than its data")
        keep.append(buf)
        ptrs[i] = buf.data_ptr()
        if buf.is_cuda:
            dev = buf.device
    sh = _stream_handle(stream, dev) if dev is not None else 0
    check(lib().axq_axon_save(path.encode(), len(tensors), ctypes.cast(infos, ctypes.c_void_p),
                              ctypes.cast(ptrs, ctypes.c_void_p), sh))


def save_tensor(t: Union[QTensor, torch.Tensor], path: str) -> None:
    """One tensor named "data", as the reference's save_tensor
    (serialize.cpp:84-96) writes it."""
    save_axon(path, {"data": t})
