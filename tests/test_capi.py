"""The C ABI library: loads, exports every declared symbol, host-side logic
(CPU only — no kernel is launched here)."""
import os
import re

import pytest

from conftest import FORMATS, ROOT

HEADER = os.path.join(ROOT, "include", "axq.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(axq_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    import ctypes
    import axon_b200
    L = axon_b200.lib()
    syms = declared_symbols()
    assert len(syms) >= 9
    for s in syms:
        assert hasattr(L, s), f"{s} declared in include/axq.h but not exported"
        assert s in axon_b200._capi.SIGNATURES, f"{s} has no Python binding"
    assert L.axq_version() >= 100
    assert isinstance(ctypes.cast(L.axq_last_error(), ctypes.c_char_p).value, (bytes, type(None)))


@pytest.mark.parametrize("fmt", FORMATS)
def test_size_helpers_match_oracle(orc, fmt):
    import oracle
    import axon_b200
    F = axon_b200.QuantFormat[fmt]
    for n in (0, 1, 31, 32, 33, 255, 256, 257, 4096, 11008, 1 << 30):
        assert axon_b200.quantized_size(n, F) == orc.lib.orc_quantized_size(n, oracle.FORMATS[fmt])
    for rows, cols in ((1, 1), (3, 300), (4096, 4096), (28672, 8192), (4096, 11008)):
        assert axon_b200.quantized_size_2d(rows, cols, F) == oracle.packed_size_2d(fmt, rows, cols)


def test_unknown_format_is_rejected_before_any_device_call():
    import axon_b200
    L = axon_b200.lib()
    assert L.axq_quantize(0, None, None, 4, 4, None) == axon_b200.Status.ERR_UNSUPPORTED
    assert b"unsupported format" in L.axq_last_error()
    assert L.axq_dequantize(99, None, None, 4, 4, None) == axon_b200.Status.ERR_UNSUPPORTED
    assert L.axq_matmul(8, None, None, None, 4, 4, 4, 0, None, 0, None) == axon_b200.Status.ERR_UNSUPPORTED
    assert L.axq_quantized_size(10, 0) == 0
    assert L.axq_matmul_workspace_size(0, 1, 1, 1) == 0


def test_shape_and_flag_errors_are_reported():
    import axon_b200
    L = axon_b200.lib()
    assert L.axq_quantize(1, None, None, -1, 4, None) == axon_b200.Status.ERR_INVALID
    assert b"negative shape" in L.axq_last_error()
    assert L.axq_matmul(1, None, None, None, 4, 4, 4, 64, None, 0, None) == axon_b200.Status.ERR_INVALID
    assert b"flag" in L.axq_last_error()
    # empty problems are successful no-ops that touch no pointer
    assert L.axq_quantize(1, None, None, 0, 4, None) == 0
    assert L.axq_matmul(1, None, None, None, 0, 4, 4, 0, None, 0, None) == 0


def test_workspace_size_grows_with_tokens():
    import axon_b200
    F = axon_b200.QuantFormat.Q4_K
    a = axon_b200.matmul_workspace_size(F, 4096, 4096, 1)
    b = axon_b200.matmul_workspace_size(F, 4096, 4096, 8)
    assert 0 < a < b
    assert a % 256 == 0 and b % 256 == 0


def test_workspace_size_follows_the_gemv_token_range():
    """Up to 8 tokens of a K-quant format (4 of Q8_0 / Q4_0) take the GEMV,
    whose workspace is the 256-byte status block plus one 592-byte activation
    record per 256 elements and token (rounded to 256 bytes); beyond that the
    GEMM's larger workspace applies."""
    import axon_b200
    Q = axon_b200.QuantFormat
    M, K = 4096, 4096

    def gemv_bytes(n):
        return 256 + -(-(K // 256) * n * 592 // 256) * 256

    for f in (Q.Q2_K, Q.Q3_K, Q.Q4_K, Q.Q5_K, Q.Q6_K):
        for n in (1, 2, 5, 8):
            assert axon_b200.matmul_workspace_size(f, M, K, n) == gemv_bytes(n), (f, n)
        assert axon_b200.matmul_workspace_size(f, M, K, 9) != gemv_bytes(9), f
    for f in (Q.Q8_0, Q.Q4_0):
        assert axon_b200.matmul_workspace_size(f, M, K, 4) == gemv_bytes(4), f
        assert axon_b200.matmul_workspace_size(f, M, K, 5) != gemv_bytes(5), f
