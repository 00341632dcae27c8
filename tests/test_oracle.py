"""The CPU oracle, pinned against the reference (CPU only).

* exact byte counts from the reference's own test
  (tests/backend/quantization_test.cpp:9-40);
* golden fixtures produced by the compiled reference (tests/golden/);
* the live compiled reference, when it was built here (oracle/_ref);
* the round-trip margins of quantization_test.cpp:74-100.
"""
import os

import numpy as np
import pytest

from conftest import FORMATS, gen

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load_golden(fmt):
    z = np.load(os.path.join(GOLDEN, f"golden_{fmt}.npz"))
    names = sorted({k.split("__")[0] for k in z.files})
    return {n: {f: z[f"{n}__{f}"] for f in ("x", "q", "deq", "b", "mm")} for n in names}


SIZE_PINS = [  # quantization_test.cpp:9-40
    (32, "Q8_0", 34), (64, "Q8_0", 68), (1, "Q8_0", 34), (33, "Q8_0", 68),
    (32, "Q4_0", 18), (64, "Q4_0", 36), (1, "Q4_0", 18), (33, "Q4_0", 36),
    (256, "Q2_K", 84), (512, "Q2_K", 168), (1, "Q2_K", 84),
    (256, "Q3_K", 110), (512, "Q3_K", 220), (1, "Q3_K", 110),
    (256, "Q4_K", 144), (512, "Q4_K", 288), (1, "Q4_K", 144),
    (256, "Q5_K", 176), (512, "Q5_K", 352), (1, "Q5_K", 176),
    (256, "Q6_K", 210), (512, "Q6_K", 420), (1, "Q6_K", 210),
]


@pytest.mark.parametrize("n,fmt,size", SIZE_PINS)
def test_quantized_size_pins(orc, n, fmt, size):
    import oracle
    assert orc.lib.orc_quantized_size(n, oracle.FORMATS[fmt]) == size


@pytest.mark.parametrize("fmt", FORMATS)
def test_oracle_matches_golden(orc, fmt):
    for name, g in load_golden(fmt).items():
        rows, cols = g["x"].shape
        q = orc.quantize(fmt, g["x"])
        assert np.array_equal(q, g["q"]), f"{fmt}/{name}: packed bytes differ"
        d = orc.dequantize(fmt, g["q"], rows, cols)
        assert np.array_equal(d.view(np.uint32), g["deq"].view(np.uint32)), f"{fmt}/{name}: dequant differs"
        mm = orc.matmul(fmt, g["q"], g["b"], rows, cols)
        if fmt in ("Q2_K", "Q3_K", "Q6_K"):  # scalar-only in the reference: same loop order, bit-equal
            assert np.array_equal(mm.view(np.uint32), g["mm"].view(np.uint32)), f"{fmt}/{name}: matmul differs"
        else:  # reference used its AVX2 (FMA) kernel or fp32 GEMM
            den = max(np.abs(g["mm"]).max(), 1e-30)
            assert np.abs(mm - g["mm"]).max() / den < 1e-5, f"{fmt}/{name}"


@pytest.mark.parametrize("fmt", FORMATS)
def test_oracle_matches_live_reference(orc, ref, fmt):
    if ref is None:
        pytest.skip("reference library not built here")
    rng = np.random.default_rng(7)
    for kind in ("sweep", "w002", "outlier"):
        for shape in ((16, 4096), (3, 1000), (2, 11008), (4, 33)):
            x = gen(rng, shape, kind)
            q = ref.quantize(fmt, x)
            assert np.array_equal(orc.quantize(fmt, x), q), (fmt, kind, shape)
            assert np.array_equal(orc.dequantize(fmt, q, *shape).view(np.uint32),
                                  ref.dequantize(fmt, q, *shape).view(np.uint32))
    x = gen(rng, 1000, "randn")
    assert np.array_equal(ref.quantize_1d(fmt, x), orc.quantize(fmt, x)), "1-D path"


@pytest.mark.parametrize("fmt", FORMATS)
def test_oracle_edge_values_match_reference(orc, ref, fmt):
    if ref is None:
        pytest.skip("reference library not built here")
    rng = np.random.default_rng(11)
    base = rng.standard_normal((2, 512)).astype(np.float32)
    variants = [np.zeros_like(base), np.full_like(base, -0.7), base * np.float32(1e7), base * np.float32(1e-6),
                base * np.float32(1e-39)]
    v = base.copy(); v[0, 5] = np.inf; v[1, 300] = -np.inf; variants.append(v)
    v = base.copy(); v[0, 7] = np.nan; v[1, 256] = np.nan; v[1, 16] = np.nan; variants.append(v)
    v = np.round(base * 4) * np.float32(0.5); variants.append(v.astype(np.float32))
    for x in variants:
        for c in (512, 300, 17):
            xx = np.ascontiguousarray(x[:, :c])
            assert np.array_equal(orc.quantize(fmt, xx), ref.quantize(fmt, xx))


MARGINS = {"Q8_0": (64, 0.5), "Q4_0": (128, 4.0), "Q2_K": (256, 10.0), "Q3_K": (256, 15.0),
           "Q4_K": (256, 8.0), "Q5_K": (256, 5.0), "Q6_K": (256, 4.0)}  # quantization_test.cpp:74-100


@pytest.mark.parametrize("fmt", FORMATS)
def test_oracle_roundtrip_margins(orc, fmt):
    count, margin = MARGINS[fmt]
    i = np.arange(count)
    v = ((i - count // 2) * 0.5).astype(np.float32)
    x = np.where((i // 8) % 2 == 0, v, -v).astype(np.float32)
    d = orc.dequantize(fmt, orc.quantize(fmt, x), 1, count)[0]
    assert np.abs(d - x).max() <= margin
