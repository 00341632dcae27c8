"""Generate the golden fixtures for the quantized-matmul path.

Run in a container where the reference sources exist, after
``make -C oracle`` built ``oracle/_ref/libaxon_ref.so`` from them:

    python tests/golden/make_golden.py

For every format it stores small seeded inputs, the reference's packed
bytes (``cpu::quantize``), its dequantized values (``cpu::dequantize``) and
its matmul outputs (``cpu::matmul_q*``; Q8_0 via dequantize + ``cpu::matmul``)
in ``tests/golden/golden_<FMT>.npz``.  The inputs include the ramp of the
reference's own round-trip test (tests/backend/quantization_test.cpp:46-52).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402


def ramp(count):
    # quantization_test.cpp:46-52: v=(i-count/2)*0.5, sign flipped every 8.
    i = np.arange(count, dtype=np.int64)
    v = ((i - count // 2).astype(np.float32) * np.float32(0.5)).astype(np.float32)
    return np.where((i // 8) % 2 == 0, v, -v).astype(np.float32)


def cases(fmt, rng):
    be = oracle.BLOCK_ELEMS[fmt]
    out = {}
    out["ramp"] = ramp(512 if be == 256 else 64).reshape(1, -1)
    out["randn"] = rng.standard_normal((6, 512)).astype(np.float32)
    x = rng.standard_normal((4, 768)).astype(np.float32)
    m = rng.random(x.shape) < 0.01
    x[m] = rng.uniform(-50, 50, m.sum()).astype(np.float32)
    out["sweep"] = x
    out["w002"] = (rng.standard_normal((5, 512)) * 0.02).astype(np.float32)
    out["tail"] = rng.standard_normal((3, 300)).astype(np.float32)
    out["short"] = rng.standard_normal((2, 17)).astype(np.float32)
    e = rng.standard_normal((4, 512)).astype(np.float32)
    e[0, :] = 0.0
    e[1, :] = 3.0
    e[2, :16] = 0.0
    e[2, 40:56] = 100.0
    e[3, ::17] = 1e-12
    out["edge"] = e
    return out


def main():
    ref = oracle.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libaxon_ref.so not built (needs the reference sources)")
    for fmt in oracle.FORMATS:
        rng = np.random.default_rng(1000 + oracle.FORMATS[fmt])
        arrs = {}
        for name, x in cases(fmt, rng).items():
            rows, cols = x.shape
            q = ref.quantize(fmt, x)
            d = ref.dequantize(fmt, q, rows, cols)
            b = rng.standard_normal((cols, 3)).astype(np.float32)
            mm = ref.matmul(fmt, q, b, rows, cols)
            arrs[f"{name}__x"] = x
            arrs[f"{name}__q"] = q
            arrs[f"{name}__deq"] = d
            arrs[f"{name}__b"] = b
            arrs[f"{name}__mm"] = mm
        path = os.path.join(HERE, f"golden_{fmt}.npz")
        np.savez_compressed(path, **arrs)
        print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
