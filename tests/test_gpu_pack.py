"""Pack and dequant kernels vs the oracle and the golden fixtures: bit-exact."""
import zlib

import numpy as np
import pytest

from conftest import FORMATS, gen
from test_oracle import load_golden

pytestmark = pytest.mark.gpu


def gpu_pack(fmt, x):
    import torch
    import axon_b200 as ax
    F = ax.QuantFormat[fmt]
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    rows, cols = (1, x.shape[0]) if x.ndim == 1 else x.shape
    q = torch.full((ax.quantized_size_2d(rows, cols, F),), 0xA5, dtype=torch.uint8, device="cuda")
    ax.quantize(q, xt, F)
    return q


def gpu_dequant(fmt, q, rows, cols):
    import torch
    import axon_b200 as ax
    qt = q if isinstance(q, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(q)).cuda()
    out = torch.full((rows, cols), float("nan"), dtype=torch.float32, device="cuda")
    ax.dequantize(out, qt, ax.QuantFormat[fmt])
    return out


@pytest.mark.parametrize("fmt", FORMATS)
def test_pack_matches_golden(cuda, fmt):
    for name, g in load_golden(fmt).items():
        q = gpu_pack(fmt, g["x"]).cpu().numpy()
        assert np.array_equal(q, g["q"]), f"{fmt}/{name}: {np.count_nonzero(q != g['q'])} bytes differ"
        d = gpu_dequant(fmt, g["q"], *g["x"].shape).cpu().numpy()
        assert np.array_equal(d.view(np.uint32), g["deq"].view(np.uint32)), f"{fmt}/{name}: dequant differs"


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("kind", ["sweep", "w002", "outlier"])
def test_pack_matches_oracle_random(cuda, orc, fmt, kind):
    rng = np.random.default_rng(zlib.crc32(f"{fmt}/{kind}".encode()))
    for shape in ((256, 4096), (7, 1000), (3, 11008), (5, 33), (1, 8), (64, 256)):
        x = gen(rng, shape, kind)
        q = gpu_pack(fmt, x).cpu().numpy()
        qo = orc.quantize(fmt, x)
        assert np.array_equal(q, qo), f"{fmt} {kind} {shape}: {np.count_nonzero(q != qo)} bytes differ"
        d = gpu_dequant(fmt, qo, *shape).cpu().numpy()
        do = orc.dequantize(fmt, qo, *shape)
        assert np.array_equal(d.view(np.uint32), do.view(np.uint32)), f"{fmt} {kind} {shape}: dequant differs"


@pytest.mark.parametrize("fmt", FORMATS)
def test_pack_edge_values(cuda, orc, fmt):
    rng = np.random.default_rng(5)
    base = rng.standard_normal((2, 512)).astype(np.float32)
    variants = [np.zeros_like(base), np.full_like(base, 3.0), np.full_like(base, -0.7),
                base * np.float32(1e7), base * np.float32(1e-6), base * np.float32(1e-39),
                (np.round(base * 4) * np.float32(0.5)).astype(np.float32)]
    v = base.copy(); v[0, 5] = np.inf; v[1, 300] = -np.inf; variants.append(v)
    v = base.copy(); v[0, 7] = np.nan; v[1, 256] = np.nan; v[1, 16] = np.nan; v[0, 32] = np.nan; variants.append(v)
    v = base.copy(); v[:, :16] = 0; v[:, 40:56] = 100.0; variants.append(v)
    for i, x in enumerate(variants):
        for c in (512, 300, 17):
            xx = np.ascontiguousarray(x[:, :c])
            q = gpu_pack(fmt, xx).cpu().numpy()
            qo = orc.quantize(fmt, xx)
            assert np.array_equal(q, qo), f"{fmt} variant {i} cols {c}"
            d = gpu_dequant(fmt, qo, *xx.shape).cpu().numpy()
            do = orc.dequantize(fmt, qo, *xx.shape)
            assert np.array_equal(d.view(np.uint32), do.view(np.uint32)), f"{fmt} variant {i} cols {c} dequant"


@pytest.mark.parametrize("fmt", FORMATS)
def test_pack_1d_and_unaligned_buffers(cuda, orc, fmt):
    import torch
    import axon_b200 as ax
    rng = np.random.default_rng(3)
    x = gen(rng, 5000, "sweep")
    assert np.array_equal(gpu_pack(fmt, x).cpu().numpy(), orc.quantize(fmt, x))
    # src starting 4 bytes into an allocation, dst 2 bytes in: the slow paths
    F = ax.QuantFormat[fmt]
    xs = torch.from_numpy(gen(rng, (9, 700), "randn")).cuda()
    big = torch.empty(xs.numel() + 1, dtype=torch.float32, device="cuda")
    big[1:].copy_(xs.flatten())
    n = ax.quantized_size_2d(9, 700, F)
    qbuf = torch.zeros(n + 2, dtype=torch.uint8, device="cuda")
    ax.quantize(qbuf[2:], big[1:].view(9, 700), F)
    assert np.array_equal(qbuf[2:].cpu().numpy(), orc.quantize(fmt, xs.cpu().numpy()))


@pytest.mark.parametrize("fmt", FORMATS)
def test_pack_full_size_sampled(cuda, orc, fmt):
    """A 2^26-element tensor (rows of 4096) packed on the GPU; 256 random rows
    compared byte-for-byte with the oracle, and dequant(pack(x)) of the whole
    tensor checked against the oracle's dequant of those rows."""
    import torch
    import axon_b200 as ax
    F = ax.QuantFormat[fmt]
    rows, cols = 1 << 14, 4096
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(rows, cols, device="cuda", generator=g)
    m = torch.rand(rows, cols, device="cuda", generator=g) < 0.01
    x[m] = (torch.rand(int(m.sum().item()), device="cuda", generator=g) * 100 - 50)
    q = torch.empty(ax.quantized_size_2d(rows, cols, F), dtype=torch.uint8, device="cuda")
    ax.quantize(q, x, F)
    d = torch.empty(rows, cols, device="cuda")
    ax.dequantize(d, q, F)
    rb = ax.quantized_size_2d(1, cols, F)
    sel = np.sort(np.random.default_rng(0).choice(rows, 256, replace=False))
    xs = x[torch.from_numpy(sel).cuda()].cpu().numpy()
    qs = q.view(rows, rb)[torch.from_numpy(sel).cuda()].cpu().numpy()
    qo = orc.quantize(fmt, xs)
    assert np.array_equal(qs.ravel(), qo)
    ds = d[torch.from_numpy(sel).cuda()].cpu().numpy()
    assert np.array_equal(ds.view(np.uint32), orc.dequantize(fmt, qo, 256, cols).view(np.uint32))
