"""Quantized matmul kernels vs the oracle (max|y - y_ref| <= 1e-3 max|y_ref|)."""
import numpy as np
import pytest

from conftest import FORMATS, gen, rel_err
from test_oracle import load_golden

pytestmark = pytest.mark.gpu

TOL = 1e-3  # max-abs error relative to the reference output's L-inf norm


def gpu_matmul(fmt, q, b, M, K, b_tokmajor=False, out_tokmajor=False):
    import torch
    import axon_b200 as ax
    qt = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    bt = torch.from_numpy(np.ascontiguousarray(b.T if b_tokmajor else b)).cuda()
    N = b.shape[1]
    out = torch.full((N, M) if out_tokmajor else (M, N), float("nan"), device="cuda")
    ax.matmul_q(out, qt, bt, ax.QuantFormat[fmt], M, K, b_tokmajor=b_tokmajor, out_tokmajor=out_tokmajor)
    y = out.cpu().numpy()
    return y.T if out_tokmajor else y


@pytest.mark.parametrize("fmt", FORMATS)
def test_matmul_matches_golden(cuda, fmt):
    for name, g in load_golden(fmt).items():
        rows, cols = g["x"].shape
        y = gpu_matmul(fmt, g["q"], g["b"], rows, cols)
        assert rel_err(y, g["mm"]) <= TOL, (fmt, name, rel_err(y, g["mm"]))


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("N", [1, 2, 3, 4, 5, 8, 17])
def test_matmul_matches_oracle(cuda, orc, fmt, N):
    rng = np.random.default_rng(100 + N)
    for (M, K, kind) in ((64, 4096, "w002"), (37, 1000, "randn"), (16, 11008, "randn"), (9, 300, "outlier"),
                         (5, 32, "randn")):
        W = gen(rng, (M, K), kind)
        q = orc.quantize(fmt, W)
        B = rng.standard_normal((K, N)).astype(np.float32)
        y_ref = orc.matmul(fmt, q, B, M, K)
        y = gpu_matmul(fmt, q, B, M, K)
        assert rel_err(y, y_ref) <= TOL, (fmt, M, K, N, kind, rel_err(y, y_ref))


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("N", [4, 6])
def test_matmul_token_major_layouts(cuda, orc, fmt, N):
    rng = np.random.default_rng(9 + N)
    M, K = 48, 2048
    q = orc.quantize(fmt, gen(rng, (M, K), "randn"))
    B = rng.standard_normal((K, N)).astype(np.float32)
    y_ref = orc.matmul(fmt, q, B, M, K)
    for bt in (False, True):
        for ot in (False, True):
            assert rel_err(gpu_matmul(fmt, q, B, M, K, bt, ot), y_ref) <= TOL, (bt, ot)


def test_matmul_zero_weights_give_exact_zero(cuda, orc):
    # Q6_K at sigma=0.02: every fp16 super-scale flushes to 0, the reference
    # output is exactly 0 and so must ours be.
    rng = np.random.default_rng(1)
    M, K = 32, 4096
    q = orc.quantize("Q6_K", gen(rng, (M, K), "w002"))
    B = rng.standard_normal((K, 2)).astype(np.float32)
    y_ref = orc.matmul("Q6_K", q, B, M, K)
    assert np.abs(y_ref).max() == 0.0
    assert np.abs(gpu_matmul("Q6_K", q, B, M, K)).max() == 0.0


def test_matmul_errors(cuda):
    import torch
    import axon_b200 as ax
    F = ax.QuantFormat.Q4_K
    q = ax.QTensor.empty(8, 256, F)
    b = torch.zeros(256, 2, device="cuda")
    out = torch.zeros(8, 2, device="cuda")
    with pytest.raises(ax.AxqError) as e:
        ax.matmul_q(out, q, torch.zeros(255, 2, device="cuda"))
    assert "inner dimension" in str(e.value)
    with pytest.raises(ax.AxqError):
        ax.matmul_q4(out, q, b)  # wrong format for the fixed-format entry
    # host pointer through the raw C ABI: rejected, not launched
    host = np.zeros(64, dtype=np.float32)
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    st = ax.lib().axq_matmul(int(F), q.data.data_ptr(), host.ctypes.data, out.data_ptr(), 8, 256, 2, 0,
                             ws.data_ptr(), ws.numel(), None)
    assert st == ax.Status.ERR_INVALID
    assert b"host memory" in ax.lib().axq_last_error() or b"not a CUDA" in ax.lib().axq_last_error()
    st = ax.lib().axq_matmul(int(F), q.data.data_ptr(), b.data_ptr(), out.data_ptr(), 8, 256, 2, 0,
                             ws.data_ptr(), 16, None)
    assert st == ax.Status.ERR_WORKSPACE
    torch.cuda.synchronize()


@pytest.mark.parametrize("fmt", ["Q2_K", "Q3_K", "Q5_K"])
def test_matmul_full_size_rows_sampled(cuda, orc, fmt):
    """W[28672 x 8192] (the large-config shape) packed and multiplied on the
    GPU at M=1 and 8; 64 random output rows compared with the oracle."""
    import torch
    import axon_b200 as ax
    F = ax.QuantFormat[fmt]
    rows, K = 28672, 8192
    g = torch.Generator(device="cuda").manual_seed(9)
    W = torch.randn(rows, K, device="cuda", generator=g) * 0.02
    m = torch.rand(rows, K, device="cuda", generator=g) < 0.001
    W[m] = torch.randn(int(m.sum().item()), device="cuda", generator=g) * 0.5
    q = torch.empty(ax.quantized_size_2d(rows, K, F), dtype=torch.uint8, device="cuda")
    ax.quantize(q, W, F)
    rb = ax.quantized_size_2d(1, K, F)
    sel = np.sort(np.random.default_rng(1).choice(rows, 64, replace=False))
    qs = q.view(rows, rb)[torch.from_numpy(sel).cuda()].cpu().numpy().ravel()
    for N in (1, 8):
        B = torch.randn(K, N, device="cuda", generator=g)
        out = torch.empty(rows, N, device="cuda")
        ax.matmul_q(out, q, B, F, rows, K)
        y_ref = orc.matmul(fmt, qs, B.cpu().numpy(), 64, K)
        assert rel_err(out[torch.from_numpy(sel).cuda()].cpu().numpy(), y_ref) <= TOL


@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("offset", [2, 6, 16])
def test_matmul_unaligned_weight_buffer(cuda, orc, fmt, offset):
    """Packed weights starting at an odd 2-byte offset inside their buffer
    (the copy pipeline then takes its byte-copy and any-alignment paths)."""
    import torch
    import axon_b200 as ax
    rng = np.random.default_rng(offset)
    for M, K in ((33, 4096), (20, 11008), (7, 700)):
        q = orc.quantize(fmt, gen(rng, (M, K), "randn"))
        buf = torch.zeros(q.size + offset, dtype=torch.uint8, device="cuda")
        buf[offset:].copy_(torch.from_numpy(q))
        B = rng.standard_normal((K, 3)).astype(np.float32)
        out = torch.empty(M, 3, device="cuda")
        ax.matmul_q(out, buf[offset:], torch.from_numpy(B).cuda(), ax.QuantFormat[fmt], M, K)
        assert rel_err(out.cpu().numpy(), orc.matmul(fmt, q, B, M, K)) <= TOL, (fmt, offset, M, K)


# ---- batched path (N > 4 activation columns: tcgen05 tensor-core GEMM) ----

@pytest.mark.parametrize("fmt", FORMATS)
@pytest.mark.parametrize("M,K,N", [(128, 4096, 16), (200, 1000, 9), (256, 4096, 64), (130, 11008, 32),
                                   (384, 2048, 256), (128, 512, 512), (64, 300, 40)])
def test_gemm_matches_oracle(cuda, orc, fmt, M, K, N):
    rng = np.random.default_rng(M * 7 + N)
    q = orc.quantize(fmt, gen(rng, (M, K), "randn"))
    B = rng.standard_normal((K, N)).astype(np.float32)
    y_ref = orc.matmul(fmt, q, B, M, K)
    y = gpu_matmul(fmt, q, B, M, K)
    assert rel_err(y, y_ref) <= TOL, (fmt, M, K, N, rel_err(y, y_ref))


@pytest.mark.parametrize("fmt", ["Q4_0", "Q4_K", "Q6_K"])
def test_gemm_token_major_and_workload_distribution(cuda, orc, fmt):
    rng = np.random.default_rng(21)
    M, K, N = 256, 4096, 48
    q = orc.quantize(fmt, gen(rng, (M, K), "w002"))
    B = rng.standard_normal((K, N)).astype(np.float32)
    y_ref = orc.matmul(fmt, q, B, M, K)
    for bt in (False, True):
        for ot in (False, True):
            assert rel_err(gpu_matmul(fmt, q, B, M, K, bt, ot), y_ref) <= TOL, (bt, ot)


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "Q8_0", "Q2_K"])
@pytest.mark.parametrize("N", [1, 3, 24])
def test_linear_with_bias_matches_oracle(cuda, orc, fmt, N):
    """Quantized Linear through the C ABI (axq_linear): y[N x M] = x W^T + bias
    against the oracle's W . x^T transposed plus the bias, and without bias."""
    import torch
    import axon_b200 as ax
    rng = np.random.default_rng(N * 13 + len(fmt))
    M, K = 200, 2048
    q = orc.quantize(fmt, gen(rng, (M, K), "randn"))
    x = rng.standard_normal((N, K)).astype(np.float32)
    bias = rng.standard_normal(M).astype(np.float32)
    w = ax.QTensor(torch.from_numpy(q).cuda(), (M, K), ax.QuantFormat[fmt])
    y_mm = orc.matmul(fmt, q, np.ascontiguousarray(x.T), M, K).T
    y = ax.linear_q(torch.from_numpy(x).cuda(), w, bias=torch.from_numpy(bias).cuda()).cpu().numpy()
    assert rel_err(y, y_mm + bias) <= TOL
    y0 = ax.linear_q(torch.from_numpy(x).cuda(), w).cpu().numpy()
    assert rel_err(y0, y_mm) <= TOL


def test_linear_errors(cuda):
    import torch
    import axon_b200 as ax
    w = ax.QTensor.empty(16, 256, ax.QuantFormat.Q4_K)
    x = torch.zeros(2, 256, device="cuda")
    with pytest.raises(ax.AxqError, match="bias must have 16"):
        ax.linear_q(x, w, bias=torch.zeros(15, device="cuda"))
    with pytest.raises(ax.AxqError, match=r"x must be \[N x 256\]"):
        ax.linear_q(torch.zeros(2, 255, device="cuda"), w)
    host = np.zeros(16, dtype=np.float32)
    L = ax.lib()
    y = torch.empty(2, 16, device="cuda")
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    st = L.axq_linear(int(ax.QuantFormat.Q4_K), w.data.data_ptr(), x.data_ptr(), host.ctypes.data, y.data_ptr(),
                      16, 256, 2, ws.data_ptr(), ws.numel(), None)
    assert st == ax.Status.ERR_INVALID and b"bias" in L.axq_last_error()
    torch.cuda.synchronize()
