"""fp32 matmul for unquantized A (axq_matmul_f32, this library's tiled fp32
kernel) against the reference's own cpu::matmul
(src/backend/cpu_backend.cpp:116-173, compiled into oracle/_ref) and a
float64 product.  The sums are the same fp32 products added in a different
order, so the tolerance is float rounding over K terms:
max|y - y_ref| <= 2e-5 * max|y_ref|."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-5


@pytest.mark.parametrize("M,K,N", [(1, 64, 1), (64, 4096, 3), (300, 1000, 257), (512, 512, 512), (7, 33, 130),
                                   (129, 17, 131), (256, 2048, 384), (1000, 3, 5)])
def test_f32_matmul_matches_reference(cuda, M, K, N):
    import oracle
    import axon_b200 as ax
    rng = np.random.default_rng(M * 7 + K + N)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    out = torch.full((M, N), float("nan"), device="cuda")
    ax.matmul(out, torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda())
    y = out.cpu().numpy()
    y64 = a.astype(np.float64) @ b.astype(np.float64)
    assert np.abs(y - y64).max() <= TOL * np.abs(y64).max()
    ref = oracle.ref()
    if ref is not None:
        y_ref = ref.matmul_f32(a, b)
        assert np.abs(y - y_ref).max() <= TOL * np.abs(y_ref).max()


def test_f32_matmul_edges_and_errors(cuda):
    import axon_b200 as ax
    out = torch.full((3, 4), float("nan"), device="cuda")
    ax.matmul(out, torch.empty(3, 0, device="cuda"), torch.empty(0, 4, device="cuda"))  # empty sum
    assert torch.equal(out.cpu(), torch.zeros(3, 4))
    with pytest.raises(ax.AxqError, match="inner dimensions"):
        ax.matmul(out, torch.zeros(3, 5, device="cuda"), torch.zeros(6, 4, device="cuda"))
    host = torch.zeros(5, 4)
    L = ax.lib()
    st = L.axq_matmul_f32(torch.zeros(3, 5, device="cuda").data_ptr(), host.data_ptr(), out.data_ptr(), 3, 5, 4, None)
    assert st == ax.Status.ERR_INVALID


def test_generic_matmul_routes_packed_a_to_the_quantized_kernel(cuda, orc):
    import axon_b200 as ax
    from conftest import gen, rel_err
    rng = np.random.default_rng(9)
    q = orc.quantize("Q4_K", gen(rng, (64, 512), "randn"))
    b = rng.standard_normal((512, 5)).astype(np.float32)
    a = ax.QTensor(torch.from_numpy(q).cuda(), (64, 512), ax.QuantFormat.Q4_K)
    out = torch.empty(64, 5, device="cuda")
    ax.matmul(out, a, torch.from_numpy(b).cuda())
    assert rel_err(out.cpu().numpy(), orc.matmul("Q4_K", q, b, 64, 512)) <= 1e-3
