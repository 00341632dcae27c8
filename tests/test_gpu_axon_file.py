""".axon files straight into device memory: files written by the reference's
serializer (tests/golden/axon_*.axon) load onto the GPU with their packed
format and feed the quantized kernels, checked against the oracle; device
tensors saved and loaded back are identical (several staging chunks)."""
import os

import numpy as np
import torch
import pytest

from conftest import ROOT, rel_err

pytestmark = pytest.mark.gpu

GOLD = os.path.join(ROOT, "tests", "golden")
EXP = np.load(os.path.join(GOLD, "axon_expect.npz"))
TOL = 1e-3  # max|y - y_ref| <= TOL * max|y_ref|, the matmul parity rule


def test_reference_checkpoint_to_device_feeds_the_kernels(cuda, orc):
    import axon_b200 as ax
    ck = ax.load_axon(os.path.join(GOLD, "axon_checkpoint.axon"))
    wg, wd = ck["mlp.w_gate"], ck["mlp.w_down"]
    assert wg.data.is_cuda and wg.fmt == ax.QuantFormat.Q4_K and wg.shape == (8, 256)
    assert np.array_equal(wg.data.cpu().numpy(), EXP["ckpt_w_gate"])
    # the loaded packed matrix in a matmul, against the oracle on the same bytes
    x = np.random.default_rng(3).standard_normal((2, 256)).astype(np.float32)
    y = ax.linear_q(torch.from_numpy(x).cuda(), wg).cpu().numpy()
    y_ref = orc.matmul("Q4_K", EXP["ckpt_w_gate"], np.ascontiguousarray(x.T), 8, 256).T
    assert rel_err(y, y_ref) <= TOL
    # and decoded bit for bit
    d = torch.empty(4, 512, device="cuda")
    ax.dequantize(d, wd)
    assert np.array_equal(d.cpu().numpy().view(np.uint32),
                          orc.dequantize("Q6_K", EXP["ckpt_w_down"], 4, 512).view(np.uint32))
    assert torch.equal(ck["mlp.bias"].cpu(), torch.from_numpy(EXP["ckpt_bias"]))
    assert torch.equal(ck["ids"].cpu(), torch.from_numpy(EXP["ckpt_ids"]))


def test_flat_packed_file_decodes_as_one_row(cuda, orc):
    import axon_b200 as ax
    t = ax.load_tensor(os.path.join(GOLD, "axon_q8_0_flat.axon"))
    assert t.shape == (1, 120)
    d = torch.empty(120, device="cuda")
    ax.dequantize(d, t)
    ref = orc.dequantize("Q8_0", EXP["q8_0_flat_data"], 1, 120)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), ref.ravel().view(np.uint32))


def test_device_round_trip_over_several_staging_chunks(cuda, tmp_path):
    """A 18.9 MB packed matrix and a 20 MB fp32 tensor (staging chunks are
    8 MiB) saved from device memory and loaded back on another stream."""
    import axon_b200 as ax
    g = torch.Generator(device="cuda").manual_seed(7)
    w = ax.QTensor.empty(4096, 8192, ax.QuantFormat.Q4_K)
    ax.quantize(w, torch.randn(4096, 8192, device="cuda", generator=g) * 0.02, ax.QuantFormat.Q4_K)
    f = torch.randn(1000, 5000, device="cuda", generator=g)
    p = str(tmp_path / "big.axon")
    ax.save_axon(p, {"w": w, "f": f})
    s = torch.cuda.Stream()
    back = ax.load_axon(p, stream=s)
    s.synchronize()
    assert back["w"].shape == (4096, 8192) and back["w"].fmt == ax.QuantFormat.Q4_K
    n = ax.quantized_size_2d(4096, 8192, ax.QuantFormat.Q4_K)
    assert torch.equal(back["w"].data[:n], w.data[:n])
    assert torch.equal(back["f"], f)
    for _ in range(2):  # loaded again, each time through a fresh handle
        again = ax.load_tensor(p)
        assert torch.equal(again.data[:n], w.data[:n])
