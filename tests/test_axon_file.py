""".axon files on the host (no GPU): the library's reader and writer against
files written by the reference's own serializer (src/core/serialize.cpp,
compiled into oracle/_ref; fixtures made by tests/golden/make_axon_golden.py).

The reference's load_tensor cannot load its own packed files (it ignores
quant_type, serialize.cpp:112-116, and fails with "Tensor data size
mismatch"); the fixtures record that, and here the same files load with
their format.  Files this library writes are byte-identical to the
reference's for the same tensors.
"""
import ctypes
import os
import struct

import numpy as np
import pytest
import torch

from conftest import ROOT

GOLD = os.path.join(ROOT, "tests", "golden")
EXP = np.load(os.path.join(GOLD, "axon_expect.npz"))


def gold(name):
    return os.path.join(GOLD, name)


def test_records_of_reference_files():
    import axon_b200 as ax
    Q = ax.QuantFormat
    r = ax.axon_records(gold("axon_q4k.axon"))
    assert [(x.name, x.dtype, x.quant, x.shape, x.layout, x.data_bytes) for x in r] == \
        [("data", 0, Q.Q4_K, (4, 512), "rows", 1152)]
    r = ax.axon_records(gold("axon_q8_0_flat.axon"))
    assert [(x.name, x.quant, x.shape, x.layout, x.data_bytes) for x in r] == [("data", Q.Q8_0, (3, 40), "flat", 136)]
    r = ax.axon_records(gold("axon_f32.axon"))
    assert [(x.name, x.dtype, x.quant, x.shape, x.layout) for x in r] == [("data", 0, Q.NONE, (2, 3), "plain")]
    r = ax.axon_records(gold("axon_checkpoint.axon"))
    assert [(x.name, x.quant, x.shape, x.layout) for x in r] == [
        ("mlp.w_gate", Q.Q4_K, (8, 256), "rows"), ("mlp.w_down", Q.Q6_K, (4, 512), "rows"),
        ("mlp.bias", Q.NONE, (8,), "plain"), ("ids", Q.NONE, (5,), "plain")]
    assert r[3].dtype == 2  # Int32


def test_reference_loader_rejects_its_own_packed_files():
    """The gap this reader closes, as recorded from the reference itself."""
    assert not bool(EXP["axon_q4k_ref_load_ok"])
    assert not bool(EXP["axon_q8_0_flat_ref_load_ok"])
    assert bool(EXP["axon_f32_ref_load_ok"])


def test_load_reference_files_into_host_memory():
    import axon_b200 as ax
    t = ax.load_tensor(gold("axon_q4k.axon"), device="cpu")
    assert isinstance(t, ax.QTensor) and t.shape == (4, 512) and t.fmt == ax.QuantFormat.Q4_K
    assert np.array_equal(t.data.numpy(), EXP["q4k_data"])
    t = ax.load_tensor(gold("axon_q8_0_flat.axon"), device="cpu")
    assert t.shape == (1, 120) and np.array_equal(t.data.numpy(), EXP["q8_0_flat_data"])
    t = ax.load_tensor(gold("axon_f32.axon"), device="cpu")
    assert t.dtype == torch.float32 and np.array_equal(t.numpy(), EXP["f32_data"])
    ck = ax.load_axon(gold("axon_checkpoint.axon"), device="cpu")
    assert list(ck) == ["mlp.w_gate", "mlp.w_down", "mlp.bias", "ids"]
    assert np.array_equal(ck["mlp.w_gate"].data.numpy(), EXP["ckpt_w_gate"])
    assert np.array_equal(ck["mlp.w_down"].data.numpy(), EXP["ckpt_w_down"])
    assert np.array_equal(ck["mlp.bias"].numpy(), EXP["ckpt_bias"])
    assert ck["ids"].dtype == torch.int32 and np.array_equal(ck["ids"].numpy(), EXP["ckpt_ids"])


def test_written_files_are_byte_identical_to_the_reference(tmp_path):
    import axon_b200 as ax
    Q = ax.QuantFormat
    p = str(tmp_path / "q4k.axon")
    ax.save_tensor(ax.QTensor(torch.from_numpy(EXP["q4k_data"].copy()), (4, 512), Q.Q4_K), p)
    assert open(p, "rb").read() == open(gold("axon_q4k.axon"), "rb").read()
    p = str(tmp_path / "f32.axon")
    ax.save_tensor(torch.from_numpy(EXP["f32_data"].copy()), p)
    assert open(p, "rb").read() == open(gold("axon_f32.axon"), "rb").read()
    p = str(tmp_path / "ck.axon")
    ax.save_axon(p, {"mlp.w_gate": ax.QTensor(torch.from_numpy(EXP["ckpt_w_gate"].copy()), (8, 256), Q.Q4_K),
                     "mlp.w_down": ax.QTensor(torch.from_numpy(EXP["ckpt_w_down"].copy()), (4, 512), Q.Q6_K),
                     "mlp.bias": torch.from_numpy(EXP["ckpt_bias"].copy()),
                     "ids": torch.from_numpy(EXP["ckpt_ids"].copy())})
    assert open(p, "rb").read() == open(gold("axon_checkpoint.axon"), "rb").read()


def test_flat_record_written_through_the_c_abi(tmp_path):
    """A flat-packed record (rows not whole blocks) through axq_axon_save."""
    import axon_b200 as ax
    from axon_b200._capi import AxonTensorInfo, check
    info = AxonTensorInfo()
    info.name, info.dtype, info.quant, info.ndims = b"data", 0, int(ax.QuantFormat.Q8_0), 2
    info.shape[0], info.shape[1] = 3, 40
    info.data_bytes = 136
    data = np.ascontiguousarray(EXP["q8_0_flat_data"])
    ptrs = (ctypes.c_void_p * 1)(data.ctypes.data)
    p = str(tmp_path / "flat.axon")
    check(ax.lib().axq_axon_save(p.encode(), 1, ctypes.addressof(info), ctypes.cast(ptrs, ctypes.c_void_p), None))
    assert open(p, "rb").read() == open(gold("axon_q8_0_flat.axon"), "rb").read()


def test_reference_reads_plain_files_written_here(tmp_path):
    import oracle
    import axon_b200 as ax
    ref = oracle.ref()
    if ref is None:
        pytest.skip("reference library not built here")
    x = torch.arange(12, dtype=torch.float32).reshape(3, 4) * 0.5
    p = str(tmp_path / "x.axon")
    ax.save_tensor(x, p)
    data, err = ref.load_tensor(p)
    assert err is None and np.array_equal(data.view(np.float32), x.numpy().ravel())


def _corrupt(tmp_path, name, mutate):
    raw = bytearray(open(gold("axon_checkpoint.axon"), "rb").read())
    mutate(raw)
    p = str(tmp_path / name)
    open(p, "wb").write(bytes(raw))
    return p


@pytest.mark.parametrize("case,fragment", [
    ("magic", "bad magic"),
    ("version", "unsupported .axon version"),
    ("truncated", "file ends inside the data"),
    ("size", "matches neither"),
    ("dtype", "unknown dtype"),
    ("quant", "unknown quant_type"),
    ("name", "name longer"),
    ("huge", "too many elements"),
])
def test_malformed_files_are_refused_with_a_message(tmp_path, case, fragment):
    import axon_b200 as ax
    first = 12  # magic, version, count
    muts = {
        "magic": lambda r: r.__setitem__(slice(0, 4), b"AXOM"),
        "version": lambda r: r.__setitem__(slice(4, 8), struct.pack("<I", 2)),
        "truncated": lambda r: r.__delitem__(slice(len(r) - 3, len(r))),
        # first record: name "mlp.w_gate" (10 bytes), 2 dims -> data_bytes at 12 + 16 + 10 + 16
        "size": lambda r: r.__setitem__(slice(first + 42, first + 50), struct.pack("<Q", 1151)),
        # the bias record is plain: give it an unknown dtype (its header follows the two packed ones)
        "dtype": None,
        "quant": lambda r: r.__setitem__(slice(first + 8, first + 12), struct.pack("<I", 9)),
        "name": lambda r: r.__setitem__(slice(first, first + 4), struct.pack("<I", 300)),
        # first record's two dims (after its 16-byte header and 10-byte name): 2^40 x 2^40 overflows int64
        "huge": lambda r: r.__setitem__(slice(first + 26, first + 42), struct.pack("<QQ", 1 << 40, 1 << 40)),
    }
    if case == "dtype":
        recs = ax.axon_records(gold("axon_checkpoint.axon"))
        bias = recs[2]
        hdr = bias.offset - 8 - 8 * len(bias.shape) - len(bias.name) - 16
        muts["dtype"] = lambda r: r.__setitem__(slice(hdr + 4, hdr + 8), struct.pack("<I", 11))
    p = _corrupt(tmp_path, case + ".axon", muts[case])
    with pytest.raises(ax.AxqError, match=fragment) as e:
        ax.axon_records(p)
    assert e.value.status == ax.Status.ERR_INVALID


def test_read_argument_errors(tmp_path):
    import axon_b200 as ax
    from axon_b200._capi import check
    L = ax.lib()
    h = ctypes.c_void_p()
    n = ctypes.c_uint32()
    with pytest.raises(ax.AxqError, match="failed to open"):
        check(L.axq_axon_open(str(tmp_path / "missing.axon").encode(), ctypes.byref(h), ctypes.byref(n)))
    check(L.axq_axon_open(gold("axon_q4k.axon").encode(), ctypes.byref(h), ctypes.byref(n)))
    try:
        small = np.zeros(1000, dtype=np.uint8)
        with pytest.raises(ax.AxqError, match="destination holds 1000"):
            check(L.axq_axon_read(h, 0, small.ctypes.data, small.nbytes, None))
        with pytest.raises(ax.AxqError, match="out of range"):
            check(L.axq_axon_read(h, 1, small.ctypes.data, small.nbytes, None))
    finally:
        L.axq_axon_close(h)


def test_edge_records(tmp_path):
    """A file with no tensors, a 0-d (scalar) tensor, an empty tensor and a
    packed tensor with an empty row range, each written by the reference's
    writer where it can express them, read back here."""
    import oracle
    import axon_b200 as ax
    ref = oracle.ref()
    p0 = str(tmp_path / "none.axon")
    open(p0, "wb").write(struct.pack("<III", 0x4E4F5841, 1, 0))  # what save_checkpoint writes for no parameters
    assert ax.axon_records(p0) == [] and ax.load_axon(p0, device="cpu") == {}
    with pytest.raises(ax.AxqError, match="no tensors"):
        ax.load_tensor(p0, device="cpu")
    ps = str(tmp_path / "scalar.axon")
    pe = str(tmp_path / "empty.axon")
    if ref is not None:
        ref.save_tensor(ps, [], 0, 0, np.array([2.5], dtype=np.float32))
        ref.save_tensor(pe, [0, 4], 0, 0, np.zeros(0, dtype=np.float32))
    else:
        ax.save_tensor(torch.tensor(2.5), ps)
        ax.save_tensor(torch.zeros(0, 4), pe)
    s = ax.load_tensor(ps, device="cpu")
    assert s.shape == () and float(s) == 2.5
    e = ax.load_tensor(pe, device="cpu")
    assert tuple(e.shape) == (0, 4)
    pq = str(tmp_path / "q0.axon")
    ax.save_tensor(ax.QTensor(torch.zeros(1, dtype=torch.uint8), (0, 256), ax.QuantFormat.Q4_K), pq)
    r = ax.axon_records(pq)[0]
    assert r.layout == "rows" and r.data_bytes == 0 and r.shape == (0, 256)
