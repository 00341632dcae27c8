"""Generate the .axon file fixtures (golden files written by the reference).

Run in a container where the reference sources exist, after
``make -C oracle`` built ``oracle/_ref/libaxon_ref.so`` (which includes the
reference's src/core/serialize.cpp and src/nn/module.cpp):

    python tests/golden/make_axon_golden.py

Every file is written by the reference's own serializer (save_tensor,
serialize.cpp:84-96; save_checkpoint, :125-148) from seeded data; packed
payloads come from the reference's quantizer (cpu::quantize).  The expected
contents go to ``tests/golden/axon_expect.npz``, and whether the reference's
own load_tensor accepts each file to ``axon_expect.npz`` too.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

FMT = oracle.FORMATS  # name -> QuantFormat ordinal


def main():
    ref = oracle.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libaxon_ref.so is missing: run make -C oracle with the reference present")
    rng = np.random.default_rng(20)
    exp = {}
    # 1. a packed Q4_K matrix [4 x 512], rows of whole blocks
    w = rng.standard_normal((4, 512)).astype(np.float32)
    q4k = ref.quantize("Q4_K", w)
    ref.save_tensor(os.path.join(HERE, "axon_q4k.axon"), [4, 512], 0, FMT["Q4_K"], q4k)
    exp["q4k_data"] = q4k
    # 2. a packed Q8_0 tensor [3 x 40] packed flat (rows are not whole blocks)
    x = rng.standard_normal((3, 40)).astype(np.float32)
    q8 = ref.quantize_1d("Q8_0", x)
    ref.save_tensor(os.path.join(HERE, "axon_q8_0_flat.axon"), [3, 40], 0, FMT["Q8_0"], q8)
    exp["q8_0_flat_data"] = q8
    exp["q8_0_flat_x"] = x
    # 3. a plain fp32 tensor [2 x 3] (the reference's own round-trip case)
    f = np.arange(6, dtype=np.float32).reshape(2, 3)
    ref.save_tensor(os.path.join(HERE, "axon_f32.axon"), [2, 3], 0, 0, f)
    exp["f32_data"] = f
    # 4. a checkpoint of four parameters: two packed matrices, a bias, indices
    g = rng.standard_normal((8, 256)).astype(np.float32)
    d = rng.standard_normal((4, 512)).astype(np.float32)
    qg, qd = ref.quantize("Q4_K", g), ref.quantize("Q6_K", d)
    bias = rng.standard_normal(8).astype(np.float32)
    ids = np.arange(5, dtype=np.int32) * 7
    ref.save_checkpoint(os.path.join(HERE, "axon_checkpoint.axon"), [
        ("mlp.w_gate", [8, 256], 0, FMT["Q4_K"], qg),
        ("mlp.w_down", [4, 512], 0, FMT["Q6_K"], qd),
        ("mlp.bias", [8], 0, 0, bias),
        ("ids", [5], 2, 0, ids),
    ])
    exp.update(ckpt_w_gate=qg, ckpt_w_down=qd, ckpt_bias=bias, ckpt_ids=ids, ckpt_gate_x=g, ckpt_down_x=d)
    # what the reference's own loader makes of each single-tensor file
    for name in ("axon_q4k", "axon_q8_0_flat", "axon_f32"):
        data, err = ref.load_tensor(os.path.join(HERE, name + ".axon"))
        exp[name + "_ref_load_ok"] = np.array(err is None)
    np.savez(os.path.join(HERE, "axon_expect.npz"), **exp)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.startswith("axon")))


if __name__ == "__main__":
    main()
