"""Packed weights on disk (apsi_b200.modelio): the reference's .apsim container, both directions.

* A checkpoint written by the reference's own save_model (tests/golden/ref_packed.apsim, made by
  tests/golden/make_golden.py) loads without re-quantising, its codes and scales bit-exact with the oracle's
  quantisation of the source arrays kept in the golden npz.
* A file written here loads back identically, keeps the B200 layout (rows, cols, group, [in, out] flag),
  rejects modified data, and -- where the reference is importable -- loads in the reference, whose dequantize
  gives the same float32 weights."""
import json
import os
import sys

import numpy as np
import pytest

from apsi_b200 import modelio
from apsi_b200.precision import QTensor, get_format, RuntimeErr
from oracle import lowbit_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "lowbit_golden.npz"))
REF_APSIM = os.path.join(HERE, "golden", "ref_packed.apsim")


def _q4(W, kn=False):
    packed, s32, s16 = O.quant_int4_g128(W)
    R, C = W.shape
    shape = (C, R) if kn else (R, C)
    return QTensor(packed.reshape(-1), s32.reshape(R, C // 128), get_format("int4"), shape, 0, None, True,
                   scale16=s16, group=128, kn=kn)


def _q8(W):
    codes, s32, s16 = O.quant_int8_rows(W)
    return QTensor(codes.reshape(-1).view(np.uint8), s32.reshape(-1, 1), get_format("int8"), W.shape, 0, None, False,
                   scale16=s16)


def test_reference_checkpoint_loads_bit_exact():
    t = modelio.load_packed(REF_APSIM)
    w4, w8 = GOLD["apsim_w4"], GOLD["apsim_w8"]
    q = t["proj"]["W"]
    assert q.fmt.name == "int4" and q.group == 128 and q.shape == (w4.size // 128, 128)
    lin = modelio.as_linear(q, w4.shape[0])
    packed, s32, s16 = O.quant_int4_g128(w4)
    assert lin.shape == w4.shape
    assert np.array_equal(np.asarray(lin.codes).reshape(packed.shape), packed)
    assert np.array_equal(np.asarray(lin.scale, np.float32), s32.reshape(lin.scale.shape))
    assert np.array_equal(np.asarray(lin.scale16).view(np.uint16), np.asarray(s16).view(np.uint16))
    q8 = t["down"]["W"]
    codes, s32_8, s16_8 = O.quant_int8_rows(w8)
    assert q8.fmt.name == "int8" and q8.shape == w8.shape
    assert np.array_equal(np.asarray(q8.codes).view(np.int8).reshape(codes.shape), codes)
    assert np.array_equal(np.asarray(q8.scale, np.float32).reshape(-1), s32_8.reshape(-1))
    assert np.array_equal(np.asarray(q8.scale16).view(np.uint16), np.asarray(s16_8).view(np.uint16))
    assert np.array_equal(t["proj"]["b"], GOLD["apsim_b4"]) and np.array_equal(t["norm"], GOLD["apsim_norm"])


def test_round_trip_keeps_the_b200_layout(tmp_path):
    rng = np.random.default_rng(11)
    W4 = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    W8 = (rng.standard_normal((24, 192)) * 0.02).astype(np.float32)
    tree = {"layers": [{"wq": _q4(W4), "wo": _q4(W4, kn=True)}, {"w8": _q8(W8)}],
            "norm": np.linspace(0, 1, 256).astype(np.float32)}
    path = modelio.save_packed(tmp_path / "m", tree, metadata={"note": "test"})
    assert path.endswith(".apsim")
    back = modelio.load_packed(path)
    for got, want in ((back["layers"][0]["wq"], tree["layers"][0]["wq"]),
                      (back["layers"][0]["wo"], tree["layers"][0]["wo"]),
                      (back["layers"][1]["w8"], tree["layers"][1]["w8"])):
        assert got.shape == want.shape and got.group == want.group and got.kn == want.kn
        assert got.fmt.name == want.fmt.name
        assert np.array_equal(np.asarray(got.codes).view(np.uint8), np.asarray(want.codes).view(np.uint8))
        assert np.array_equal(np.asarray(got.scale, np.float32).reshape(-1), np.asarray(want.scale, np.float32).reshape(-1))
        assert np.array_equal(np.asarray(got.scale16).view(np.uint16).reshape(-1),
                              np.asarray(want.scale16).view(np.uint16).reshape(-1))
    assert np.array_equal(back["norm"], tree["norm"])
    # the container is the reference's: format tag and the per-tensor QTensor description
    with open(path, "rb") as fh:
        n = int(np.frombuffer(fh.read(8), "<u8")[0])
        header = json.loads(fh.read(n))
    meta = header["__metadata__"]
    assert meta["format"] == "apsi-model" and "sha256" in meta
    info = json.loads(meta["qtensors"])["layers.0.wq"]
    assert info["shape"] == [64 * 256 // 128, 128] and info["scale_shape"] == [64 * 256 // 128, 1]
    assert header["layers.0.wq"]["dtype"] == "U8" and header["layers.0.wq__qscale"]["dtype"] == "F32"


def test_modified_data_is_rejected(tmp_path):
    W = (np.random.default_rng(2).standard_normal((8, 128)) * 0.02).astype(np.float32)
    path = modelio.save_packed(tmp_path / "m.apsim", {"w": _q4(W)})
    raw = bytearray(open(path, "rb").read())
    raw[-1] ^= 0x01
    open(path, "wb").write(bytes(raw))
    with pytest.raises(RuntimeErr, match="SHA-256"):
        modelio.load_packed(path)


def test_file_written_here_loads_in_the_reference(tmp_path):
    root = os.environ.get("APSI_REF")
    if not root or not os.path.isdir(os.path.join(root, "apsi")):
        pytest.skip("APSI_REF does not name a reference checkout")
    sys.path.insert(0, root)
    try:
        from apsi import modelio as ref_io, precision as ref_p
    except Exception as e:            # noqa: BLE001
        pytest.skip(f"the reference does not import: {e}")
    W = (np.random.default_rng(4).standard_normal((32, 512)) * 0.02).astype(np.float32)
    W8 = (np.random.default_rng(5).standard_normal((16, 128)) * 0.02).astype(np.float32)
    path = modelio.save_packed(tmp_path / "x.apsim", {"a": {"W": _q4(W)}, "b": _q8(W8)})
    t = ref_io.load_model(path)
    d4 = np.asarray(ref_p.dequantize(t.a.W), np.float32).reshape(W.shape)
    packed, s32, _ = O.quant_int4_g128(W)
    assert np.array_equal(d4, O.dequant_int4_g128(packed, s32.astype(np.float32).reshape(32, 4)).astype(np.float32))
    d8 = np.asarray(ref_p.dequantize(t.b), np.float32)
    assert np.array_equal(d8, np.asarray(ref_p.dequantize(ref_p.quantize(W8, "int8", axis=0)), np.float32))
