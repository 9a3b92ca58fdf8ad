"""models.load_safetensors (apsi/models.py:61-108): a checkpoint read memory-mapped, with dtype None / f32 keeping
the values (bfloat16 widened to float32), nesting by the dotted names, and dtype "int4" / "int8" packing every
float matrix on the device in the fused kernels' layout (bit-exact with the oracle's quantisation)."""
import json
import struct

import numpy as np
import pytest

import oracle as O
from apsi_b200 import models


def _write(path, tensors):
    """A .safetensors file: 8-byte header length, JSON table, data."""
    table, blobs, off = {}, [], 0
    for name, (st, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        table[name] = {"dtype": st, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(table).encode()
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def _checkpoint(tmp_path):
    rng = np.random.default_rng(4)
    W = (rng.standard_normal((384, 512)) * 0.02).astype(np.float32)
    bits = (O.bf16_round(W).view(np.uint32) >> np.uint32(16)).astype(np.uint16)
    tensors = {"layers.0.proj.weight": ("F32", W), "layers.0.proj.bias": ("F32", np.linspace(-1, 1, 384, dtype=np.float32)),
               "layers.1.proj.weight": ("BF16", bits), "norm.weight": ("F16", np.ones(512, np.float16)),
               "odd.weight": ("F32", np.ones((4, 100), np.float32))}
    path = tmp_path / "m.safetensors"
    _write(path, tensors)
    return path, W, bits


def test_stored_precision_and_nesting(tmp_path):
    path, W, bits = _checkpoint(tmp_path)
    flat = models.load_safetensors(str(path), nested=None)
    assert np.array_equal(flat["layers.0.proj.weight"], W)
    assert np.array_equal(flat["layers.1.proj.weight"], (bits.astype(np.uint32) << 16).view(np.float32))
    assert flat["norm.weight"].dtype == np.float16
    tree = models.load_safetensors(str(path), dtype="f32")
    assert isinstance(tree["layers"], list) and len(tree["layers"]) == 2
    assert tree["layers"][0]["proj"]["bias"].dtype == np.float32 and tree["norm"]["weight"].dtype == np.float32
    flat2 = models.load_safetensors(str(path), nested=False, names={"norm.weight"})
    assert list(flat2) == ["norm_weight"]


def test_damaged_offsets_are_refused(tmp_path):
    path = tmp_path / "bad.safetensors"
    h = json.dumps({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 1 << 20]}}).encode()
    path.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 16)
    with pytest.raises(Exception, match="outside the file"):
        models.load_safetensors(str(path))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["int4", "int8"])
def test_packed_on_load(cuda, tmp_path, dtype):
    import torch
    from apsi_b200 import precision as P
    path, W, bits = _checkpoint(tmp_path)
    tree = models.load_safetensors(str(path), dtype=dtype, nested=None)
    q = tree["layers.0.proj.weight"]
    assert isinstance(q, P.QTensor) and q.shape == (384, 512)
    assert isinstance(tree["layers.0.proj.bias"], np.ndarray)            # vectors stay float32
    assert isinstance(tree["odd.weight"], np.ndarray)                    # rows of 100 values: no fused product
    codes, s16 = q.device_tensors()
    if dtype == "int4":
        o_codes, _, o_s16 = O.quant_int4_g128(W)
        Wd = O.dequant_int4_g128(o_codes, o_s16)
    else:
        o_codes, _, o_s16 = O.quant_int8_rows(W)
        Wd = O.dequant_int8_rows(o_codes, o_s16)
    assert np.array_equal(codes.cpu().numpy().reshape(o_codes.shape), o_codes)
    assert np.array_equal(s16.cpu().numpy().view(np.uint16).reshape(-1), o_s16.view(np.uint16).reshape(-1))
    x = O.bf16_round(np.random.default_rng(1).standard_normal((3, 512)).astype(np.float32))
    y = P.qmatmul(x, q)                                                  # x @ W.T, the checkpoint's orientation
    ref = O.linear_ref(x, Wd)
    assert O.max_abs_ratio(y, ref) <= 1e-2 and O.rel_frobenius(y, ref) <= 2e-3
