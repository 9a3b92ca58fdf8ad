"""The quantized-layer entry points of ``apsi/models.py`` on the B200 library.

* ``qlinear(x, W, b)`` -- ``x @ W (+ b)`` where W may be a packed QTensor (apsi/models.py:302-308).  A packed
  ``[in, out]`` weight (``precision.quantize_linear`` / ``quantize_model``) runs the fused kernels, with the
  bias added in the kernel epilogue; the result is bfloat16 on the device (fp32 accumulation).  A dense W
  keeps the reference's ``x @ W (+ b)``.
* ``quantize_model(params, dtype, min_size)`` -- every float matrix of at least ``min_size`` elements stored
  packed for the kernels (apsi/models.py:272-281).  The formats are ``"int4"`` (groups of 128, the default
  here) and ``"int8"`` (one scale per output); ``"int4_g128"``, ``"w4g128"``, ``"int8_row"`` and ``"w8"`` are
  accepted too.
* ``dequantize_model(params)`` -- every QTensor back to float32 (apsi/models.py:284-285).
* ``load_safetensors(path, dtype, names, nested)`` -- a ``.safetensors`` checkpoint, memory-mapped
  (apsi/models.py:61-108).  With a packed ``dtype`` ("int4" -- groups of 128 here --, "int8", or a minifloat
  format) every float matrix is quantised on the device as it is read, straight into the kernels' layout
  (``[out, in]`` rows, as checkpoints store them; ``x @ q`` multiplies by its transpose).
"""
import json
import os
import struct

import numpy as np

from . import kernels as _k
from . import precision as P
from .lowbit import parse_linear, tree_map

__all__ = ["qlinear", "quantize_model", "dequantize_model", "model_size", "load_safetensors"]

_LINEAR_TO_FMT = {"int4_g128": "int4", "int8_row": "int8"}


def _fmt_name(dtype):
    name = getattr(dtype, "name", dtype) if dtype is not None else "int4"
    k = parse_linear(name)
    return _LINEAR_TO_FMT[k] if k else P.get_format(name).name


def qlinear(x, W, b=None):
    """x @ W (+ b) where W may be a packed QTensor: dequantise-and-multiply in the fused kernels, fp32 accumulate."""
    if isinstance(W, P.QTensor):
        import torch
        if not W.kn:
            raise P.RuntimeErr("qlinear takes an [in, out] weight quantised with quantize_linear / quantize_model")
        R, C = W.rows
        xt = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(x, np.float32))
        was_host = not xt.is_cuda
        dev = torch.device("cuda", torch.cuda.current_device()) if was_host else xt.device
        lead = tuple(xt.shape[:-1])
        x2 = xt.reshape(-1, C).to(dev).to(torch.bfloat16).contiguous()
        bias = None
        if b is not None:
            bt = b if isinstance(b, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(b, np.float32))
            bias = bt.reshape(-1).to(dev).to(torch.bfloat16).contiguous()
        codes, s16 = W.device_tensors(dev)
        y = _k.linear(W.kernel_format, x2, codes, s16, R, bias=bias).reshape(*lead, R)
        if not isinstance(x, torch.Tensor):
            return y.float().cpu().numpy()
        return y.cpu() if was_host else y
    y = x @ W
    return y + b if b is not None else y


def quantize_model(params, dtype=None, min_size=1024):
    """Store every weight matrix (>= min_size elements) packed for the fused kernels; others stay as they are."""
    fmt = _fmt_name(dtype)

    def q(x):
        try:
            import torch
            is_t = isinstance(x, torch.Tensor)
        except ImportError:  # pragma: no cover
            is_t = False
        if is_t:
            ok = x.is_floating_point() and x.dim() == 2 and x.numel() >= min_size
        else:
            ok = isinstance(x, np.ndarray) and x.dtype.kind == "f" and x.ndim == 2 and x.size >= min_size
        return P.quantize_linear(x, fmt) if ok else x
    return tree_map(q, params)


def dequantize_model(params):
    return tree_map(lambda x: P.dequantize(x) if isinstance(x, P.QTensor) else x, params)


def model_size(params):
    """Bytes used by all tensors in a parameter tree (packed weights at their real size)."""
    total = 0

    def add(x):
        nonlocal total
        if isinstance(x, P.QTensor):
            total += x.nbytes
        elif isinstance(x, np.ndarray):
            total += x.nbytes
        else:
            try:
                import torch
                if isinstance(x, torch.Tensor):
                    total += x.numel() * x.element_size()
            except ImportError:  # pragma: no cover
                pass
        return x
    tree_map(add, params)
    return total


# ------------------------------------------------------------------------------------------------ safetensors
_ST_NP = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "I64": np.int64, "I32": np.int32,
          "I16": np.int16, "I8": np.int8, "U8": np.uint8, "BOOL": np.bool_, "U16": np.uint16, "U32": np.uint32,
          "U64": np.uint64}
_HEADER_CAP = 100 << 20                     # bytes of JSON header accepted (the reference's bound)


def _safetensors_table(path):
    """(tensor table, offset of the data section) of a .safetensors file."""
    with open(path, "rb") as fh:
        head = fh.read(8)
        if len(head) != 8:
            raise P.RuntimeErr(f"{path}: not a safetensors file (no header length)")
        (n,) = struct.unpack("<Q", head)
        if n > _HEADER_CAP:
            raise P.RuntimeErr(f"{path}: safetensors header of {n} bytes is too large (corrupt or malicious file)")
        table = json.loads(fh.read(n).decode("utf-8"))
    return table, 8 + n


def _decode(raw, st, shape):
    """Stored bytes -> a NumPy array (bfloat16 and fp8 widened to float32, as the reference does)."""
    if st in _ST_NP:
        return raw.view(_ST_NP[st]).reshape(shape)
    if st == "BF16":
        return (raw.view(np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32).reshape(shape)
    if st in ("F8_E4M3", "F8_E5M2"):
        import torch
        t = torch.from_numpy(np.array(raw, np.uint8)).view(torch.float8_e4m3fn if st == "F8_E4M3" else
                                                             torch.float8_e5m2)
        return t.float().numpy().reshape(shape)
    raise P.RuntimeErr(f"safetensors: unsupported dtype {st}")


def _pack_for_device(arr, want):
    """The reference's _convert (apsi/models.py:95-108) for this library: f32 / f16 / f64 convert; a packed
    format quantises float matrices on the device (int4: groups of 128 along the row).  Matrices whose rows the
    fused products cannot take (a length that is not a multiple of 128 for 4-bit codes, 16 for 6-bit, 64 for
    8-bit), vectors and integer tensors stay float32, as the reference keeps biases and norms."""
    if want is None:
        return arr
    if want in ("f64", "fp64"):
        return np.asarray(arr, np.float64)
    if want in ("f32", "fp32"):
        return np.asarray(arr, np.float32)
    if want in ("f16", "fp16"):
        return np.asarray(arr, np.float16)
    if np.asarray(arr).dtype.kind != "f" or np.ndim(arr) != 2:
        return np.asarray(arr, np.float32)
    import torch
    fmt = _fmt_name(want)
    f = P.get_format(fmt)
    if arr.shape[1] % {4: 128, 6: 16}.get(f.bits, 64):   # rows the fused products take: 4-bit 128k, 6-bit 16k, 8-bit 64k
        return np.asarray(arr, np.float32)
    w = torch.from_numpy(np.array(arr, np.float32)).to(torch.device("cuda", torch.cuda.current_device()))
    if f.kind == "minifloat":
        return P.quantize(w, fmt, axis=0)
    return P.quantize(w, fmt, axis=0, group=128 if f.bits == 4 else None)


def _nest(flat):
    """"a.0.b" names -> nested dicts, with lists where every key of a level is a number."""
    root = {}
    for name, v in flat.items():
        node = root
        parts = name.split(".")
        for part in parts[:-1]:
            node = node.setdefault(part, {})
        node[parts[-1]] = v

    def build(d):
        if not isinstance(d, dict):
            return d
        if d and all(k.isdigit() for k in d):
            return [build(d[k]) for k in sorted(d, key=int)]
        return {k: build(v) for k, v in d.items()}
    return build(root)


def load_safetensors(path, dtype=None, names=None, nested=True):
    """A .safetensors checkpoint, memory-mapped (apsi/models.py:61-92).  dtype None keeps the stored precision
    (bfloat16 / fp8 widened to float32); "f32" / "f16" / "f64" convert; "int4" / "int8" / a minifloat format
    packs every float matrix on the device (a QTensor in the fused kernels' layout).  nested: True -> nested
    dicts and lists by the dotted names; False -> one flat dict with "." replaced by "_"; None -> the flat dict
    under the exact names."""
    table, start = _safetensors_table(path)
    size = os.path.getsize(path)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    want = None if dtype is None else str(getattr(dtype, "name", dtype)).lower()
    out = {}
    for name, info in table.items():
        if name == "__metadata__" or (names is not None and name not in names):
            continue
        a, b = info["data_offsets"]
        if not (0 <= a <= b and start + b <= size):
            raise P.RuntimeErr(f"safetensors: tensor '{name}' points outside the file (corrupt or malicious)")
        arr = _decode(mm[start + a:start + b], info["dtype"], tuple(info["shape"]))
        out[name] = _pack_for_device(arr, want)
    if nested is None:
        return out
    return _nest(out) if nested else {k.replace(".", "_"): v for k, v in out.items()}
