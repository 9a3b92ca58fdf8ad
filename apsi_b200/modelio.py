"""Packed low-bit weights on disk: Apsi checkpoints (``.apsim``) that load without re-quantising.

An ``.apsim`` file is the reference's checkpoint container (apsi/modelio.py:337-600): a safetensors file (8-byte
little-endian header length, JSON header, raw tensor bytes) whose ``__metadata__`` holds ``format`` =
"apsi-model", ``version``, the JSON strings ``units``, ``qtensors`` and ``metadata``, and a SHA-256 of the tensor
table plus the data.  A quantised tensor is stored as its codes under its own name and its float32 scales under
``NAME__qscale``, with ``qtensors[NAME]`` = {fmt, shape, axis, packed, scale_shape, dim}
(apsi/modelio.py:361-382, 586-591).

The B200 layouts map onto the reference's QTensor forms, so files cross in both directions:

* int4 groups of 128 of a [R, C] weight: the reference quantises ``W.reshape(-1, 128)`` with ``axis=0``, a
  QTensor of shape [R C / 128, 128] with scales [R C / 128, 1].  The packed bytes and the scales are the same
  arrays in the same order as the B200 [R, C] layout, so they are written as that reference QTensor; an extra
  ``b200`` entry in ``qtensors[NAME]`` records rows, cols, group and the [in, out] flag.  The reference's loader
  reads the known keys only and ignores it.
* int8 with one scale per row: the reference's own [R, C], ``axis=0`` form.

On load the binary16 scales the kernels read are recomputed as fp16 of the stored float32 scales, which is how
the quantisers define them, so a loaded layer is bit-identical to a freshly quantised one.  A reference file
without the ``b200`` entry loads as the reference QTensor it is; ``as_linear`` views a [R C / 128, 128] int4
QTensor as the [R, C] layer.

No GPU is needed to save or load; ``load_packed(..., device=...)`` also places the kernel layout on a GPU.
"""
import hashlib
import json
import os
import struct

import numpy as np

from . import kernels as _k
from .precision import QTensor, get_format, RuntimeErr

__all__ = ["save_packed", "load_packed", "as_linear", "FORMAT", "VERSION", "gguf_q8_0", "gguf_q4_0", "gguf_dequant"]

FORMAT = "apsi-model"          # the reference's container tag (apsi/modelio.py:30-31)
VERSION = "1"
_DT = {np.dtype(np.float64): "F64", np.dtype(np.float32): "F32", np.dtype(np.float16): "F16",
       np.dtype(np.int64): "I64", np.dtype(np.int32): "I32", np.dtype(np.int16): "I16", np.dtype(np.int8): "I8",
       np.dtype(np.uint8): "U8", np.dtype(np.uint16): "U16", np.dtype(np.uint32): "U32",
       np.dtype(np.uint64): "U64", np.dtype(np.bool_): "BOOL"}
_DT_R = {v: k for k, v in _DT.items()}


def _host(a):
    """numpy view of an array or a (CPU or CUDA) torch tensor."""
    if hasattr(a, "detach"):
        return a.detach().cpu().numpy()
    return np.asarray(a)


def _flatten(tree, prefix=""):
    if isinstance(tree, dict):
        items = tree.items()
    elif isinstance(tree, (list, tuple)):
        items = ((str(i), v) for i, v in enumerate(tree))
    else:
        return {prefix.rstrip("."): tree}
    out = {}
    for k, v in items:
        out.update(_flatten(v, f"{prefix}{k}."))
    return out


def _nest(flat):
    root = {}
    for name, v in flat.items():
        parts = name.split(".")
        node = root
        for p in parts[:-1]:
            node = node.setdefault(p, {})
        node[parts[-1]] = v

    def build(d):
        if not isinstance(d, dict):
            return d
        if d and all(k.isdigit() for k in d):
            return [build(d[k]) for k in sorted(d, key=int)]
        return {k: build(v) for k, v in d.items()}
    return build(root)


def _layout(header):
    """The tensor table in the fixed form the reference hashes (apsi/modelio.py:385-389)."""
    t = {k: [v["dtype"], [int(d) for d in v["shape"]], [int(o) for o in v["data_offsets"]]]
         for k, v in header.items() if k != "__metadata__"}
    return json.dumps(t, sort_keys=True, separators=(",", ":")).encode("utf-8")


def _entries(params):
    tensors, qts = {}, {}
    for name, v in _flatten(params).items():
        if isinstance(v, QTensor):
            codes = np.ascontiguousarray(_host(v.codes)).reshape(-1).view(np.uint8)
            sc = np.ascontiguousarray(_host(v.scale), dtype=np.float32).reshape(-1)
            R, C = v.rows
            if v.fmt.bits == 4 and v.group == 128:
                shape, scale_shape = [R * C // 128, 128], [R * C // 128, 1]
            elif v.fmt.bits == 8 and not v.group:
                shape, scale_shape = [R, C], [R, 1]
            else:
                raise RuntimeErr(f"'{name}': only int4 groups of 128 and int8 rows have a packed layout")
            tensors[name] = codes
            tensors[name + "__qscale"] = sc
            qts[name] = {"fmt": v.fmt.name, "shape": shape, "axis": 0, "packed": bool(v.fmt.bits == 4),
                         "scale_shape": scale_shape, "dim": None,
                         "b200": {"rows": R, "cols": C, "group": v.group, "kn": bool(v.kn)}}
            continue
        a = _host(v)
        if a.dtype not in _DT:
            a = a.astype(np.float32)
        tensors[name] = np.ascontiguousarray(a)
    return tensors, qts


def save_packed(path, params, metadata=None):
    """Write a parameter tree (dicts / lists of arrays and packed QTensors) as one ``.apsim`` file."""
    path = str(path)
    if not path.endswith(".apsim"):
        path += ".apsim"
    tensors, qts = _entries(params)
    header, offset = {}, 0
    for name, a in tensors.items():
        header[name] = {"dtype": _DT[a.dtype], "shape": list(a.shape), "data_offsets": [offset, offset + a.nbytes]}
        offset += a.nbytes
    h = hashlib.sha256(_layout(header))
    for a in tensors.values():
        h.update(memoryview(a).cast("B") if a.size else b"")
    header["__metadata__"] = {"format": FORMAT, "version": VERSION, "apsi": "apsi_b200",
                              "units": "{}", "qtensors": json.dumps(qts),
                              "metadata": json.dumps({str(k): v for k, v in (metadata or {}).items()}, default=str),
                              "sha256": h.hexdigest()}
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * ((-len(hb)) % 8)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    tmp = path + ".tmp"
    with open(tmp, "wb") as fh:
        fh.write(struct.pack("<Q", len(hb)))
        fh.write(hb)
        for a in tensors.values():
            if a.size:
                fh.write(memoryview(a).cast("B"))
    os.replace(tmp, path)
    return path


def _read(path, verify):
    bad = f"{os.path.basename(path)} is not a valid Apsi checkpoint"
    if os.path.getsize(path) < 8:
        raise RuntimeErr(bad + " (too short)")
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    n = int(np.frombuffer(mm[:8], "<u8")[0])
    if n > min(len(mm) - 8, 100 << 20):
        raise RuntimeErr(bad + " (header size out of range)")
    try:
        header = json.loads(bytes(mm[8:8 + n]).decode("utf-8"))
    except (UnicodeDecodeError, ValueError):
        raise RuntimeErr(bad + " (unreadable header)")
    meta = header.pop("__metadata__", {})
    start = 8 + n
    for name, info in header.items():
        try:
            a, b = (int(x) for x in info["data_offsets"])
            dt = _DT_R[info["dtype"]]
            count = int(np.prod([int(d) for d in info["shape"]], dtype=np.int64))
        except (KeyError, TypeError, ValueError):
            raise RuntimeErr(bad + f" (tensor '{name}' is described incorrectly)")
        if not 0 <= a <= b <= len(mm) - start or b - a != count * dt.itemsize:
            raise RuntimeErr(bad + f" (tensor '{name}' lies outside the file)")
    if verify and "sha256" in meta:
        h = hashlib.sha256(_layout(header))
        end = start + max((v["data_offsets"][1] for v in header.values()), default=0)
        for p in range(start, end, 1 << 26):
            h.update(mm[p:min(end, p + (1 << 26))])
        if h.hexdigest() != meta["sha256"]:
            raise RuntimeErr(f"{os.path.basename(path)} is damaged or was modified: its data does not match the "
                             f"SHA-256 stored in the file")
    arrays = {}
    for name, info in header.items():
        a, b = info["data_offsets"]
        dt = _DT_R[info["dtype"]]
        arrays[name] = np.frombuffer(mm, dt, count=(b - a) // dt.itemsize, offset=start + a).reshape(info["shape"])
    return arrays, meta


def load_packed(path, verify=True, device=None):
    """Read an ``.apsim`` file: packed QTensors come back in the B200 layout (binary16 scales recomputed from
    the stored float32 scales), other tensors as numpy arrays.  ``device``: also place every packed layer's
    kernel tensors (codes, fp16 scales) on that CUDA device."""
    path = str(path)
    if not os.path.exists(path) and os.path.exists(path + ".apsim"):
        path += ".apsim"
    flat, meta = _read(path, verify)
    if meta.get("format") != FORMAT:
        raise RuntimeErr(f"{os.path.basename(path)} is not an Apsi checkpoint")
    try:
        qts = json.loads(meta.get("qtensors", "{}"))
        out = {}
        for name, info in qts.items():
            codes = np.array(flat.pop(name)).reshape(-1).view(np.uint8)
            sc = np.array(flat.pop(name + "__qscale"), np.float32)
            fmt = get_format(info["fmt"])
            b2 = info.get("b200")
            if b2:
                R, C, group, kn = int(b2["rows"]), int(b2["cols"]), b2.get("group"), bool(b2.get("kn"))
                scale = sc.reshape(R, C // 128) if group == 128 else sc.reshape(R, 1)
                s16 = scale.astype(np.float16) if group == 128 else sc.astype(np.float16)   # int8: [R]
                shape = (C, R) if kn else (R, C)
                q = QTensor(codes, scale, fmt, shape, 0, None, fmt.bits == 4, scale16=s16, group=group, kn=kn)
            else:
                shape = tuple(int(d) for d in info["shape"])
                scale = sc.reshape(info["scale_shape"])
                if fmt.bits == 4 and len(shape) == 2 and shape[1] == 128 and info.get("axis") in (0, -2):
                    q = QTensor(codes, scale, fmt, shape, 0, None, True, scale16=scale.astype(np.float16),
                                group=128)
                elif fmt.bits == 8 and len(shape) == 2 and info.get("axis") in (0, -2):
                    q = QTensor(codes, scale, fmt, shape, 0, None, False, scale16=scale.reshape(-1).astype(np.float16))
                else:
                    raise RuntimeErr(f"'{name}': {info['fmt']} {shape} axis {info.get('axis')} has no B200 layout")
            if device is not None:
                q.device_tensors(device)
            out[name] = q
        for name, a in flat.items():
            out[name] = np.array(a)
        return _nest(out)
    except RuntimeErr:
        raise
    except (KeyError, TypeError, ValueError, AttributeError) as e:
        raise RuntimeErr(f"{os.path.basename(path)} has an inconsistent header ({type(e).__name__}: {e})")


def as_linear(q, rows):
    """An int4 group-128 QTensor stored the reference's way ([R C / 128, 128]) seen as the [rows, C] layer it
    came from (no copy of the codes)."""
    if q.fmt.bits != 4 or q.group != 128 or len(q.shape) != 2 or q.shape[1] != 128:
        raise RuntimeErr("as_linear takes an int4 QTensor of shape [R C / 128, 128]")
    total = q.shape[0] * 128
    if total % rows:
        raise RuntimeErr(f"{total} values do not form {rows} rows")
    C = total // rows
    scale = np.asarray(q.scale, np.float32).reshape(rows, C // 128)
    s16 = np.asarray(q.scale16).reshape(rows, C // 128)
    return QTensor(q.codes, scale, q.fmt, (rows, C), 0, None, True, scale16=s16, group=128)


# ------------------------------------------------------------------------------------------------ GGUF blocks
def _gguf_device_input(a):
    import torch
    if isinstance(a, torch.Tensor):
        t = a.detach().reshape(-1)
        was_np = False
    else:
        t = torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32).reshape(-1)))
        was_np = True
    if not t.is_cuda:
        t = t.to(torch.device("cuda", torch.cuda.current_device()))
    return t.to(torch.float32).contiguous(), was_np


def gguf_q8_0(a):
    """GGUF Q8_0 block bytes of a float array (size a multiple of 32), computed on the GPU: the bytes of the
    reference's ``modelio._q8_0`` (apsi/modelio.py:56-67).  NumPy in -> ``bytes`` out; CUDA tensor in -> uint8
    CUDA tensor out."""
    t, was_np = _gguf_device_input(a)
    out = _k.gguf_encode(t, 8)
    return out.cpu().numpy().tobytes() if was_np else out


def gguf_q4_0(a):
    """GGUF Q4_0 block bytes (apsi/modelio.py:70-81, ``modelio._q4_0``), computed on the GPU."""
    t, was_np = _gguf_device_input(a)
    out = _k.gguf_encode(t, 4)
    return out.cpu().numpy().tobytes() if was_np else out


def gguf_dequant(buf, kind, n):
    """float32 values of Q8_0 (kind "q8_0") or Q4_0 ("q4_0") blocks (apsi/modelio.py:84-95), on the GPU."""
    import torch
    if isinstance(buf, torch.Tensor):
        b, was_np = buf.reshape(-1).contiguous(), False
        if not b.is_cuda:
            b, was_np = b.to(torch.device("cuda", torch.cuda.current_device())), True
    else:
        b = torch.from_numpy(np.frombuffer(bytes(buf), np.uint8).copy()).to(
            torch.device("cuda", torch.cuda.current_device()))
        was_np = True
    nb = (n + 31) // 32 * 32
    out = _k.gguf_decode(b, 8 if kind == "q8_0" else 4, nb)[:n]
    return out.cpu().numpy() if was_np else out
