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
import tempfile

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


_MAX_HEADER = 256 << 20      # a header above this is treated as damage, not read into memory
_CHUNK = 16 << 20            # bytes hashed per read


def _table(tensors):
    """Tensor table of the container: each tensor's dtype tag, shape and [begin, end) byte range in the data
    section, in write order."""
    table, pos = {}, 0
    for name, a in tensors.items():
        table[name] = {"dtype": _DT[a.dtype], "shape": list(a.shape), "data_offsets": [pos, pos + a.nbytes]}
        pos += a.nbytes
    return table


def _digest(table, chunks):
    """SHA-256 over the canonical tensor table followed by the data bytes (``chunks`` in file order): the
    checksum the container stores, so files written here and by the reference verify in both."""
    h = hashlib.sha256(_layout(table))
    for c in chunks:
        h.update(c)
    return h.hexdigest()


def save_packed(path, params, metadata=None):
    """Write a parameter tree (dicts / lists of arrays and packed QTensors) as one ``.apsim`` file.

    The file is assembled under a temporary name in the target directory and renamed over ``path`` at the end,
    so a reader never sees a half-written checkpoint."""
    path = str(path) if str(path).endswith(".apsim") else str(path) + ".apsim"
    tensors, qts = _entries(params)
    table = _table(tensors)
    blobs = [memoryview(a).cast("B") for a in tensors.values() if a.size]
    meta = {"format": FORMAT, "version": VERSION, "apsi": "apsi_b200", "units": "{}", "qtensors": json.dumps(qts),
            "metadata": json.dumps({str(k): v for k, v in (metadata or {}).items()}, default=str),
            "sha256": _digest(table, blobs)}
    head = json.dumps(dict(table, __metadata__=meta), separators=(",", ":")).encode("utf-8")
    head = head.ljust(len(head) + (8 - len(head) % 8) % 8, b" ")    # data section 8-byte aligned
    folder = os.path.dirname(os.path.abspath(path))
    os.makedirs(folder, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix=".apsim-", dir=folder)
    try:
        with os.fdopen(fd, "wb") as out:
            out.write(len(head).to_bytes(8, "little"))
            out.write(head)
            for b in blobs:
                out.write(b)
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise
    return path


class _Container:
    """Reader of one ``.apsim`` file: parses and checks the header when opened, verifies the checksum on
    request, and reads tensors by name."""

    def __init__(self, path):
        self.path = path
        self.name = os.path.basename(path)
        size = os.path.getsize(path)
        with open(path, "rb") as fh:
            raw = fh.read(8)
            hlen = int.from_bytes(raw, "little") if len(raw) == 8 else -1
            if hlen < 2 or hlen > min(size - 8, _MAX_HEADER):
                self._fail("its header length field is missing or larger than the file")
            text = fh.read(hlen)
        try:
            head = json.loads(text.decode("utf-8"))
        except (UnicodeDecodeError, ValueError):
            head = None
        if not isinstance(head, dict):
            self._fail("its header is not a JSON object")
        self.meta = head.pop("__metadata__", {}) or {}
        self.table = head
        self.base = 8 + hlen
        self.data_end = 0
        room = size - self.base
        self.layout = {}
        for tname, info in head.items():
            try:
                dt = _DT_R[info["dtype"]]
                shape = tuple(int(d) for d in info["shape"])
                lo, hi = (int(v) for v in info["data_offsets"])
            except (KeyError, TypeError, ValueError):
                self._fail(f"the header entry of '{tname}' has no valid dtype, shape or data_offsets")
            want = int(np.prod(shape, dtype=np.int64)) * dt.itemsize if shape else dt.itemsize
            if min(shape, default=0) < 0 or lo < 0 or hi > room or hi - lo != want:
                self._fail(f"the byte range of '{tname}' does not fit its shape or the file")
            self.layout[tname] = (dt, shape, lo)
            self.data_end = max(self.data_end, hi)

    def _fail(self, why):
        raise RuntimeErr(f"{self.name} cannot be read as an Apsi checkpoint: {why}")

    def verify(self):
        """Recompute the stored SHA-256 (when there is one) over the table and the data section."""
        want = self.meta.get("sha256")
        if not want:
            return

        def chunks():
            left = self.data_end
            with open(self.path, "rb") as fh:
                fh.seek(self.base)
                while left > 0:
                    b = fh.read(min(_CHUNK, left))
                    if not b:
                        break
                    left -= len(b)
                    yield b
        if _digest(self.table, chunks()) != want:
            raise RuntimeErr(f"{self.name}: checksum (SHA-256) mismatch -- the tensor data or table changed after "
                             f"the file was written")

    def arrays(self):
        """Every tensor as a read-only array mapped from the file."""
        out = {}
        for tname, (dt, shape, lo) in self.layout.items():
            count = int(np.prod(shape, dtype=np.int64)) if shape else 1
            if count == 0:
                out[tname] = np.empty(shape, dt)
                continue
            out[tname] = np.memmap(self.path, dtype=dt, mode="r", offset=self.base + lo, shape=shape)
        return out


def _read(path, verify):
    c = _Container(path)
    if verify:
        c.verify()
    return c.arrays(), c.meta


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
