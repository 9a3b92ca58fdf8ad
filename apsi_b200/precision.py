"""The public entry points of ``apsi/precision.py`` on the B200 library.

Same names, argument meanings and error types as the reference module (apsi/precision.py:142-339) for the
formats on the B200 path:

* ``quantize(x, "int8", axis=0)`` -- int8 with one absmax/127 scale per row of a 2-D array (bit-exact with the
  reference: codes, float32 scale); the QTensor also carries the binary16 scale the kernels use.
* ``quantize(x, "int4", axis=0, group=128)`` -- int4 with one absmax/7 scale per 128 values along each row;
  bit-exact with ``quantize(x.reshape(-1, 128), "int4", axis=0)`` of the reference.  ``group`` is the one new
  keyword.  A 2-D ``[R, 128]`` array with ``axis=0`` (the reference's own spelling) takes the same kernel.
* ``dequantize(q)``, ``qmatmul(a, b)``, ``round_to``, ``quant_error``, ``nbytes``, ``QTensor``, ``FORMATS``.
* ``quantize_linear(W, fmt)`` -- new: quantizes an Apsi ``Linear`` weight stored ``[in, out]`` into the kernel
  layout (rows = outputs, groups along the inputs); ``qmatmul(x, q)`` / ``x @ q`` then run the fused
  dequantise-and-matmul kernels.

Every computation runs on the GPU.  NumPy inputs are copied to the current CUDA device, processed there and
the results copied back; torch CUDA inputs stay on the device.  Formats, axes or scale modes the B200 path does
not implement raise ``RuntimeErr`` with the reason (the reference's error type), never a silent CPU path.
"""
import math

import numpy as np

from . import kernels as _k
from ._lib import FMT_INT8_ROW, FMT_INT4_G128, MINIFLOAT_FMT, LowbitError

__all__ = ["RuntimeErr", "Format", "FORMATS", "ALIASES", "get_format", "QTensor", "quantize", "dequantize",
           "round_to", "qmatmul", "nbytes", "quant_error", "format_info", "quantize_linear", "module"]


class RuntimeErr(Exception):
    """Error type of the reference language runtime (apsi/errors.py RuntimeErr) for bad precision requests."""


class Format:
    """A numeric format.  The B200 path implements the integer and the minifloat formats; the table keeps the
    reference's names so ``get_format`` accepts the same spellings (apsi/precision.py:43-74)."""

    def __init__(self, name, bits, kind, qmax=None, maxval=None):
        self.name, self.bits, self.kind = name, bits, kind
        self.qmax = qmax
        self.max = float(qmax) if qmax is not None else maxval

    def __repr__(self):
        return self.name


FORMATS = {
    "int8": Format("int8", 8, "int", qmax=127),
    "int4": Format("int4", 4, "int", qmax=7),
    # OCP fp8 and MX fp6 / fp4 element formats, largest finite values of the reference's tables
    "fp8_e4m3": Format("fp8_e4m3", 8, "minifloat", maxval=448.0),
    "fp8_e5m2": Format("fp8_e5m2", 8, "minifloat", maxval=57344.0),
    "fp6_e3m2": Format("fp6_e3m2", 6, "minifloat", maxval=28.0),
    "fp6_e2m3": Format("fp6_e2m3", 6, "minifloat", maxval=7.5),
    "fp4_e2m1": Format("fp4_e2m1", 4, "minifloat", maxval=6.0),
}
# names the reference knows whose quantisation is not on the B200 path (error message, not silence)
_OTHER = ("f64", "f32", "f16", "bf16", "uint8")
ALIASES = {"fp64": "f64", "fp32": "f32", "fp16": "f16", "fp8": "fp8_e4m3", "bf8": "fp8_e5m2",
           "e4m3": "fp8_e4m3", "e5m2": "fp8_e5m2", "fp6": "fp6_e3m2", "fp4": "fp4_e2m1",
           "int4_g128": "int4", "w4g128": "int4", "w8": "int8"}


def get_format(f):
    name = getattr(f, "name", f)
    name = ALIASES.get(name, name)
    if name in FORMATS:
        return FORMATS[name]
    if name in _OTHER:
        raise RuntimeErr(f"numeric format '{name}' is not on the B200 low-bit path (int8, int4, fp8, fp6, fp4)")
    raise RuntimeErr(f"unknown numeric format '{name}'; choose one of {', '.join(FORMATS)}")


# ------------------------------------------------------------------------------------------------ QTensor
class QTensor:
    """Codes + scales of a quantised array (apsi/precision.py:142-165), with the kernel layout attached.

    ``codes``/``scale`` follow the reference (flat uint8 codes -- int4 packed two per byte, low nibble first --
    and float32 scales shaped as the reference returns them).  B200 additions: ``scale16`` (the binary16
    scales the kernels read), ``group`` (128 for int4 groups, None for one scale per row), ``kn`` (True when
    the logical array is ``[in, out]`` and the rows stored are its transpose, see ``quantize_linear``)."""
    __slots__ = ("codes", "scale", "fmt", "shape", "axis", "dim", "packed", "scale16", "group", "kn", "_dev",
                 "_fast", "_settled")
    # NumPy defers ``x @ q`` (and every other binary operator) to this class, so a model written with plain
    # ``x @ p.W`` -- the reference's Linear.apply (apsi/layers.py:251-253), its attention and SwiGLU blocks --
    # multiplies a QTensor weight through __rmatmul__ and the fused kernels, unchanged
    __array_ufunc__ = None

    def __init__(self, codes, scale, fmt, shape, axis, dim=None, packed=False, scale16=None, group=None, kn=False):
        self.codes, self.scale, self.fmt, self.shape = codes, scale, fmt, tuple(shape)
        self.axis, self.dim, self.packed = axis, dim, packed
        self.scale16, self.group, self.kn = scale16, group, kn
        self._dev = None
        self._fast = None
        self._settled = False

    def touch(self):
        """Call after writing into ``codes`` / ``scale16`` in place: the next product waits for every earlier
        kernel before it reads the weights (see ``qmatmul``)."""
        self._settled = False

    def fast_spec(self):
        """(fmt, codes pointer, scales pointer, N, K, device index) for the per-call fast path of ``qmatmul``, or
        None when the operand does not qualify (host codes, minifloat formats).  Rebuilt when ``codes`` or
        ``scale16`` are replaced."""
        c, s16 = self.codes, self.scale16
        f = self._fast
        if f is not None and f[0] is c and f[1] is s16:
            return f[2]
        self._settled = False                  # new weight tensors: their writer may still be running
        spec = None
        if self.fmt.kind == "int" and _is_torch(c) and c.is_cuda and s16 is not None and s16.is_cuda:
            R, C = self.rows
            fmt, cp, sp, dev = self.kernel_format, c.data_ptr(), s16.data_ptr(), c.get_device()
            spec = (fmt, cp, sp, R, C, dev, _k.prepare_weight(fmt, cp, sp, R, C, dev))
        self._fast = (c, s16, spec)
        return spec

    @property
    def nbytes(self):
        n = _nbytes_of(self.codes)
        if self.scale16 is not None:
            n += _nbytes_of(self.scale16)
        elif self.scale is not None and not isinstance(self.scale, float):
            n += _nbytes_of(self.scale)
        return n

    @property
    def ndim(self):
        return len(self.shape)

    @property
    def rows(self):
        """(rows, cols) of the stored row-major code matrix (outputs x inputs for a linear weight)."""
        return (self.shape[1], self.shape[0]) if self.kn else (self.shape[0], int(np.prod(self.shape[1:])))

    @property
    def kernel_format(self):
        if self.fmt.kind == "minifloat":
            return MINIFLOAT_FMT[self.fmt.name]
        return FMT_INT4_G128 if self.fmt.bits == 4 else FMT_INT8_ROW

    def device_tensors(self, device=None):
        """(codes, scale16) as CUDA tensors in the kernel layout (cached for host QTensors)."""
        import torch
        if _is_torch(self.codes) and self.codes.is_cuda:
            return self.codes, self.scale16
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        if self.fmt.kind == "minifloat":
            if self._dev is None or self._dev[0] != dev:
                codes = torch.from_numpy(np.ascontiguousarray(self.codes).view(np.uint8).reshape(-1)).to(dev)
                sc = self.scale
                if not isinstance(sc, float):
                    sc = torch.from_numpy(np.ascontiguousarray(sc, np.float32).reshape(-1)).to(dev)
                self._dev = (dev, codes, sc)
            return self._dev[1], self._dev[2]
        if self._dev is None or self._dev[0] != dev:
            R, C = self.rows
            ncols = C // 2 if self.fmt.bits == 4 else C
            codes = torch.from_numpy(np.ascontiguousarray(self.codes).view(np.uint8).reshape(R, ncols)).to(dev)
            s16 = torch.from_numpy(np.ascontiguousarray(self.scale16)).to(dev)
            self._dev = (dev, codes, s16)
        return self._dev[1], self._dev[2]

    def dequantize(self):
        return dequantize(self)

    def __matmul__(self, other):
        raise RuntimeErr("a quantised weight is the right operand: write x @ q")

    def __rmatmul__(self, x):
        return qmatmul(x, self)

    def __repr__(self):
        g = f", g{self.group}" if self.group else ""
        return f"QTensor[{'x'.join(map(str, self.shape))}, {self.fmt.name}{g}, {self.nbytes} bytes]"


def _torch_types():
    try:
        import torch
        return (torch.Tensor, torch.bfloat16)
    except ImportError:                                  # pragma: no cover
        return (None, None)


_TORCH_TENSOR = _torch_types()


def _is_torch(a):
    try:
        import torch
        return isinstance(a, torch.Tensor)
    except ImportError:  # pragma: no cover
        return False


def _nbytes_of(a):
    if _is_torch(a):
        return a.numel() * a.element_size()
    return int(np.asarray(a).nbytes)


def _to_device_weight(x):
    """(torch CUDA tensor float32/bfloat16 [R, C], was_numpy)."""
    import torch
    if _is_torch(x):
        if not x.is_cuda:
            x = x.cuda()
        if x.dtype not in (torch.float32, torch.bfloat16):
            x = x.float()
        return x.contiguous(), False
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    return torch.from_numpy(a).cuda(), True


# ------------------------------------------------------------------------------------------------ quantise
def quantize(x, fmt, scale="auto", axis=None, group=None):
    """Quantise an array on the GPU (apsi/precision.py:216-246 semantics for int8 / int4).

    Supported: 2-D arrays with ``axis=0`` (one scale per row), and for int4 ``group=128`` (one scale per 128
    values along each row).  ``scale`` must be "auto"."""
    f = get_format(fmt)
    if scale != "auto":
        raise RuntimeErr("the B200 path quantises with scale='auto' (absmax) only")
    if f.kind == "minifloat":
        return _quantize_minifloat(x, f, axis)
    if getattr(x, "ndim", np.ndim(x)) != 2 or axis not in (0, -2):
        raise RuntimeErr("the B200 path quantises 2-D arrays with axis=0 (one scale per row, or per row group)")
    R, C = (int(s) for s in x.shape)
    if f.bits == 4:
        if group is None and C == 128:
            group = 128                                   # quantize(W.reshape(-1, 128), "int4", axis=0)
        if group != 128:
            raise RuntimeErr("int4 on the B200 path uses groups of 128 along the row (group=128)")
        if C % 128:
            raise RuntimeErr(f"int4 groups of 128 need a row length that is a multiple of 128 (got {C})")
    else:
        if group not in (None, C):
            raise RuntimeErr("int8 on the B200 path uses one scale per row (group=None)")
        if C % 8:
            raise RuntimeErr(f"int8 rows need a length that is a multiple of 8 (got {C})")
        group = None
    w, was_np = _to_device_weight(x)
    if f.bits == 4:
        codes, s16, s32 = _k.quant_int4_g128(w)
        scale_shape = (R * C // 128, 1) if group == 128 and C == 128 else (R, C // 128)
    else:
        codes, s16, s32 = _k.quant_int8_rows(w)
        scale_shape = (R, 1)
    if was_np:
        codes = codes.cpu().numpy().reshape(-1).view(np.uint8)
        s32 = s32.cpu().numpy().reshape(scale_shape)
        s16 = s16.cpu().numpy()
    else:
        s32 = s32.reshape(scale_shape)
    return QTensor(codes, s32, f, (R, C), axis, None, f.bits == 4, scale16=s16, group=group)


def _quantize_minifloat(x, f, axis):
    """Minifloat quantisation on the device (apsi/precision.py:205-246): axis=0 of a 2-D array (one float32
    scale per row, shaped [R, 1] as the reference returns it) or axis=None (one float64 scale for the tensor)."""
    if axis is None:
        shape = tuple(int(s) for s in np.shape(x))
        n = int(np.prod(shape)) if shape else 1
        if n == 0:
            raise RuntimeErr("cannot quantise an empty array")
        flat = x.reshape(1, n) if _is_torch(x) else np.asarray(x).reshape(1, n)
        w, was_np = _to_device_weight(flat)
    else:
        if getattr(x, "ndim", np.ndim(x)) != 2 or axis not in (0, -2):
            raise RuntimeErr("the B200 path quantises minifloats per tensor (axis=None) or per row of a 2-D array "
                             "(axis=0)")
        shape = tuple(int(s) for s in x.shape)
        w, was_np = _to_device_weight(x)
    R, C = (int(s) for s in w.shape)
    fmt_id = MINIFLOAT_FMT[f.name]
    codes, aux = _k.quant_minifloat(w, fmt_id, per_row=axis is not None)
    if axis is None:
        m = float(aux.cpu().numpy()[0])
        scale = m / f.max if (m > 0 and not math.isnan(m)) else 1.0      # the reference's float64 scale
    else:
        scale = aux.reshape(R, 1)
    if was_np:
        codes = codes.cpu().numpy()
        if axis is not None:
            scale = scale.cpu().numpy()
    packed = f.bits in (4, 6)
    if f.bits == 8:
        codes = codes.reshape(shape)
    return QTensor(codes, scale, f, shape, axis, None, packed)


def quantize_linear(W, fmt="int4", group=128):
    """An Apsi Linear weight ``W[in, out]`` quantised for the fused kernels: rows are the outputs, the scales run
    along the inputs (int8: one per output; int4: one per 128 inputs).  ``x @ q`` computes ``x @ W``.

    The rounding is the reference's own quantize applied to ``W.T`` (per output row / group)."""
    import torch
    f = get_format(fmt)
    if _is_torch(W):
        Wt = W.detach().t().contiguous()
    else:
        Wt = np.ascontiguousarray(np.asarray(W, np.float32).T)
    q = quantize(Wt, f, axis=0, group=group if f.bits == 4 else None)
    q.shape = (q.shape[1], q.shape[0])
    q.kn = True
    del torch
    return q


# ------------------------------------------------------------------------------------------------ dequantise
def dequantize(q):
    """float32 values ``code * scale`` (apsi/precision.py:249-274), computed on the GPU with the float32 scale
    (bit-exact with the reference).  Returns NumPy for host QTensors, a CUDA tensor for device ones."""
    if not isinstance(q, QTensor):
        return q
    import torch
    if q.fmt.kind == "minifloat":
        on_host = not _is_torch(q.codes)
        codes, sc = q.device_tensors()
        n = int(np.prod(q.shape)) if q.shape else 1
        R, C = (q.shape[0], n // q.shape[0]) if (q.axis is not None and q.shape) else (1, n)
        out = _k.dequant_minifloat(MINIFLOAT_FMT[q.fmt.name], codes.reshape(-1), R, C,
                                   sc.reshape(-1) if not isinstance(sc, float) else sc)
        return out.cpu().numpy().reshape(q.shape) if on_host else out.reshape(q.shape)
    R, C = q.rows
    fmt = q.kernel_format
    on_host = not _is_torch(q.codes)
    codes, _ = q.device_tensors()
    s32 = q.scale
    s32 = torch.from_numpy(np.ascontiguousarray(s32, np.float32)).to(codes.device) if on_host else s32
    out = _k.dequant(fmt, codes, s32.reshape(-1), R, C, out_dtype=torch.float32, scale_f32=True)
    if q.kn:
        out = out.t().contiguous()
    if on_host:
        return out.cpu().numpy().reshape(q.shape)
    return out.reshape(q.shape)


# ------------------------------------------------------------------------------------------------ products
def qmatmul(a, b, out=None):
    """``a @ b`` with a quantised right operand on the fused kernels (apsi/precision.py:294-299).

    The weights of a device QTensor are treated as static from its second decode product on: that launch
    streams them before the previous kernel on the stream has finished (programmatic dependent launch; the
    activations and the output still wait for it).  The first product after the QTensor's weight tensors were
    set runs without it, so the kernel that wrote them has completed.  After writing into ``codes`` or
    ``scale16`` in place, call ``b.touch()``.

    ``b`` must be a QTensor in the kernel layout (``quantize_linear``, or ``quantize(W, ..., axis=0)`` of a
    ``[N, K]`` weight, which multiplies as ``a @ W.T`` -- the hub / HF orientation).  ``a`` is ``[..., K]``:
    a CUDA tensor stays on the device (bfloat16 out); NumPy / CPU inputs are copied in and the result copied
    back as float32 (NumPy) or bfloat16 (torch).  ``out`` (B200 extension): a bfloat16 CUDA tensor ``[..., N]``
    to write into (CUDA inputs only)."""
    # per-call fast path: a contiguous bfloat16 CUDA matrix times a device int4 / int8 weight
    if type(b) is QTensor and type(a) is _TORCH_TENSOR[0]:
        spec = b.fast_spec()
        if spec is not None and a.dtype is _TORCH_TENSOR[1] and a.dim() == 2 and a.is_cuda:
            y = _k.linear_spec(spec, a, out, b._settled)
            if y is not None:
                b._settled = True
                return y
    import torch
    if isinstance(a, QTensor):
        raise RuntimeErr("the B200 path quantises the weight (right) operand only")
    if not isinstance(b, QTensor):
        raise RuntimeErr("qmatmul on the B200 path needs a quantised right operand")
    R, C = b.rows
    was_np = not _is_torch(a)
    if was_np:
        xa = np.asarray(a)
        xt = torch.from_numpy(np.ascontiguousarray(xa, np.float32))
    else:
        xt = a
    lead = tuple(xt.shape[:-1])
    if xt.shape[-1] != C:
        raise RuntimeErr(f"shapes {tuple(xt.shape)} and {b.shape} do not multiply")
    host = not xt.is_cuda
    dev = torch.device("cuda", torch.cuda.current_device()) if host else xt.device
    x2 = xt.reshape(-1, C)
    if x2.dtype != torch.bfloat16:
        x2 = x2.to(torch.bfloat16)
    x2 = x2.to(dev, non_blocking=True).contiguous()
    if b.fmt.kind == "minifloat":
        y = _minifloat_product(x2, b, R, C, dev, out if not host else None)
        if y is out and out is not None:
            return out
        y = y.reshape(*lead, R)
        if host:
            y = y.to("cpu")
        return y.float().numpy() if was_np else y
    codes, s16 = b.device_tensors(dev)
    if out is not None and not host:
        _k.linear(b.kernel_format, x2, codes, s16, R, out=out.view(-1, R))
        return out
    y = _k.linear(b.kernel_format, x2, codes, s16, R)
    y = y.reshape(*lead, R)
    if host:
        y = y.to("cpu")
    if was_np:
        return y.float().numpy()
    return y


def _minifloat_product(x2, b, R, C, dev, out):
    """x2 [M, C] bfloat16 @ W^T for a minifloat weight W [R, C].  fp8 e4m3 / e5m2: the fused kernels (codes to
    exact fp16, float32 row scales; a tensor scale is broadcast to the rows).  fp4 e2m1 with C % 128 == 0: the
    fused kernels the same way; fp6 e3m2 / e2m3: the fused decode product for M <= 16 (C % 16 == 0) and the
    tcgen05 GEMM above (C % 64 == 0).  Otherwise (fp6 / fp4 rows of other lengths): the library's
    dequantisation to float32 on the device, then a float32 library GEMM (the reference's own qmatmul order,
    apsi/precision.py:294-299)."""
    import torch
    from ._lib import FMT_FP8_E4M3, FMT_FP8_E5M2, FMT_FP4_E2M1, FMT_FP6_E3M2, FMT_FP6_E2M3
    fmt_id = b.kernel_format
    codes, sc = b.device_tensors(dev)
    fused = (fmt_id in (FMT_FP8_E4M3, FMT_FP8_E5M2) or (fmt_id == FMT_FP4_E2M1 and C % 128 == 0) or
             (fmt_id in (FMT_FP6_E3M2, FMT_FP6_E2M3) and
              ((x2.shape[0] <= 16 and C % 16 == 0) or C % 64 == 0)))
    if fused:
        if isinstance(sc, float):
            s32 = torch.full((R,), float(np.float32(sc)), dtype=torch.float32, device=dev)
        else:
            s32 = sc.reshape(-1)
        if out is not None:
            _k.linear(fmt_id, x2, codes, s32, R, out=out.view(-1, R))
            return out
        return _k.linear(fmt_id, x2, codes, s32, R)
    w = _k.dequant_minifloat(fmt_id, codes.reshape(-1), *((R, C) if not isinstance(sc, float) else (1, R * C)),
                             sc.reshape(-1) if not isinstance(sc, float) else sc).reshape(R, C)
    y = (x2.float() @ w.t()).to(torch.bfloat16)
    if out is not None:
        out.view(-1, R).copy_(y)
        return out
    return y


def round_to(x, fmt, scale="auto", axis=None, group=None):
    """What the format stores, as an ordinary float array (apsi/precision.py:278-292, no autodiff here)."""
    r = dequantize(quantize(x, fmt, scale, axis, group))
    return np.asarray(r, dtype=np.float64) if not _is_torch(r) else r


def nbytes(x):
    if isinstance(x, QTensor):
        return x.nbytes
    return _nbytes_of(x)


def quant_error(x, fmt, axis=0, group=None):
    """Relative RMS error of storing x in `fmt` (apsi/precision.py:310-316)."""
    xv = np.asarray(x, dtype=np.float64)
    r = np.asarray(round_to(np.asarray(x, np.float32), fmt, "auto", axis, group), dtype=np.float64)
    denom = math.sqrt(float(np.mean(xv * xv))) or 1.0
    return math.sqrt(float(np.mean((r - xv) ** 2))) / denom


# exponent bits, mantissa bits, bias, no infinities, top code of the top binade is NaN: the OCP fp8 and MX fp6 /
# fp4 element formats (the reference's table, apsi/precision.py:65-72)
_MF_SPEC = {"fp8_e4m3": (4, 3, 7, True, True), "fp8_e5m2": (5, 2, 15, False, False),
            "fp6_e3m2": (3, 2, 3, True, False), "fp6_e2m3": (2, 3, 1, True, False),
            "fp4_e2m1": (2, 1, 1, True, False)}


def _minifloat_magnitudes(name):
    """Value of every sign-less code of a minifloat format (inf / NaN where the format has them)."""
    E, Mb, bias, finite_only, nan_top = _MF_SPEC[name]
    code = np.arange(1 << (E + Mb))
    e, m = code >> Mb, code & ((1 << Mb) - 1)
    frac = m / float(1 << Mb)
    v = np.where(e == 0, frac * 2.0 ** (1 - bias), (1.0 + frac) * 2.0 ** (e - bias))
    top = e == (1 << E) - 1
    if not finite_only:
        v = np.where(top, np.where(m == 0, np.inf, np.nan), v)
    if nan_top:
        v = np.where(top & (m == (1 << Mb) - 1), np.nan, v)
    return v


def format_info(fmt):
    """name, bits, largest finite value, relative spacing (eps) and smallest positive value of a format
    (apsi/precision.py:319-331); minifloats also give the number of distinct finite values.  Accepts every
    name the reference knows, including the formats whose quantisation is not on the B200 path."""
    name = getattr(fmt, "name", fmt)
    name = ALIASES.get(name, name)
    native = {"f64": np.float64, "f32": np.float32, "f16": np.float16}
    if name in native:
        fi = np.finfo(native[name])
        return {"name": name, "bits": fi.bits, "max": float(fi.max), "eps": float(fi.eps), "tiny": float(fi.tiny)}
    if name == "bf16":
        return {"name": "bf16", "bits": 16, "max": 3.3895313892515355e38, "eps": 2.0 ** -7, "tiny": 2.0 ** -126}
    if name == "uint8":
        return {"name": "uint8", "bits": 8, "max": 255.0, "eps": 1.0, "tiny": 1.0}
    f = get_format(name)
    if f.kind == "minifloat":
        v = _minifloat_magnitudes(f.name)
        fin = v[np.isfinite(v)]
        return {"name": f.name, "bits": f.bits, "max": f.max, "eps": 2.0 ** -_MF_SPEC[f.name][1],
                "tiny": float(fin[fin > 0].min()), "values": int(fin.size * 2 - 1)}
    return {"name": f.name, "bits": f.bits, "max": f.max, "eps": 1.0, "tiny": 1.0}


def module():
    return {"quantize": quantize, "dequantize": dequantize, "round_to": round_to, "qmatmul": qmatmul,
            "nbytes": nbytes, "quant_error": quant_error, "format_info": format_info,
            "quantize_linear": quantize_linear}


__all__ += ["LowbitError"]
