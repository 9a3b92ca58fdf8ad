"""A ``hub_gpu``-compatible device ops object for the quantized projections (apsi/hub_gpu.py:1160-1362).

``hub_models.Decoder`` drives the GPU through a duck-typed ops object: ``qmatrix(w, kind)`` to put a weight on
the device, ``linear(m, X, Y, T, bias, acc)`` for every projection, plus ``alloc / free / put / get / begin /
close``.  ``Ops`` keeps those names and argument meanings for the packed formats of this library, backed by
its kernels:

* ``qmatrix(w, "int4")`` -- int4, one fp16 scale per 128 inputs (``"int4_g128"`` / ``"w4g128"`` too);
  ``qmatrix(w, "int8")`` -- int8, one fp16 scale per row.  ``w`` is ``[rows, cols]`` = ``[out, in]``
  (float32, or uint16 bfloat16 bits, as the reference takes it).  Quantised on the device, bit-exact with
  ``precision.quantize``.  The reference's g32 ggml formats and minifloats are not products here and raise.
* ``linear(m, X, Y, T, bias=None, acc=False, ln=None, eps=1e-6, off=0.0, xoff=0)`` -- ``Y (+)= norm(X) @ W.T
  (+ bias)`` for T rows: the decode GEMV for T <= 16, the tcgen05 GEMM above.  With ``ln`` (RMSNorm weights)
  the rows are first normalised (``x / sqrt(mean(x^2) + eps) * (ln + off)``, float32 arithmetic, rounded once
  to bf16) by ``lb_linear_rms``: inside the decode GEMV's activation staging for T <= 16 (the reference's
  gemvq*n kernels), by ``lb_rmsnorm`` into a workspace before the GEMM above (its ``rms`` op).
* ``rms(X, Y, W, rows, n, eps, off, xoff=0, yoff=0)`` -- that normalisation on its own.
* ``gemv``, ``gemm``, ``matmul``, ``matmul_rows`` -- the same product under the reference's other names.

One difference in representation: a ``Buf`` here holds bfloat16 elements in a CUDA tensor.  The reference
holds float32, and the fused kernels read and write bfloat16.  ``put`` rounds float32 input to bfloat16
(nearest even), and ``get`` returns float32.
"""
import threading

import numpy as np
import torch

from . import kernels as _k
from ._lib import LowbitError, LB_E_ARG, LB_E_UNSUPPORTED, FMT_INT4_G128, FMT_INT8_ROW
from .lowbit import parse_linear

__all__ = ["Buf", "Matrix", "Ops", "QBYTES", "runner", "GEMM_ROWS"]

GEMM_ROWS = 17                       # T < GEMM_ROWS: the decode GEMV; else the tensor-core GEMM
QBYTES = {"bf16": 2.0, "int8": 1.0, "int4": 0.515625}   # bytes per weight on the device, scales included
_KIND_FMT = {"int4": FMT_INT4_G128, "int4_g128": FMT_INT4_G128, "int8": FMT_INT8_ROW, "int8_row": FMT_INT8_ROW}
_lock = threading.Lock()


class Buf:
    """Device memory: `n` bfloat16 elements (a CUDA tensor ``t``); ``ptr`` is its address."""
    __slots__ = ("t", "n")

    def __init__(self, t):
        self.t, self.n = t, t.numel()

    @property
    def ptr(self):
        return self.t.data_ptr()


class Matrix:
    """Packed codes with fp16 scales (kind "int4": groups of 128 along cols; "int8": one scale per row)."""
    __slots__ = ("buf", "rows", "cols", "kind", "scales", "fmt")

    def __init__(self, codes, rows, cols, kind, scales, fmt):
        self.buf, self.rows, self.cols, self.kind, self.scales, self.fmt = codes, rows, cols, kind, scales, fmt

    @property
    def bits(self):
        return 4 if self.fmt == FMT_INT4_G128 else 8


def _kind(kind):
    k = str(kind).strip().lower()
    k = parse_linear(k) or k
    if k not in _KIND_FMT:
        raise LowbitError(LB_E_UNSUPPORTED, f"weight format '{kind}' has no fused product here (int4, int8)")
    return ("int4" if _KIND_FMT[k] == FMT_INT4_G128 else "int8"), _KIND_FMT[k]


class Ops:
    """The device ops object (one CUDA device)."""
    full = False                      # projections only: hub_models.Decoder's other kernels are not here

    def __init__(self, device=0):
        self.dev = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if self.dev.type != "cuda":
            raise LowbitError(LB_E_ARG, "Ops needs a CUDA device (the B200 path has no CPU fallback)")
        self.used = 0
        self._own = []
        self._ws = {}

    # ---- memory
    def alloc(self, n):
        b = Buf(torch.empty(max(int(n), 1), dtype=torch.bfloat16, device=self.dev))
        self._own.append(b)
        self.used += 2 * b.n
        return b

    def free(self, b):
        if b in self._own:
            self._own.remove(b)
            self.used -= 2 * b.n
            b.t = torch.empty(0, dtype=torch.bfloat16, device=self.dev)

    def put(self, b, a, off=0):
        src = torch.as_tensor(np.ascontiguousarray(np.asarray(a, np.float32)).reshape(-1))
        if off + src.numel() > b.n:
            raise LowbitError(LB_E_ARG, "put: past the end of the buffer")
        b.t[off:off + src.numel()].copy_(src.to(self.dev, non_blocking=False).to(torch.bfloat16))

    def get(self, b, n, off=0):
        return b.t[off:off + n].float().cpu().numpy()

    def begin(self):
        """Start of a batch of launches (kept for the reference's call sequence; nothing to do here)."""

    def vec(self, a):
        a = np.asarray(a, np.float32).reshape(-1)
        b = self.alloc(max(1, a.size))
        self.put(b, a)
        return b

    def ws(self, name, n):
        b = self._ws.get(name)
        if b is None or b.n < n:
            if b is not None:
                self.free(b)
            b = self._ws[name] = self.alloc(max(n, 2 * (b.n if b else 0), 64))
        return b

    # ---- weights
    def qmatrix(self, w, kind):
        """A [rows, cols] weight quantised on the device for the fused kernels."""
        k, fmt = _kind(kind)
        if isinstance(w, torch.Tensor):
            wt = w.to(self.dev)
            if wt.dtype not in (torch.float32, torch.bfloat16):
                wt = wt.float()
        elif np.asarray(w).dtype == np.uint16:       # bfloat16 bits
            wt = torch.from_numpy(np.ascontiguousarray(w).view(np.int16)).to(self.dev).view(torch.bfloat16)
        else:
            wt = torch.from_numpy(np.ascontiguousarray(np.asarray(w, np.float32))).to(self.dev)
        wt = wt.contiguous()
        rows, cols = wt.shape
        if fmt == FMT_INT4_G128:
            if cols % 128:
                raise LowbitError(LB_E_ARG, f"int4 needs cols % 128 == 0 (got {cols})")
            codes, s16, _ = _k.quant_int4_g128(wt, want_scale32=False)
        else:
            if cols % 64:
                raise LowbitError(LB_E_ARG, f"int8 needs cols % 64 == 0 (got {cols})")
            codes, s16, _ = _k.quant_int8_rows(wt, want_scale32=False)
        self.used += codes.numel() + 2 * s16.numel()
        return Matrix(codes, rows, cols, k, s16, fmt)

    # ---- products
    def rms(self, X, Y, W, rows, n, eps, off, xoff=0, yoff=0):
        """Y[yoff:] = X[xoff:] / sqrt(mean(X^2) + eps) * (W + off) for `rows` rows of n (hub_gpu rms)."""
        if X.n < xoff + rows * n or Y.n < yoff + rows * n or W.n < n:
            raise LowbitError(LB_E_ARG, "rms: buffers too small")
        _k.rmsnorm(X.t[xoff:xoff + rows * n].view(rows, n), W.t[:n], eps=eps, off=off,
                   out=Y.t[yoff:yoff + rows * n].view(rows, n))

    def linear(self, m, X, Y, T, bias=None, acc=False, ln=None, eps=1e-6, off=0.0, xoff=0):
        """Y (+)= norm(X) @ W.T (+ bias) for T rows (X: [T, cols] from element xoff, Y: [T, rows]); ln: RMSNorm
        weights applied to each row of X first."""
        if X.n < xoff + T * m.cols or Y.n < T * m.rows:
            raise LowbitError(LB_E_ARG, "linear: buffers too small for T rows")
        x = X.t[xoff:xoff + T * m.cols].view(T, m.cols)
        y = Y.t[:T * m.rows].view(T, m.rows)
        b = bias.t[:m.rows] if bias is not None else None
        if ln is not None:                       # the norm inside the decode GEMV (T <= 16), else lb_rmsnorm first
            if ln.n < m.cols:
                raise LowbitError(LB_E_ARG, "linear: ln holds fewer than cols values")
            _k.linear_rms(m.fmt, x, ln.t[:m.cols], m.buf, m.scales, m.rows, eps=eps, off=off, bias=b, out=y,
                          accumulate=bool(acc))
            return
        _k.linear(m.fmt, x, m.buf, m.scales, m.rows, bias=b, out=y, accumulate=bool(acc))

    def gemv(self, m, X, Y, T, xoff=0, yoff=0, bias=None, acc=False, ln=None, eps=1e-6, off=0.0):
        if yoff:
            Y = Buf(Y.t[yoff:])
        self.linear(m, X, Y, T, bias=bias, acc=acc, ln=ln, eps=eps, off=off, xoff=xoff)

    def gemm(self, m, X, Y, T, xoff=0, bias=None, acc=False):
        self.linear(m, X, Y, T, bias=bias, acc=acc, xoff=xoff)

    def matmul(self, x, m):
        """x @ W.T with x on the host (float32 in, float32 out)."""
        lead = x.shape[:-1]
        x2 = np.ascontiguousarray(np.asarray(x, np.float32).reshape(-1, m.cols))
        T = x2.shape[0]
        with _lock:
            xb = self.ws("mm_x", x2.size)
            yb = self.ws("mm_y", T * m.rows)
            self.put(xb, x2.reshape(-1))
            self.linear(m, xb, yb, T)
            y = self.get(yb, T * m.rows)
        return y.reshape(*lead, m.rows)

    matmul_rows = matmul

    def free_memory(self):
        free, _ = torch.cuda.mem_get_info(self.dev)
        return free

    def close(self):
        for b in list(self._own):
            self.free(b)
        self._own, self._ws, self.used = [], {}, 0


def runner(device="auto"):
    """(Ops or None, why not), as hub_gpu.runner: device "auto", "cuda" or "cuda:N"."""
    d = str(device or "auto").lower()
    if d == "cpu":
        return None, "device=cpu"
    if not torch.cuda.is_available():
        return None, "no CUDA device"
    idx = 0
    if d.startswith("cuda:"):
        try:
            idx = int(d[5:])
        except ValueError:
            return None, f"unknown device '{device}'"
    elif d not in ("auto", "cuda", "gpu"):
        return None, f"unknown device '{device}' (use auto, cpu, cuda or cuda:N)"
    if idx >= torch.cuda.device_count():
        return None, f"no GPU {idx}"
    try:
        return Ops(idx), ""
    except LowbitError as e:
        return None, str(e)
