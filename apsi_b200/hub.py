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
* the rest of the whole-decoder interface (``full = True``; apsi/hub_gpu.py:1534-1600): ``matrix`` (a dense
  bfloat16 matrix, for the tied embedding / head), ``embed``, ``qkv_prep`` (``lb_qkv_prep``: split, optional
  q / k norms, half-split rotary from float32 cos / sin tables, cache write), ``attention`` (causal, optional
  sliding window, grouped heads, over the [kv heads, capacity, head dim] cache), ``act_mul`` (``lb_act_mul``),
  ``alloc_kv`` / ``copy_kv``, ``sample_prep``, ``copy``, ``trim``.

Representation: a ``Buf`` is a CUDA allocation of ``n`` float32-sized slots, as the reference's buffers are
float32.  The library's kernels read and write bfloat16, so a buffer holds one of two forms, recorded in
``Buf.kind``: "bf16" (the first ``n`` bfloat16 values of the storage, written by the products and the decoder
kernels) or "f32" (all of it, written by ``put``, the reference's convention: float32 tables such as RoPE's,
int32 token ids viewed as float32, norm weights).  An operation that needs the other form converts the buffer
in place once (activations put from the host are rounded to bfloat16 there, nearest even); ``get`` returns
float32 either way.  Attention and sampling are torch operations (they are not on the quantized-linear path).
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
    """Device memory of `n` elements in float32-sized slots (a CUDA tensor ``raw``; see the module docstring
    for the two forms it holds).  ``t``: the bfloat16 view of the first n elements; ``f``: the float32 view."""
    __slots__ = ("raw", "n", "kind")

    def __init__(self, raw, n=None, kind="bf16"):
        self.raw, self.kind = raw, kind
        self.n = raw.numel() if n is None else int(n)

    @property
    def t(self):
        return self.raw.view(torch.bfloat16)[:self.n]

    @property
    def f(self):
        if self.raw.numel() < self.n:
            raise LowbitError(LB_E_ARG, "this buffer holds bfloat16 only (a key / value cache)")
        return self.raw[:self.n]

    @property
    def ptr(self):
        return self.raw.data_ptr()

    def as_bf16(self):
        """The bfloat16 view, converting float32 contents in place first."""
        if self.kind == "f32":
            self.t.copy_(self.raw[:self.n].to(torch.bfloat16))
            self.kind = "bf16"
        return self.t

    def as_f32(self):
        """The float32 view, converting bfloat16 contents in place first."""
        if self.kind == "bf16":
            self.f.copy_(self.t.float())
            self.kind = "f32"
        return self.f

    def written_bf16(self):
        """The bfloat16 view for an operation that overwrites the buffer's front."""
        if self.kind == "f32":
            self.as_bf16()
        return self.t


class Matrix:
    """Packed codes with fp16 scales (kind "int4": groups of 128 along cols; "int8": one scale per row), or a dense
    bfloat16 matrix (kind "bf16": ``buf`` the [rows, cols] tensor, no scales)."""
    __slots__ = ("buf", "rows", "cols", "kind", "scales", "fmt")

    def __init__(self, codes, rows, cols, kind, scales, fmt):
        self.buf, self.rows, self.cols, self.kind, self.scales, self.fmt = codes, rows, cols, kind, scales, fmt

    @property
    def bits(self):
        return {FMT_INT4_G128: 4, FMT_INT8_ROW: 8}.get(self.fmt, 16)


def _kind(kind):
    k = str(kind).strip().lower()
    k = parse_linear(k) or k
    if k not in _KIND_FMT:
        raise LowbitError(LB_E_UNSUPPORTED, f"weight format '{kind}' has no fused product here (int4, int8)")
    return ("int4" if _KIND_FMT[k] == FMT_INT4_G128 else "int8"), _KIND_FMT[k]


class _Dev:
    """The device facts the reference reads from its ops object (``r.dev.index``, ``r.dev.memory``)."""

    def __init__(self, dev):
        self.index = dev.index
        self.memory = torch.cuda.get_device_properties(dev).total_memory
        self.sms = torch.cuda.get_device_properties(dev).multi_processor_count


class Ops:
    """The device ops object (one CUDA device)."""
    full = True                       # runs hub_models.Decoder's whole-network path (every op below)
    name = "B200 low-bit kernels"

    def __init__(self, device=0):
        self.dev_t = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        if self.dev_t.type != "cuda":
            raise LowbitError(LB_E_ARG, "Ops needs a CUDA device (the B200 path has no CPU fallback)")
        if self.dev_t.index is None:
            self.dev_t = torch.device("cuda", torch.cuda.current_device())
        self.dev = _Dev(self.dev_t)
        self.used = 0
        self._own = []
        self._ws = {}

    # ---- memory
    def alloc(self, n):
        b = Buf(torch.zeros(max(int(n), 1), dtype=torch.float32, device=self.dev_t))
        self._own.append(b)
        self.used += 4 * b.raw.numel()
        return b

    def free(self, b):
        if isinstance(b, Matrix):
            b = b.buf
        if b in self._own:
            self._own.remove(b)
            self.used -= 4 * b.raw.numel()
            b.raw = torch.empty(0, dtype=torch.float32, device=self.dev_t)
            b.n = 0

    def put(self, b, a, off=0):
        """Write host values at element `off` (float32; uint32 / int32 arrays are stored bit for bit)."""
        a = np.ascontiguousarray(a).reshape(-1)
        if a.dtype in (np.uint32, np.int32):
            a = a.view(np.float32)
        src = torch.from_numpy(np.asarray(a, np.float32))
        if off + src.numel() > b.n:
            raise LowbitError(LB_E_ARG, "put: past the end of the buffer")
        b.as_f32()[off:off + src.numel()].copy_(src.to(self.dev_t))

    def get(self, b, n, off=0):
        if b.kind == "f32":
            return b.raw[off:off + n].cpu().numpy().copy()
        return b.t[off:off + n].float().cpu().numpy()

    def copy(self, dst, doff, src, soff, n):
        if src.kind == "f32":
            dst.as_f32()[doff:doff + n].copy_(src.raw[soff:soff + n])
        else:
            dst.written_bf16()[doff:doff + n].copy_(src.t[soff:soff + n])

    def begin(self):
        """Start of a batch of launches (kept for the reference's call sequence; nothing to do here)."""

    def vec(self, a):
        a = np.asarray(a, np.float32).reshape(-1)
        b = self.alloc(max(1, a.size))
        self.put(b, a)
        return b

    def ws(self, name, n):
        """A scratch buffer of at least n elements that grows as needed."""
        b = self._ws.get(name)
        if b is None or b.n < n:
            if b is not None:
                self.free(b)
            b = self._ws[name] = self.alloc(max(n, 2 * (b.n if b else 0), 64))
        return b

    def trim(self):
        """Drop the scratch buffers (they are made again on demand)."""
        for b in list(self._ws.values()):
            self.free(b)
        self._ws = {}

    def alloc_kv(self, n, half):
        """A key / value cache buffer of n elements.  The cache is bfloat16 whatever `half` asks (this library's
        qkv_prep writes bfloat16 and attention reads it)."""
        b = Buf(torch.zeros(max((int(n) + 1) // 2, 1), dtype=torch.float32, device=self.dev_t), n=int(n))
        self._own.append(b)
        self.used += 4 * b.raw.numel()
        return b

    def copy_kv(self, dst, doff, src, soff, n, half):
        dst.t[doff:doff + n].copy_(src.t[soff:soff + n])

    # ---- weights
    def _device_weight(self, w):
        if isinstance(w, torch.Tensor):
            wt = w.to(self.dev_t)
            if wt.dtype not in (torch.float32, torch.bfloat16):
                wt = wt.float()
        elif np.asarray(w).dtype == np.uint16:       # bfloat16 bits
            wt = torch.from_numpy(np.ascontiguousarray(w).view(np.int16)).to(self.dev_t).view(torch.bfloat16)
        else:
            wt = torch.from_numpy(np.ascontiguousarray(np.asarray(w, np.float32))).to(self.dev_t)
        return wt.contiguous()

    def qmatrix(self, w, kind):
        """A [rows, cols] weight quantised on the device for the fused kernels ("bf16": a dense matrix)."""
        if str(kind).strip().lower() == "bf16":
            return self.matrix(w)
        k, fmt = _kind(kind)
        wt = self._device_weight(w)
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

    def matrix(self, w):
        """A dense [rows, cols] bfloat16 matrix (float32 is rounded; uint16 is taken as bfloat16 bits)."""
        wt = self._device_weight(w).to(torch.bfloat16)
        rows, cols = wt.shape
        self.used += 2 * wt.numel()
        return Matrix(wt, rows, cols, "bf16", None, None)

    upload = matrix

    # ---- products
    def rms(self, X, Y, W, rows, n, eps, off, xoff=0, yoff=0):
        """Y[yoff:] = X[xoff:] / sqrt(mean(X^2) + eps) * (W + off) for `rows` rows of n (hub_gpu rms)."""
        if X.n < xoff + rows * n or Y.n < yoff + rows * n or W.n < n:
            raise LowbitError(LB_E_ARG, "rms: buffers too small")
        x = X.as_bf16()[xoff:xoff + rows * n].view(rows, n)
        w = W.f[:n] if W.kind == "f32" else W.t[:n]
        _k.rmsnorm(x, w, eps=eps, off=off, out=Y.written_bf16()[yoff:yoff + rows * n].view(rows, n))

    def linear(self, m, X, Y, T, bias=None, acc=False, ln=None, eps=1e-6, off=0.0, xoff=0):
        """Y (+)= norm(X) @ W.T (+ bias) for T rows (X: [T, cols] from element xoff, Y: [T, rows]); ln: RMSNorm
        weights applied to each row of X first."""
        if X.n < xoff + T * m.cols or Y.n < T * m.rows:
            raise LowbitError(LB_E_ARG, "linear: buffers too small for T rows")
        x = X.as_bf16()[xoff:xoff + T * m.cols].view(T, m.cols)
        y = (Y.as_bf16() if acc else Y.written_bf16())[:T * m.rows].view(T, m.rows)
        b = bias.as_bf16()[:m.rows] if bias is not None else None
        lnw = None
        if ln is not None:
            if ln.n < m.cols:
                raise LowbitError(LB_E_ARG, "linear: ln holds fewer than cols values")
            lnw = ln.f[:m.cols] if ln.kind == "f32" else ln.t[:m.cols]
        if m.fmt is None:                        # a dense bfloat16 matrix (tied embedding / head): library GEMM
            if lnw is not None:
                x = _k.rmsnorm(x, lnw, eps=eps, off=off)
            r = torch.matmul(x, m.buf.t())
            if b is not None:
                r = r + b
            if acc:
                y.add_(r)
            else:
                y.copy_(r)
            return
        if lnw is not None:                      # the norm inside the decode GEMV (T <= 16), else lb_rmsnorm first
            _k.linear_rms(m.fmt, x, lnw, m.buf, m.scales, m.rows, eps=eps, off=off, bias=b, out=y,
                          accumulate=bool(acc))
            return
        _k.linear(m.fmt, x, m.buf, m.scales, m.rows, bias=b, out=y, accumulate=bool(acc))

    def gemv(self, m, X, Y, T, xoff=0, yoff=0, bias=None, acc=False, ln=None, eps=1e-6, off=0.0):
        if yoff:
            Y = _Offset(Y, yoff)
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

    # ---- the rest of a decoder layer
    def embed(self, m, ids, X, scale=1.0):
        """X[t] = row ids[t] of the bfloat16 matrix m (times scale)."""
        idx = torch.as_tensor(np.ascontiguousarray(ids, np.int64).reshape(-1)).to(self.dev_t)
        rows = m.buf.index_select(0, idx)
        if scale != 1.0:
            rows = (rows.float() * scale).to(torch.bfloat16)
        X.written_bf16()[:idx.numel() * m.cols].view(idx.numel(), m.cols).copy_(rows)

    def qkv_prep(self, QKV, Q, Kc, Vc, COS, SIN, QN, KN, T, nh, kvh, dh, rot, start, cap, eps, half=False):
        """The fused projection QKV [T, (nh + 2 kvh) dh] -> Q [T, nh, dh] and cache slots [start, start + T) of
        Kc / Vc [kvh, cap, dh]: optional per-head RMSNorm (QN / KN), half-split rotary of the first `rot` values
        with the float32 tables COS / SIN [positions, rot / 2] (lb_qkv_prep; hub_gpu.py:1575-1581)."""
        width = (nh + 2 * kvh) * dh
        qkv = QKV.as_bf16()[:T * width].view(T, width)
        q = Q.written_bf16()
        qn = QN.as_bf16()[:dh] if QN is not None else None
        kn = KN.as_bf16()[:dh] if KN is not None else None
        cos = COS.as_f32()
        sin = SIN.as_f32()
        with torch.cuda.device(self.dev_t):
            _k._lib.call("lb_qkv_prep", qkv.data_ptr(), 1, T, nh, kvh, dh, rot, cos.data_ptr(), sin.data_ptr(),
                         qn.data_ptr() if qn is not None else None, kn.data_ptr() if kn is not None else None,
                         _k.ctypes.c_float(eps), None, int(start), q.data_ptr(), 0, nh * dh, dh,
                         Kc.t.data_ptr(), Vc.t.data_ptr(), kvh * cap * dh, cap * dh,
                         torch.cuda.current_stream(self.dev_t).cuda_stream)

    def attention(self, Q, Kc, Vc, O, S, T, nh, kvh, dh, start, cap, window, scale, splits=None, half=False):
        """O [T, nh dh] = softmax(scale Q K^T + causal / window mask) V over cache slots [0, start + T) of
        Kc / Vc [kvh, cap, dh]; query t sits at position start + t.  A torch operation (S is unused)."""
        import torch.nn.functional as F
        L = start + T
        q = Q.as_bf16()[:T * nh * dh].view(T, nh, dh).transpose(0, 1)          # [nh, T, dh]
        k = Kc.t[:kvh * cap * dh].view(kvh, cap, dh)[:, :L]
        v = Vc.t[:kvh * cap * dh].view(kvh, cap, dh)[:, :L]
        qp = torch.arange(start, L, device=self.dev_t)[:, None]
        kp = torch.arange(L, device=self.dev_t)[None, :]
        allowed = kp <= qp
        if window:
            allowed = allowed & (qp - kp < window)
        mask = torch.zeros((T, L), dtype=torch.bfloat16, device=self.dev_t).masked_fill_(~allowed, float("-inf"))
        o = F.scaled_dot_product_attention(q[None], k[None], v[None], attn_mask=mask, scale=float(scale),
                                           enable_gqa=True)[0]                   # [nh, T, dh]
        O.written_bf16()[:T * nh * dh].view(T, nh, dh).copy_(o.transpose(0, 1))

    def act_mul(self, GU, M, T, I, kind):
        """M[t] = act(G[t]) * U[t] of GU [T, 2 I] = [G | U] (lb_act_mul; kind 0 silu, 1 gelu tanh form)."""
        gu = GU.as_bf16()[:T * 2 * I].view(T, 2 * I)
        _k.act_mul(gu, I, int(kind), out=M.written_bf16()[:T * I].view(T, I))

    def sample_prep(self, LOG, SEEN, V, rp, inv_t, delta, cap):
        """(max, softmax denominator, candidate ids, their scaled logits, how many there were) for the logits in
        LOG after the repetition penalty (SEEN marks the tokens) and the temperature (hub_gpu.py:1583-1596)."""
        lg = (LOG.f[:V] if LOG.kind == "f32" else LOG.t[:V].float()).clone()
        seen = (SEEN.f[:V] if SEEN.kind == "f32" else SEEN.t[:V].float()) != 0
        lg = torch.where(seen, torch.where(lg > 0, lg / rp, lg * rp), lg) * float(inv_t)
        g = lg.max()
        Z = torch.exp((lg - g).double()).sum()
        ids = torch.nonzero(lg >= g - delta).flatten()
        return (float(g), float(Z), ids[:cap].cpu().numpy().astype(np.int64), lg[ids[:cap]].cpu().numpy(),
                int(ids.numel()))

    @property
    def memory(self):
        return self.dev.memory

    def free_memory(self):
        free, _ = torch.cuda.mem_get_info(self.dev_t)
        return free

    def close(self):
        for b in list(self._own):
            self.free(b)
        self._own, self._ws, self.used = [], {}, 0


class _Offset:
    """A view of a buffer from element `off` (gemv's yoff), in bfloat16 form."""

    def __init__(self, b, off):
        self.base, self.off = b, off
        self.n = b.n - off
        self.kind = "bf16"

    def as_bf16(self):
        return self.base.as_bf16()[self.off:]

    def written_bf16(self):
        return self.base.written_bf16()[self.off:]

    @property
    def t(self):
        return self.base.t[self.off:]


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
