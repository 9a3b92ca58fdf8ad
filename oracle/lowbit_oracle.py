"""CPU restatement of Apsi's low-bit quantisation and quantized products (TEST INFRASTRUCTURE).

This module is the parity oracle.  It is pinned against golden vectors written by the reference itself
(``tests/golden/make_golden.py`` imports ``apsi.precision`` / ``apsi.hub_gpu`` and stores their outputs), and
the tests check every function here against those vectors before trusting it.  Nothing in ``apsi_b200`` may
import it: the CUDA path is the product, this is the checker.

Formats restated (reference file:line in ATECTechnologies/apsi):

* symmetric absmax int8 / int4 with one scale per segment -- ``apsi/precision.py:205-246``
  (``_scale_for`` + ``quantize``): absmax in float64, ``s = m / qmax`` when m > 0 else 1.0, cast to float32;
  codes ``clip(rint(x64 / s), -qmax, qmax)`` (round half to even on the float64 quotient).
* int4 packing -- ``apsi/precision.py:168-179`` (``_pack4`` / ``_unpack4``): two's-complement nibbles, the even
  flat index in the low nibble.
* int4 with one scale per 128 values along K -- ``precision.quantize(W.reshape(-1, 128), "int4", axis=0)``; the
  stored scale is float16(scale_fp32), round to nearest even.
* dequantisation -- ``apsi/precision.py:249-274``: ``float32(code) * float32(scale)``.
* quantized product -- ``apsi/precision.py:294-299`` (``qmatmul``): dequantise and multiply.
* ggml-style blocks of 32 (``hub_gpu.qnumpy``) -- ``apsi/hub_gpu.py:1215-1241``; the device word layout of
  those codes -- ``apsi/hub_gpu.py:786-800`` (int8: byte j of a word = value j; int4: nibble j = q + 8).
* minifloat formats (fp8 e4m3 / e5m2, fp6 e3m2 / e2m3, fp4 e2m1) -- ``apsi/precision.py:23-138, 182-246``:
  value tables, round-to-nearest-even onto the grid with saturation, 6-bit packing, per-row / per-tensor scales.
* GGUF Q8_0 / Q4_0 block bytes -- ``apsi/modelio.py:56-95``.
"""
import math

import numpy as np

__all__ = [
    "bf16_round", "bf16_to_f32", "f32_to_bf16_bits", "scale_for_segments", "quant_segments", "pack4", "unpack4",
    "quant_int8_rows", "quant_int4_g128", "dequant_int8_rows", "dequant_int4_g128", "linear_ref",
    "qnumpy_g32", "pack_q4_0_words", "pack_q8_0_words", "dequant_g32", "rel_frobenius", "max_abs_ratio",
    "make_config_inputs", "qmatmul_dequant_reference", "round_weights_g32",
    "MINIFLOATS", "minifloat_table", "minifloat_max", "minifloat_encode", "minifloat_decode", "pack6", "unpack6",
    "quant_minifloat", "dequant_minifloat", "gguf_q8_0", "gguf_q4_0", "gguf_dequant",
]


# ------------------------------------------------------------------------------------------- bfloat16 helpers
def f32_to_bf16_bits(a):
    """float32 -> bfloat16 bit patterns (uint16), round to nearest even; NaN -> 0x7FC0."""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = 0x7FC0
    return r


def bf16_to_f32(bits):
    return (np.ascontiguousarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(a):
    """float32 values rounded to the nearest bfloat16 (returned as float32)."""
    return bf16_to_f32(f32_to_bf16_bits(a)).reshape(np.shape(a))


# ------------------------------------------------------------------------------------------- absmax segments
def scale_for_segments(seg, qmax):
    """One float32 scale per row of ``seg`` ([S, L]): absmax in float64, ``m / qmax`` if m > 0 else 1.0.

    precision.py:205-213 with ``axis=0`` of a 2-D view (the reduction covers every axis but 0)."""
    m = np.max(np.abs(np.asarray(seg, np.float64)), axis=1)
    return np.where(m > 0, m / float(qmax), 1.0).astype(np.float32)


def quant_segments(seg, qmax):
    """Codes (int8 values) and float32 scales for absmax quantisation of each row of ``seg``.

    precision.py:226-232: the quotient is taken in float64 against the float32 scale, rounded half to even
    by ``np.rint`` and clipped to +-qmax."""
    seg64 = np.asarray(seg, np.float64)
    s = scale_for_segments(seg64, qmax)
    y = seg64 / s.astype(np.float64)[:, None]
    codes = np.clip(np.rint(y), -qmax, qmax).astype(np.int8)
    return codes, s


def pack4(codes):
    """int4 codes (int8 values in [-8, 7]) -> packed bytes; element 2j in the low nibble of byte j.

    precision.py:168-172 (odd lengths padded with a zero nibble)."""
    flat = np.ascontiguousarray(codes).reshape(-1).view(np.uint8) & np.uint8(0x0F)
    if flat.size % 2:
        flat = np.concatenate([flat, np.zeros(1, np.uint8)])
    return (flat[0::2] | (flat[1::2] << np.uint8(4))).astype(np.uint8)


def unpack4(packed, n):
    """Packed bytes -> signed int4 codes as int8 (precision.py:175-179 followed by the c > 7 -> c - 16 step of
    precision.py:265-266)."""
    p = np.ascontiguousarray(packed, np.uint8).reshape(-1)
    out = np.empty(p.size * 2, np.int16)
    out[0::2] = p & 0x0F
    out[1::2] = p >> 4
    out = np.where(out > 7, out - 16, out)
    return out[:n].astype(np.int8)


# ------------------------------------------------------------------------------------------- row / group formats
def quant_int8_rows(W):
    """int8 with one absmax scale per output row: ``precision.quantize(W, "int8", axis=0)``.

    Returns (codes int8 [N, K], scale fp32 [N], scale fp16 [N])."""
    W = np.asarray(W)
    codes, s = quant_segments(W.reshape(W.shape[0], -1), 127)
    return codes.reshape(W.shape), s, s.astype(np.float16)


def quant_int4_g128(W):
    """int4 with one absmax/7 scale per 128 values along K: ``precision.quantize(W.reshape(-1,128), "int4",
    axis=0)``.  Returns (packed uint8 [N, K/2], scale fp32 [N, K/128], scale fp16 [N, K/128])."""
    W = np.asarray(W)
    N, K = W.shape
    if K % 128:
        raise ValueError("K must be a multiple of 128")
    codes, s = quant_segments(W.reshape(-1, 128), 7)
    return pack4(codes).reshape(N, K // 2), s.reshape(N, K // 128), s.reshape(N, K // 128).astype(np.float16)


def dequant_int8_rows(codes, scale16):
    return np.asarray(codes, np.int8).astype(np.float32) * np.asarray(scale16, np.float32)[:, None]


def dequant_int4_g128(packed, scale16):
    """float32(code) * float32(fp16 scale), precision.py:264-268 with the stored fp16 scale."""
    packed = np.asarray(packed, np.uint8)
    N, KB = packed.shape
    K = KB * 2
    c = unpack4(packed, N * K).reshape(N, K // 128, 128).astype(np.float32)
    return (c * np.asarray(scale16, np.float32)[:, :, None]).reshape(N, K)


def linear_ref(x, Wd, bias=None, y0=None):
    """The exact product the kernels approximate: float64 x[M,K] @ Wd[N,K]^T (+ bias) (+ y0)."""
    y = np.asarray(x, np.float64) @ np.asarray(Wd, np.float64).T
    if bias is not None:
        y = y + np.asarray(bias, np.float64)[None, :]
    if y0 is not None:
        y = y + np.asarray(y0, np.float64)
    return y


def rms_norm(x, w, eps=1e-6, off=0.0):
    """RMSNorm of rows in float32, as the reference's host rms op computes it (apsi/hub_gpu.py:1690-1693):
    x / sqrt(mean(x * x) + eps) * (w + off)."""
    x = np.asarray(x, np.float32)
    w = np.asarray(w, np.float32)
    return (x / np.sqrt((x * x).mean(-1, keepdims=True) + np.float32(eps)) * (w + np.float32(off))).astype(np.float32)


def qkv_prep(qkv, cos, sin, qn, kn, nh, kvh, dh, rot, start, eps):
    """The reference host qkv_prep (apsi/hub_gpu.py:1701-1723) for one sequence: qkv [T, (nh + 2 kvh) dh]
    float32, cos / sin [positions, rot / 2] -> q [T, nh, dh], k [T, kvh, dh], v [T, kvh, dh] (float32)."""
    qkv = np.asarray(qkv, np.float32)
    T = qkv.shape[0]
    x = qkv.reshape(T, nh + 2 * kvh, dh)
    half = rot // 2
    c = np.asarray(cos, np.float32)[start:start + T].reshape(T, 1, half)
    s = np.asarray(sin, np.float32)[start:start + T].reshape(T, 1, half)

    def prep(v, w):
        if w is not None:
            v = v / np.sqrt((v * v).mean(-1, keepdims=True) + np.float32(eps)) * np.asarray(w, np.float32)[:dh]
        r1, r2, rest = v[..., :half], v[..., half:rot], v[..., rot:]
        return np.concatenate([r1 * c - r2 * s, r2 * c + r1 * s, rest], -1)
    return prep(x[:, :nh], qn), prep(x[:, nh:nh + kvh], kn), x[:, nh + kvh:]


def act_mul(gu, I, kind):
    """The reference host act_mul (apsi/hub_gpu.py:1755-1762): silu(g) * u (kind 0) or tanh-gelu(g) * u."""
    gu = np.asarray(gu, np.float32)
    g, u = gu[:, :I], gu[:, I:]
    if kind == 0:
        a = g / (1 + np.exp(-g))
    else:
        a = 0.5 * g * (1 + np.tanh(math.sqrt(2 / math.pi) * (g + 0.044715 * g ** 3)))
    return (a * u).astype(np.float32)


def qmatmul_dequant_reference(x, packed_or_codes, scale16, fmt):
    """The reference CPU path for a quantized product (precision.qmatmul: dequantise, then a float32
    matmul, precision.py:294-299).  This is what ``bench.py --impl reference`` times."""
    if fmt == "int4_g128":
        Wd = dequant_int4_g128(packed_or_codes, scale16)
    else:
        Wd = dequant_int8_rows(packed_or_codes, scale16)
    return np.asarray(x, np.float32) @ Wd.T


# ------------------------------------------------------------------------------------------- ggml-style g32
def qnumpy_g32(w, kind):
    """hub_gpu.qnumpy for "int8" / "int4" (hub_gpu.py:1215-1241): float32 arithmetic throughout.

    int8: scale = max|v| / 127; int4: scale = (value of largest magnitude, first one) / -8; inv = 1/scale
    (0 when the scale is 0); q = clip(rint(float32(v * inv)), lo, hi).  Returns (q float32 [O, I],
    scale float32 [O, I/32])."""
    w = np.asarray(w, np.float32)
    O, I = w.shape
    blk = w.reshape(O, I // 32, 32)
    a = np.abs(blk)
    if kind == "int8":
        sc = (a.max(axis=2) / np.float32(127.0)).astype(np.float32)
        lo, hi = -127, 127
    elif kind == "int4":
        first = a.argmax(axis=2)
        mval = np.take_along_axis(blk, first[:, :, None], 2)[:, :, 0]
        sc = (mval / np.float32(-8.0)).astype(np.float32)
        lo, hi = -8, 7
    else:
        raise ValueError(kind)
    safe = np.where(sc != 0, sc, np.float32(1))
    inv = np.where(sc != 0, (np.float32(1.0) / safe).astype(np.float32), np.float32(0)).astype(np.float32)
    prod = (blk * inv[:, :, None]).astype(np.float32)
    q = np.clip(np.rint(prod), lo, hi)
    return q.reshape(O, I).astype(np.float32), sc


def pack_q4_0_words(q):
    """int4 g32 values (float, -8..7) -> uint32 words [O, I/8], nibble j of word w = q[8w + j] + 8
    (hub_gpu.py:796-800)."""
    v = (np.asarray(q, np.int32) + 8).astype(np.uint32) & np.uint32(0xF)
    O, I = v.shape
    v = v.reshape(O, I // 8, 8)
    words = np.zeros((O, I // 8), np.uint32)
    for j in range(8):
        words |= v[:, :, j] << np.uint32(4 * j)
    return words


def pack_q8_0_words(q):
    """int8 g32 values -> uint32 words [O, I/4], byte j of word w = q[4w + j] (two's complement)."""
    v = np.asarray(q, np.int32).astype(np.int8).view(np.uint8).astype(np.uint32)
    O, I = v.shape
    v = v.reshape(O, I // 4, 4)
    words = np.zeros((O, I // 4), np.uint32)
    for j in range(4):
        words |= v[:, :, j] << np.uint32(8 * j)
    return words


def dequant_g32(q, sc):
    """hub_gpu.Emulator._dense (hub_gpu.py:1654-1658): values times the block scale, float32."""
    O, I = q.shape
    return (np.asarray(q, np.float32).reshape(O, I // 32, 32) * np.asarray(sc, np.float32)[:, :, None]) \
        .reshape(O, I).astype(np.float32)


# ------------------------------------------------------------------------------------------- minifloats
# (exp_bits, man_bits, bias, finite_only, nan_top) of the reference's minifloat formats, apsi/precision.py:70-76
MINIFLOATS = {
    "fp8_e4m3": (4, 3, 7, True, True),
    "fp8_e5m2": (5, 2, 15, False, False),
    "fp6_e3m2": (3, 2, 3, True, False),
    "fp6_e2m3": (2, 3, 1, True, False),
    "fp4_e2m1": (2, 1, 1, True, False),
}


def minifloat_table(name):
    """Value of every magnitude code (apsi/precision.py:23-39): subnormals at exponent field 0, inf / NaN in
    the top exponent unless the format is finite-only, the all-ones code NaN when ``nan_top``."""
    eb, mb, bias, finite_only, nan_top = MINIFLOATS[name]
    top = (1 << eb) - 1
    out = []
    for code in range(1 << (eb + mb)):
        e, m = code >> mb, code & ((1 << mb) - 1)
        v = math.ldexp(m, 1 - bias - mb) if e == 0 else math.ldexp((1 << mb) + m, e - bias - mb)
        if not finite_only and e == top:
            v = math.inf if m == 0 else math.nan
        if nan_top and e == top and m == (1 << mb) - 1:
            v = math.nan
        out.append(v)
    return np.array(out)


def minifloat_max(name):
    t = minifloat_table(name)
    return float(np.max(t[np.isfinite(t)]))


def minifloat_encode(name, y):
    """Codes of float64 values on the format's grid (apsi/precision.py:109-130): round to nearest with ties to the
    even code (the even mantissa), magnitudes above the largest finite value saturate, the sign bit follows
    signbit (so -0.0 keeps it), NaN takes the format's first NaN code, or the all-ones magnitude when the
    format has no NaN.  Restated with exponent arithmetic: the quotient by the ulp of the value's binade
    (the subnormal ulp below the smallest normal) is rounded half-to-even."""
    eb, mb, bias, _, _ = MINIFLOATS[name]
    y = np.asarray(y, np.float64)
    sign = np.signbit(y)
    a = np.minimum(np.abs(y), minifloat_max(name))
    nan = np.isnan(y)
    a = np.where(nan, 0.0, a)
    _, ex = np.frexp(a)
    e = np.where(a > 0, np.maximum(ex - 1, 1 - bias), 1 - bias)   # binade exponent; the smallest normal one for
                                                                  # subnormals and zero
    r = np.rint(np.ldexp(a, -(e - mb)))                  # exact power-of-two scaling, round half to even
    code = ((e + bias).astype(np.int64) << mb) + r.astype(np.int64) - (1 << mb)
    code = code | (sign.astype(np.int64) << (eb + mb))
    if nan.any():
        t = minifloat_table(name)
        nan_code = int(np.argmax(np.isnan(t))) if np.isnan(t).any() else (1 << (eb + mb)) - 1
        code = np.where(nan, nan_code, code)
    return code.astype(np.uint8)


def minifloat_decode(name, codes):
    """float32 values of codes (apsi/precision.py:133-138)."""
    eb, mb = MINIFLOATS[name][:2]
    codes = np.asarray(codes).astype(np.int64)
    mag = minifloat_table(name)[codes & ((1 << (eb + mb)) - 1)]
    return (mag * np.where((codes >> (eb + mb)) & 1, -1.0, 1.0)).astype(np.float32)


def pack6(codes):
    """Four 6-bit codes per three bytes, little-endian 24-bit words, zero-padded (apsi/precision.py:182-192)."""
    flat = np.asarray(codes).reshape(-1).astype(np.uint32) & 0x3F
    flat = np.concatenate([flat, np.zeros((-flat.size) % 4, np.uint32)])
    g = flat.reshape(-1, 4)
    word = g[:, 0] | (g[:, 1] << 6) | (g[:, 2] << 12) | (g[:, 3] << 18)
    return np.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], axis=1).astype(np.uint8).reshape(-1)


def unpack6(packed, n):
    b = np.asarray(packed, np.uint8).reshape(-1, 3).astype(np.uint32)
    word = b[:, 0] | (b[:, 1] << 8) | (b[:, 2] << 16)
    return np.stack([(word >> (6 * k)) & 0x3F for k in range(4)], axis=1).astype(np.uint8).reshape(-1)[:n]


def quant_minifloat(x, name, axis):
    """``precision.quantize(x, name, axis=axis)`` for a minifloat format (apsi/precision.py:205-246).

    axis=0 on a 2-D array: one float32 scale per row, ``max|row| / fmt.max`` (1.0 when the maximum is zero or
    NaN); axis=None: one float64 scale for the tensor.  Codes of ``x64 / scale`` flat in row-major order,
    packed for the 4- and 6-bit formats.  Returns (codes, scale)."""
    xv = np.asarray(x, np.float64)
    fmax = minifloat_max(name)
    with np.errstate(invalid="ignore", divide="ignore"):
        return _quant_minifloat(xv, name, axis, fmax)


def _quant_minifloat(xv, name, axis, fmax):
    if axis is None:
        m = float(np.max(np.abs(xv))) if xv.size else 0.0
        s = m / fmax if m > 0 else 1.0
        y = xv / s
    else:
        m = np.max(np.abs(xv), axis=1, keepdims=True)
        s = np.where(m > 0, m / fmax, 1.0).astype(np.float32)
        y = xv / s
    codes = minifloat_encode(name, y).reshape(-1)
    bits = {"fp8": 8, "fp6": 6, "fp4": 4}[name[:3]]
    if bits == 4:
        codes = pack4(codes)
    elif bits == 6:
        codes = pack6(codes)
    return codes, s


def dequant_minifloat(codes, name, shape, scale):
    """``precision.dequantize`` of a minifloat QTensor: ``decode(code) * float32(scale)`` (precision.py:249-274)."""
    n = int(np.prod(shape))
    bits = {"fp8": 8, "fp6": 6, "fp4": 4}[name[:3]]
    c = np.asarray(codes, np.uint8).reshape(-1)
    if bits == 4:
        c = unpack4(c, n)
    elif bits == 6:
        c = unpack6(c, n)
    v = minifloat_decode(name, c[:n]).reshape(shape)
    with np.errstate(invalid="ignore"):
        return (v * np.asarray(scale, np.float32)).astype(np.float32)


# ------------------------------------------------------------------------------------------- GGUF Q8_0 / Q4_0
def gguf_q8_0(a):
    """ggml Q8_0 blocks of 32 (apsi/modelio.py:56-67): binary16 d = amax / 127 (float32 arithmetic), then the 32
    int8 codes sign(y) * floor(|y| + 0.5) of y = x * (1 / d) (0 when d == 0), all in float32."""
    x = np.asarray(a, np.float32).reshape(-1, 32)
    d = (np.max(np.abs(x), axis=1) / np.float32(127.0)).astype(np.float32)
    inv = np.zeros_like(d)
    np.divide(np.float32(1.0), d, out=inv, where=d != 0)
    y = x * inv[:, None]
    q = (np.sign(y) * np.floor(np.abs(y) + np.float32(0.5))).astype(np.int8)
    return np.concatenate([d.astype(np.float16).view(np.uint8).reshape(-1, 2), q.view(np.uint8)], axis=1).reshape(-1)


def gguf_q4_0(a):
    """ggml Q4_0 blocks of 32 (apsi/modelio.py:70-81): d = x[argmax|x|] / -8 (the first largest magnitude, signed),
    codes min(15, trunc(x * (1 / d) + 8.5)) in float32, value j in the low nibble of byte j, value j + 16 in its
    high nibble."""
    x = np.asarray(a, np.float32).reshape(-1, 32)
    mx = x[np.arange(x.shape[0]), np.argmax(np.abs(x), axis=1)]
    d = (mx / np.float32(-8.0)).astype(np.float32)
    inv = np.zeros_like(d)
    np.divide(np.float32(1.0), d, out=inv, where=d != 0)
    q = np.minimum(15, (x * inv[:, None] + np.float32(8.5)).astype(np.int8)).astype(np.uint8)
    body = q[:, :16] | (q[:, 16:] << 4)
    return np.concatenate([d.astype(np.float16).view(np.uint8).reshape(-1, 2), body], axis=1).reshape(-1)


def gguf_dequant(buf, kind, n):
    """float32 values of Q8_0 / Q4_0 blocks (apsi/modelio.py:84-95)."""
    b = np.asarray(buf, np.uint8).reshape(-1, 34 if kind == "q8_0" else 18)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    if kind == "q8_0":
        v = b[:, 2:].view(np.int8).astype(np.float32)
    else:
        v = np.concatenate([(b[:, 2:] & 0x0F).astype(np.int8) - 8, (b[:, 2:] >> 4).astype(np.int8) - 8],
                           axis=1).astype(np.float32)
    return (v * d).reshape(-1)[:n]


# ------------------------------------------------------------------------------------------- error metrics
def round_weights_g32(a, kind):
    """apsi/lowbit.py:37-50 (``round_weights``) for "int8" / "int4": a [..., in, out] weight read as rows
    [out, in*...], each row padded with zeros to a multiple of 32, rounded with qnumpy_g32, multiplied back by
    the block scale (float32), the padding dropped and the result returned in a's shape and dtype."""
    a = np.asarray(a)
    if a.ndim < 2 or a.dtype.kind != "f":
        return a
    n_in, n_out = int(np.prod(a.shape[:-1])), int(a.shape[-1])
    rows = np.asarray(a, np.float32).reshape(n_in, n_out).T
    pad = (-n_in) % 32
    if pad:
        rows = np.concatenate([rows, np.zeros((n_out, pad), np.float32)], axis=1)
    q, sc = qnumpy_g32(rows, kind)
    d = dequant_g32(q, sc)[:, :n_in]
    return d.T.reshape(a.shape).astype(a.dtype)


def rel_frobenius(y, ref):
    ref = np.asarray(ref, np.float64)
    d = np.asarray(y, np.float64) - ref
    den = np.linalg.norm(ref)
    return float(np.linalg.norm(d) / den) if den > 0 else float(np.linalg.norm(d))


def max_abs_ratio(y, ref):
    ref = np.asarray(ref, np.float64)
    den = float(np.abs(ref).max()) if ref.size else 0.0
    d = float(np.abs(np.asarray(y, np.float64) - ref).max()) if ref.size else 0.0
    return d / den if den > 0 else d


# ------------------------------------------------------------------------------------------- seeded inputs
def make_config_inputs(M, N, K, seed=0, wstd=0.02, outliers=0.0):
    """Seeded synthetic inputs of the benchmark configurations: x ~ N(0,1) (optionally a fraction of entries
    multiplied by 20), cast to bfloat16; W ~ N(0, wstd) float32 [N, K]."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K)).astype(np.float32)
    if outliers:
        hit = rng.random((M, K)) < outliers
        x[hit] *= 20.0
    W = (rng.standard_normal((N, K)) * wstd).astype(np.float32)
    return bf16_round(x), W
