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
"""
import math

import numpy as np

__all__ = [
    "bf16_round", "bf16_to_f32", "f32_to_bf16_bits", "scale_for_segments", "quant_segments", "pack4", "unpack4",
    "quant_int8_rows", "quant_int4_g128", "dequant_int8_rows", "dequant_int4_g128", "linear_ref",
    "qnumpy_g32", "pack_q4_0_words", "pack_q8_0_words", "dequant_g32", "rel_frobenius", "max_abs_ratio",
    "make_config_inputs", "qmatmul_dequant_reference", "round_weights_g32",
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
