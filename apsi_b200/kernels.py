"""Torch-level wrappers of the C ABI: device tensors in, device tensors out, on the current CUDA stream.

Torch supplies device memory and streams only; every computation is one of the library's sm_100a kernels.
Inputs that are not CUDA tensors are rejected (there is no CPU path here).
"""
import ctypes
import threading

import torch

from . import _lib
from ._lib import FMT_INT8_ROW, FMT_INT4_G128, FMT_Q8_0_G32, FMT_Q4_0_G32, DT_F32, DT_BF16, LowbitError

__all__ = ["quant_int8_rows", "quant_int4_g128", "quant_q8_0_g32", "quant_q4_0_g32", "round_g32", "dequant", "linear",
           "linear_workspace_bytes", "interleave_cols", "device_errors", "FMT_INT8_ROW", "FMT_INT4_G128",
           "FMT_Q8_0_G32", "FMT_Q4_0_G32", "LowbitError", "minifloat_bytes", "quant_minifloat", "dequant_minifloat",
           "gguf_encode", "gguf_decode", "linear_spec",
           "prepare_weight", "PreparedWeight"]


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need_cuda(t, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise LowbitError(_lib.LB_E_DEVICE, f"{name} must be a CUDA tensor (the B200 path has no CPU fallback)")
    if not t.is_contiguous():
        raise LowbitError(_lib.LB_E_ARG, f"{name} must be contiguous")


def _weight_dtype(w):
    if w.dtype == torch.float32:
        return DT_F32
    if w.dtype == torch.bfloat16:
        return DT_BF16
    raise LowbitError(_lib.LB_E_ARG, f"weights must be float32 or bfloat16, got {w.dtype}")


# ------------------------------------------------------------------------------------------------ quantise
def quant_int8_rows(w, want_scale32=True):
    """int8 codes [N, K], fp16 scales [N] (and the reference's fp32 scales [N]) of a [N, K] weight."""
    _need_cuda(w, "w")
    N, K = w.shape
    codes = torch.empty((N, K), dtype=torch.int8, device=w.device)
    s16 = torch.empty((N,), dtype=torch.float16, device=w.device)
    s32 = torch.empty((N,), dtype=torch.float32, device=w.device) if want_scale32 else None
    with torch.cuda.device(w.device):
        _lib.call("lb_quant_int8_rows", _ptr(w), _weight_dtype(w), N, K, _ptr(codes), _ptr(s16), _ptr(s32),
                  _stream(w.device))
    return codes, s16, s32


def quant_int4_g128(w, want_scale32=True):
    """Packed int4 [N, K/2] (uint8), fp16 scales [N, K/128] (and fp32 scales) of a [N, K] weight."""
    _need_cuda(w, "w")
    N, K = w.shape
    packed = torch.empty((N, K // 2), dtype=torch.uint8, device=w.device)
    s16 = torch.empty((N, K // 128), dtype=torch.float16, device=w.device)
    s32 = torch.empty((N, K // 128), dtype=torch.float32, device=w.device) if want_scale32 else None
    with torch.cuda.device(w.device):
        _lib.call("lb_quant_int4_g128", _ptr(w), _weight_dtype(w), N, K, _ptr(packed), _ptr(s16), _ptr(s32),
                  _stream(w.device))
    return packed, s16, s32


def quant_q8_0_g32(w):
    """hub_gpu-layout int8 words [N, K/4] (int32 storage of uint32 words) and fp32 scales [N, K/32]."""
    _need_cuda(w, "w")
    N, K = w.shape
    words = torch.empty((N, K // 4), dtype=torch.int32, device=w.device)
    s32 = torch.empty((N, K // 32), dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        _lib.call("lb_quant_q8_0_g32", _ptr(w), _weight_dtype(w), N, K, _ptr(words), _ptr(s32), _stream(w.device))
    return words, s32


def quant_q4_0_g32(w):
    """hub_gpu-layout int4 words [N, K/8] (nibble = q + 8) and fp32 scales [N, K/32]."""
    _need_cuda(w, "w")
    N, K = w.shape
    words = torch.empty((N, K // 8), dtype=torch.int32, device=w.device)
    s32 = torch.empty((N, K // 32), dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        _lib.call("lb_quant_q4_0_g32", _ptr(w), _weight_dtype(w), N, K, _ptr(words), _ptr(s32), _stream(w.device))
    return words, s32


def round_g32(w, fmt):
    """lowbit.round_weights on rows: [N, K] float32 values clip(rint(w * inv)) * scale per block of 32 along K
    (fmt FMT_Q8_0_G32 or FMT_Q4_0_G32), signed zeros as the reference's float arithmetic gives them."""
    _need_cuda(w, "w")
    N, K = w.shape
    out = torch.empty((N, K), dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        _lib.call("lb_round_g32", fmt, _ptr(w), _weight_dtype(w), N, K, _ptr(out), _stream(w.device))
    return out


# ------------------------------------------------------------------------------------------------ minifloats
def minifloat_bytes(fmt, n):
    """Bytes of the packed codes of n values in minifloat format ``fmt`` (FMT_FP8_E4M3 .. FMT_FP4_E2M1)."""
    return int(_lib.load().lb_minifloat_bytes(fmt, n))


def quant_minifloat(w, fmt, per_row=True):
    """precision.quantize(w, <minifloat>, axis=0 if per_row else None) of a 2-D weight on the device.

    Returns (codes, scale): packed uint8 codes (flat row-major) and, per row, the float32 scales [R]; per tensor,
    a one-element float32 tensor holding max|w| (the tensor scale is max / fmt.max in float64)."""
    _need_cuda(w, "w")
    R, C = w.shape
    codes = torch.empty((minifloat_bytes(fmt, R * C),), dtype=torch.uint8, device=w.device)
    aux = torch.empty((R if per_row else 1,), dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        _lib.call("lb_quant_minifloat", fmt, _ptr(w), _weight_dtype(w), R, C, 1 if per_row else 0, _ptr(codes),
                  _ptr(aux) if per_row else ctypes.c_void_p(0), ctypes.c_void_p(0) if per_row else _ptr(aux),
                  _stream(w.device))
    return codes, aux


def dequant_minifloat(fmt, codes, R, C, scale, out_dtype=torch.float32):
    """value(code) * scale as [R, C]: ``scale`` a float32 CUDA tensor [R] (per row) or a Python float."""
    _need_cuda(codes, "codes")
    out = torch.empty((R, C), dtype=out_dtype, device=codes.device)
    per_row = isinstance(scale, torch.Tensor)
    if per_row:
        _need_cuda(scale, "scale")
    dt = DT_F32 if out_dtype == torch.float32 else DT_BF16
    with torch.cuda.device(codes.device):
        _lib.call("lb_dequant_minifloat", fmt, _ptr(codes), R, C, 1 if per_row else 0,
                  _ptr(scale) if per_row else ctypes.c_void_p(0), ctypes.c_float(0.0 if per_row else float(scale)),
                  _ptr(out), dt, _stream(codes.device))
    return out


# ------------------------------------------------------------------------------------------------ GGUF
def gguf_encode(x, kind):
    """GGUF Q8_0 (kind 8) or Q4_0 (kind 4) block bytes of a float32 CUDA tensor (size a multiple of 32)."""
    _need_cuda(x, "x")
    if x.dtype != torch.float32:
        raise LowbitError(_lib.LB_E_ARG, f"x must be float32, got {x.dtype}")
    n = x.numel()
    out = torch.empty(((n // 32) * (34 if kind == 8 else 18),), dtype=torch.uint8, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("lb_gguf_encode", kind, _ptr(x), n, _ptr(out), _stream(x.device))
    return out


def gguf_decode(blocks, kind, n):
    """float32 values [n] of GGUF Q8_0 / Q4_0 blocks (a uint8 CUDA tensor)."""
    _need_cuda(blocks, "blocks")
    out = torch.empty((n,), dtype=torch.float32, device=blocks.device)
    with torch.cuda.device(blocks.device):
        _lib.call("lb_gguf_decode", kind, _ptr(blocks), n, _ptr(out), _stream(blocks.device))
    return out


# ------------------------------------------------------------------------------------------------ dequantise
def dequant(fmt, codes, scales, N, K, out_dtype=torch.float32, scale_f32=None):
    """code * scale as [N, K] float32 (or bfloat16).  The scale dtype follows the tensor (float16 or float32)."""
    _need_cuda(codes, "codes")
    _need_cuda(scales, "scales")
    out = torch.empty((N, K), dtype=out_dtype, device=codes.device)
    dt = DT_F32 if out_dtype == torch.float32 else DT_BF16
    sdt = DT_F32 if scales.dtype == torch.float32 else _lib.DT_F16
    with torch.cuda.device(codes.device):
        _lib.call("lb_dequant", fmt, _ptr(codes), _ptr(scales), sdt, N, K, _ptr(out), dt, _stream(codes.device))
    return out


# ------------------------------------------------------------------------------------------------ products
_ws_lock = threading.Lock()
_ws = {}
_ws_retired = []   # outgrown workspaces stay allocated: a captured CUDA graph may still use their addresses


def linear_workspace_bytes(fmt, M, N, K):
    n = ctypes.c_size_t(0)
    _lib.call("lb_linear_workspace_size", fmt, M, N, K, ctypes.byref(n))
    return n.value


def _workspace(device, nbytes):
    """A per-device scratch buffer of at least nbytes (grown on demand, never shrunk).  A buffer that is
    outgrown is kept, not freed: a CUDA graph captured with it replays into its address, so that memory must
    not pass to another tensor.  The cost is at most the sum of the sizes on the way to the largest.

    There is ONE buffer per device, shared by every stream: two prefill products (M > 16) issued on different
    streams of one device at the same time race on it.  Serialise prefill calls per device (one stream, or
    events between the streams)."""
    if nbytes == 0:
        return None
    key = device.index if device.index is not None else torch.cuda.current_device()
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None:
                _ws_retired.append(buf)
            buf = torch.zeros(max(nbytes, 2 * (buf.numel() if buf is not None else 0), 1 << 20), dtype=torch.uint8,
                              device=device)
            _ws[key] = buf
        return buf


_fast = {}


def _fn(name):
    f = _fast.get(name)
    if f is None:
        f = _fast[name] = getattr(_lib.load(), name)
    return f


def _code_bytes(fmt, N, K):
    """(bytes of the codes, bytes of the scales) lb_linear reads for a [N, K] weight in format ``fmt``."""
    if fmt == FMT_INT4_G128:
        return N * K // 2, N * (K // 128) * 2
    if fmt == FMT_INT8_ROW:
        return N * K, N * 2
    if fmt in (_lib.FMT_FP8_E4M3, _lib.FMT_FP8_E5M2):
        return N * K, N * 4
    if fmt == _lib.FMT_FP4_E2M1:
        return N * K // 2, N * 4
    if fmt in (_lib.FMT_FP6_E3M2, _lib.FMT_FP6_E2M3):
        return N * K * 3 // 4, N * 4
    return 0, 0


def _check_product(fmt, x, M, K, codes, scales, N, bias, out):
    """The operand checks of a product, so that nothing the library is given lies outside its tensor: codes,
    scales and bias hold what the format needs for [N, K] on x's device, and out is a bfloat16 [>= M, >= N] view
    with unit column stride on that device.  Raises LowbitError(LB_E_ARG)."""
    dev = x.device
    cb, sb = _code_bytes(fmt, N, K)
    for t, name, need in ((codes, "codes", cb), (scales, "scales", sb)):
        if not isinstance(t, torch.Tensor) or t.device != dev:
            raise LowbitError(_lib.LB_E_ARG, f"{name} must be a CUDA tensor on {dev}")
        if t.numel() * t.element_size() < need:
            raise LowbitError(_lib.LB_E_ARG, f"{name} holds {t.numel() * t.element_size()} bytes, the format needs "
                                             f"{need} for N={N}, K={K}")
        if not t.is_contiguous():
            raise LowbitError(_lib.LB_E_ARG, f"{name} must be contiguous")
    if bias is not None:
        if (not isinstance(bias, torch.Tensor) or bias.device != dev or bias.dtype != torch.bfloat16
                or bias.numel() < N or not bias.is_contiguous()):
            raise LowbitError(_lib.LB_E_ARG, f"bias must be a contiguous bfloat16 tensor of {N} values on {dev}")
    if out.dtype != torch.bfloat16 or out.device != dev:
        raise LowbitError(_lib.LB_E_ARG, f"out must be a bfloat16 tensor on {dev}")
    if out.dim() == 0 or out.stride(-1) != 1 or out.shape[-1] < N:
        raise LowbitError(_lib.LB_E_ARG, f"out must have unit column stride and at least N={N} columns")
    rows = out.numel() // max(out.shape[-1], 1)
    if rows < M or (out.dim() > 2 and not out.is_contiguous()):
        raise LowbitError(_lib.LB_E_ARG, f"out must hold M={M} rows of a row-major [M, ldy] output")


def linear(fmt, x, codes, scales, N, bias=None, out=None, accumulate=False, static_weights=False):
    """y[M, N] = x[M, K] . deq(W)^T (+ bias) (+ out if accumulate), bf16 out, fp32 accumulation.

    ``static_weights``: no kernel still running on the current stream writes ``codes``/``scales`` (weights
    quantised before the previous launch); the GEMV then overlaps its weight stream with that kernel.
    This is the per-call hot path of the host layer, so it avoids anything but pointer and size lookups."""
    if not (isinstance(x, torch.Tensor) and x.is_cuda):
        _need_cuda(x, "x")
    if x.dtype != torch.bfloat16:
        raise LowbitError(_lib.LB_E_ARG, f"x must be bfloat16, got {x.dtype}")
    K = x.shape[-1]
    M = x.numel() // K
    if not x.is_contiguous():
        raise LowbitError(_lib.LB_E_ARG, "x must be contiguous")
    dev = x.device
    if out is None:
        if accumulate:
            raise LowbitError(_lib.LB_E_ARG, "accumulate needs an output tensor")
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _check_product(fmt, x, M, K, codes, scales, N, bias, out)
    ldy = out.stride(-2) if out.dim() >= 2 else N
    switch = dev.index != torch.cuda.current_device()
    if switch:
        prev = torch.cuda.current_device()
        torch.cuda.set_device(dev)
    try:
        nbytes = 0 if M <= 16 else linear_workspace_bytes(fmt, M, N, K)
        ws = _workspace(dev, nbytes) if nbytes else None
        rc = _fn("lb_linear_ex")(fmt, x.data_ptr(), M, K, codes.data_ptr(), scales.data_ptr(), N,
                                 bias.data_ptr() if bias is not None else None, 1 if accumulate else 0,
                                 out.data_ptr(), ldy, ws.data_ptr() if ws is not None else None, nbytes,
                                 _lib.LINEAR_STATIC_WEIGHTS if static_weights else 0,
                                 torch.cuda.current_stream(dev).cuda_stream)
    finally:
        if switch:
            torch.cuda.set_device(prev)
    if rc:
        _lib.check(rc)
    return out


try:                                                   # raw current stream / device of torch, without objects
    _raw_stream = torch._C._cuda_getCurrentRawStream
    _cur_dev = torch._C._cuda_getDevice
except AttributeError:                                 # pragma: no cover
    _raw_stream = None
    _cur_dev = None


class PreparedWeight:
    """An ``lb_weight`` handle: a weight checked once, with the tensor maps of its stream encoded once, for the
    per-call decode product (``lb_weight_linear``).  It holds the pointers of the codes and scales, not the
    tensors: the owner keeps them alive (a QTensor holds both).  Destroyed with the object."""
    __slots__ = ("ptr", "_destroy")

    def __init__(self, fmt, cptr, sptr, N, K, dev):
        self.ptr = None
        self._destroy = _fn("lb_weight_destroy")
        h = ctypes.c_void_p()
        with torch.cuda.device(dev):
            _lib.call("lb_weight_create", fmt, cptr, sptr, N, K, ctypes.byref(h))
        self.ptr = h.value

    def __del__(self):
        p, self.ptr = self.ptr, None
        if p:
            self._destroy(p)


def prepare_weight(fmt, cptr, sptr, N, K, dev):
    """A ``PreparedWeight``, or None when the weight has no decode product (the caller uses ``lb_linear_ex``)."""
    try:
        return PreparedWeight(fmt, cptr, sptr, N, K, dev)
    except _lib.LowbitError:
        return None


def linear_spec(spec, x, out=None, static_weights=False):
    """``linear`` for a weight described by ``spec`` = (fmt, codes pointer, scales pointer, N, K, device index,
    PreparedWeight or None) and a contiguous bfloat16 CUDA x [M, K] on the current device, in the fewest host
    operations: the per-call path of ``precision.qmatmul``.  ``static_weights`` as in ``linear``.  Returns None
    (the caller takes the general path) when x, out or the device do not fit it."""
    fmt, cptr, sptr, N, K, dev, pw = spec
    if _raw_stream is None or x.shape[1] != K or not x.is_contiguous() or x.get_device() != dev or _cur_dev() != dev:
        return None
    M = x.shape[0]
    if M > 16:
        return None                                     # the prefill path needs a workspace: general path
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    elif out.dim() != 2 or out.shape[0] != M or out.shape[1] != N or out.stride(1) != 1 or out.dtype != x.dtype:
        return None
    flags = _lib.LINEAR_STATIC_WEIGHTS if static_weights else 0
    if pw is not None:
        rc = _fn("lb_weight_linear")(pw.ptr, x.data_ptr(), M, out.data_ptr(), out.stride(0), flags, _raw_stream(dev))
    else:
        rc = _fn("lb_linear_ex")(fmt, x.data_ptr(), M, K, cptr, sptr, N, None, 0, out.data_ptr(), out.stride(0),
                                 None, 0, flags, _raw_stream(dev))
    if rc:
        _lib.check(rc)
    return out


def interleave_cols(src, G, M, Nl):
    """[G][M][Nl] rank-major shards -> [M][G*Nl]."""
    _need_cuda(src, "src")
    dst = torch.empty((M, G * Nl), dtype=src.dtype, device=src.device)
    with torch.cuda.device(src.device):
        _lib.call("lb_interleave_cols", _ptr(src), G, M, Nl, _ptr(dst), _stream(src.device))
    return dst


def device_errors(device=None):
    """Reads and clears the device error word (bit 1: a bounded in-kernel wait gave up)."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    v = ctypes.c_int(0)
    with torch.cuda.device(device):
        _lib.call("lb_device_errors", _stream(device), ctypes.byref(v))
    return v.value


# ----------------------------------------------------------------------------------------- multi-GPU
class _DevBuf:
    """A raw device allocation as torch sees it through the CUDA array interface (torch does not own it)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


def peer_alloc(nbytes, device):
    """A zeroed buffer other processes can map: (uint8 tensor view, device pointer, IPC handle bytes).

    The memory belongs to the library; release it with ``peer_free(ptr, device)`` once no rank uses it."""
    device = torch.device(device)
    p = ctypes.c_void_p()
    h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    with torch.cuda.device(device):
        _lib.call("lb_peer_alloc", int(nbytes), ctypes.byref(p), h)
        t = torch.as_tensor(_DevBuf(p.value, int(nbytes)), device=device)
    return t, p.value, h.raw


def peer_open(handle, device):
    """Device pointer of another rank's ``peer_alloc`` buffer, mapped into this process."""
    p = ctypes.c_void_p()
    with torch.cuda.device(torch.device(device)):
        _lib.call("lb_peer_open", handle, ctypes.byref(p))
    return p.value


def peer_close(ptr, device):
    with torch.cuda.device(torch.device(device)):
        _lib.call("lb_peer_close", ptr)


def peer_free(ptr, device):
    with torch.cuda.device(torch.device(device)):
        _lib.call("lb_peer_free", ptr)


def linear_sharded(fmt, x, codes, scales, n_local, y_ptrs, rank, ldy, bias=None, static_weights=False):
    """This rank's columns [rank * n_local, (rank + 1) * n_local) of x . deq(W)^T (+ bias), stored into every
    rank's [M, ldy] output (``y_ptrs``: one device pointer per rank, this rank's own included).  Follow with
    ``rank_barrier`` before reading an output."""
    if not (isinstance(x, torch.Tensor) and x.is_cuda):
        _need_cuda(x, "x")
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise LowbitError(_lib.LB_E_ARG, "x must be a contiguous bfloat16 tensor")
    K = x.shape[-1]
    M = x.numel() // K
    dev = x.device
    G = len(y_ptrs)
    arr = (ctypes.c_void_p * G)(*y_ptrs)
    with torch.cuda.device(dev):
        nbytes = 0 if M <= 16 else linear_workspace_bytes(fmt, M, n_local, K)
        ws = _workspace(dev, nbytes) if nbytes else None
        rc = _fn("lb_linear_sharded")(fmt, x.data_ptr(), M, K, codes.data_ptr(), scales.data_ptr(), n_local,
                                      bias.data_ptr() if bias is not None else None, arr, G, rank, ldy,
                                      ws.data_ptr() if ws is not None else None, nbytes,
                                      _lib.LINEAR_STATIC_WEIGHTS if static_weights else 0,
                                      torch.cuda.current_stream(dev).cuda_stream)
    if rc:
        _lib.check(rc)


def rank_barrier(flag_ptrs, rank, epoch, device, timeout_ms=0):
    """Cross-rank barrier on the current stream (see lb_rank_barrier); ``flag_ptrs``: every rank's flag array."""
    G = len(flag_ptrs)
    arr = (ctypes.c_void_p * G)(*flag_ptrs)
    device = torch.device(device)
    with torch.cuda.device(device):
        _lib.call("lb_rank_barrier", arr, G, rank, ctypes.c_uint32(epoch & 0xFFFFFFFF),
                  ctypes.c_uint32(timeout_ms), _stream(device))


def rmsnorm(x, w, eps=1e-6, off=0.0, out=None):
    """bf16(x * (1 / sqrt(mean(x^2) + eps)) * (w + off)) per row of bf16 x [.., K]; w float32 or bf16 [K]."""
    _need_cuda(x, "x")
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise LowbitError(_lib.LB_E_ARG, "x must be a contiguous bfloat16 tensor")
    K = x.shape[-1]
    M = x.numel() // K
    w = w.to(x.device)
    if w.dtype not in (torch.float32, torch.bfloat16):
        w = w.float()
    w = w.contiguous()
    if w.numel() < K:
        raise LowbitError(_lib.LB_E_ARG, f"w holds {w.numel()} values, K is {K}")
    if out is None:
        out = torch.empty_like(x)
    wdt = _lib.DT_F32 if w.dtype == torch.float32 else _lib.DT_BF16
    with torch.cuda.device(x.device):
        _lib.call("lb_rmsnorm", _ptr(x), M, K, _ptr(w), wdt, ctypes.c_float(eps), ctypes.c_float(off), _ptr(out),
                  _stream(x.device))
    return out


def linear_rms(fmt, x, ln, codes, scales, N, eps=1e-6, off=0.0, bias=None, out=None, accumulate=False,
               static_weights=False):
    """y[M, N] = rmsnorm(x; ln, eps, off) . deq(W)^T (+ bias) (+ out if accumulate): the bits of ``rmsnorm``
    followed by ``linear``.  For M <= 16 the norm runs inside the decode GEMV (one launch); above, the normalised
    rows go through a workspace.  ``ln``: float32 or bfloat16 [K] CUDA tensor."""
    _need_cuda(x, "x")
    if x.dtype != torch.bfloat16 or not x.is_contiguous():
        raise LowbitError(_lib.LB_E_ARG, "x must be a contiguous bfloat16 tensor")
    K = x.shape[-1]
    M = x.numel() // K
    dev = x.device
    if not (isinstance(ln, torch.Tensor) and ln.device == dev and ln.dtype in (torch.float32, torch.bfloat16)
            and ln.is_contiguous()):
        ln = ln.to(dev)
        ln = (ln if ln.dtype in (torch.float32, torch.bfloat16) else ln.float()).contiguous()
    if ln.numel() < K:
        raise LowbitError(_lib.LB_E_ARG, f"ln holds {ln.numel()} values, K is {K}")
    if out is None:
        if accumulate:
            raise LowbitError(_lib.LB_E_ARG, "accumulate needs an output tensor")
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _check_product(fmt, x, M, K, codes, scales, N, bias, out)
    ldy = out.stride(-2) if out.dim() >= 2 else N
    wdt = _lib.DT_F32 if ln.dtype == torch.float32 else _lib.DT_BF16
    with torch.cuda.device(dev):
        nbytes = 0
        if M > 16:
            n = ctypes.c_size_t(0)
            _lib.call("lb_linear_rms_workspace_size", fmt, M, N, K, ctypes.byref(n))
            nbytes = n.value
        ws = _workspace(dev, nbytes) if nbytes else None
        _lib.call("lb_linear_rms", fmt, _ptr(x), M, K, _ptr(ln), wdt, ctypes.c_float(eps), ctypes.c_float(off),
                  _ptr(codes), _ptr(scales), N, _ptr(bias) if bias is not None else None, 1 if accumulate else 0,
                  _ptr(out), ldy, _ptr(ws) if ws is not None else None, nbytes,
                  _lib.LINEAR_STATIC_WEIGHTS if static_weights else 0, _stream(dev))
    return out


def qkv_prep(qkv, B, T, nh, kvh, dh, rot, cos, sin, q_out, k_cache, v_cache, pos0=None, start=0, qn=None, kn=None,
             eps=1e-6):
    """Split / (optionally) RMSNorm / rotate the fused QKV projection; q_out [B, nh, T, dh]; k_cache, v_cache
    [B, kvh, cap, dh] written at positions pos0 + t (device int64 tensor) or start + t.  See lb_qkv_prep."""
    _need_cuda(qkv, "qkv")
    if qkv.dtype != torch.bfloat16 or not qkv.is_contiguous():
        raise LowbitError(_lib.LB_E_ARG, "qkv must be a contiguous bfloat16 tensor")
    for t, n in ((q_out, "q_out"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        if t.dtype != torch.bfloat16 or not t.is_contiguous():
            raise LowbitError(_lib.LB_E_ARG, f"{n} must be a contiguous bfloat16 tensor")
    cap = k_cache.shape[-2]
    with torch.cuda.device(qkv.device):
        _lib.call("lb_qkv_prep", _ptr(qkv), B, T, nh, kvh, dh, rot, _ptr(cos), _ptr(sin), _ptr(qn), _ptr(kn),
                  ctypes.c_float(eps), _ptr(pos0), int(start), _ptr(q_out), nh * T * dh, dh, T * dh,
                  _ptr(k_cache), _ptr(v_cache), kvh * cap * dh, cap * dh, _stream(qkv.device))


def act_mul(gu, I, kind=0, out=None):
    """act(g) * u of the fused [g | u] projection gu [M, 2 I] (bf16); kind 0 silu, 1 gelu (tanh form)."""
    _need_cuda(gu, "gu")
    if gu.dtype != torch.bfloat16 or not gu.is_contiguous():
        raise LowbitError(_lib.LB_E_ARG, "gu must be a contiguous bfloat16 tensor")
    M = gu.numel() // (2 * I)
    if out is None:
        out = torch.empty((M, I), dtype=torch.bfloat16, device=gu.device)
    with torch.cuda.device(gu.device):
        _lib.call("lb_act_mul", _ptr(gu), M, I, kind, _ptr(out), _stream(gu.device))
    return out
