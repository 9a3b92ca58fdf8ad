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
"""
import numpy as np

from . import kernels as _k
from . import precision as P
from .lowbit import parse_linear, tree_map

__all__ = ["qlinear", "quantize_model", "dequantize_model", "model_size"]

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
