"""The public entry points of ``apsi/lowbit.py`` on the B200 library.

Same names and argument meanings as the reference module (apsi/lowbit.py:15-181):

* ``KINDS``, ``ALIASES``, ``BLOCK``, ``parse`` -- unchanged.  Two names are added for the packed layer
  formats of the fused kernels: ``LINEAR_KINDS`` / ``parse_linear`` (``"int4_g128"``, ``"int8_row"`` and
  their aliases ``"w4g128"``, ``"int4g128"``, ``"w8"``).
* ``round_weights``, ``round_tree``, ``round_weights_torch``, ``fake_quant_torch``, ``fake_quant_tree_torch``
  -- the weights rounded as the format stores them (one scale per 32 values along the input side, the
  ``hub_gpu.qnumpy`` rounding).  The rounding runs in the library's one-pass g32 rounding kernel and gives the
  same bits as the reference, signed zeros included.  int8 and int4 are on the B200 path; the minifloat kinds (fp8, fp6,
  fp4) raise ``LowbitError``.
* ``matmul(x, w)`` -- the dispatch point.  A packed weight (``precision.QTensor`` from ``quantize_linear``)
  runs the fused dequantise-and-matmul kernels.  A dense weight keeps the reference behaviour: ``x @ w``, or
  fp8 tensor cores through ``torch._scaled_mm`` when ``_HW["on"]``.  ``fp8_matmul_available`` is unchanged.

Every rounding runs on the GPU: NumPy arrays are copied to the current CUDA device and back.  Without a GPU or
the library these calls raise; there is no CPU fallback.
"""
import numpy as np

from . import kernels as _k
from ._lib import LowbitError, LB_E_UNSUPPORTED, LB_E_ARG, FMT_Q8_0_G32, FMT_Q4_0_G32

__all__ = ["KINDS", "ALIASES", "BLOCK", "parse", "LINEAR_KINDS", "LINEAR_ALIASES", "parse_linear", "round_weights",
           "round_tree", "round_weights_torch", "fake_quant_torch", "fake_quant_tree_torch", "fp8_matmul_available",
           "matmul", "tree_map"]

KINDS = ("fp8", "fp6", "fp6_e2m3", "fp4", "int8", "int4")
ALIASES = {"mxfp8": "fp8", "e4m3": "fp8", "fp8_e4m3": "fp8", "mxfp6": "fp6_e2m3", "e2m3": "fp6_e2m3",
           "fp6_e3m2": "fp6", "e3m2": "fp6", "mxfp4": "fp4", "e2m1": "fp4", "fp4_e2m1": "fp4", "q8": "int8",
           "q4": "int4", "mxint8": "int8"}
BLOCK = 32

# packed formats of the fused layer kernels (no counterpart in the reference, which stores g32 only)
LINEAR_KINDS = ("int4_g128", "int8_row")
LINEAR_ALIASES = {"w4g128": "int4_g128", "int4g128": "int4_g128", "w8": "int8_row", "int8_rows": "int8_row"}

_G32_FMT = {"int8": FMT_Q8_0_G32, "int4": FMT_Q4_0_G32}


def parse(precision):
    """The low-bit format named by `precision`, or None for the ordinary precisions (fp32, bf16, ...)."""
    if not isinstance(precision, str):
        return None
    k = precision.strip().lower()
    k = ALIASES.get(k, k)
    return k if k in KINDS else None


def parse_linear(precision):
    """The packed layer format named by `precision` ("int4_g128" / "int8_row"), or None."""
    if not isinstance(precision, str):
        return None
    k = precision.strip().lower()
    k = LINEAR_ALIASES.get(k, k)
    return k if k in LINEAR_KINDS else None


def tree_map(f, *trees):
    """f over the leaves of nested lists / tuples / dicts (the containers of parameter trees)."""
    t0 = trees[0]
    if isinstance(t0, list):
        return [tree_map(f, *xs) for xs in zip(*trees)]
    if isinstance(t0, tuple):
        return tuple(tree_map(f, *xs) for xs in zip(*trees))
    if isinstance(t0, dict):
        return {k: tree_map(f, *(t[k] for t in trees)) for k in t0}
    return f(*trees)


def _as_rows(shape):
    """[..., in, out] weights as [out, in*...] rows (blocks run along the input side)."""
    return int(np.prod(shape[:-1])), int(shape[-1])


def _kernel_format(kind):
    k = parse(kind)
    if k is None:
        raise LowbitError(LB_E_ARG, f"unknown low-bit format '{kind}' (use one of {', '.join(KINDS)})")
    if k not in _G32_FMT:
        raise LowbitError(LB_E_UNSUPPORTED, f"format '{k}' (minifloat) is not on the B200 path; int8 and int4 are")
    return _G32_FMT[k]


# ------------------------------------------------------------------------------------------------ PyTorch
def round_weights_torch(w, kind):
    """The rounded weights (same dtype as w), computed without gradient on the GPU (apsi/lowbit.py:62-94)."""
    import torch
    fmt = _kernel_format(kind)
    if not (isinstance(w, torch.Tensor) and w.is_cuda):
        raise LowbitError(LB_E_ARG, "round_weights_torch takes CUDA tensors (the B200 path has no CPU fallback)")
    n_in, n_out = _as_rows(tuple(w.shape))
    rows = w.detach().float().reshape(n_in, n_out).t()
    pad = (-n_in) % BLOCK
    if pad:
        rows = torch.cat([rows, rows.new_zeros((n_out, pad))], dim=1)
    d = _k.round_g32(rows.contiguous(), fmt)[:, :n_in]
    return d.t().reshape(w.shape).to(w.dtype)


def fake_quant_torch(w, kind):
    """w in the format for the forward pass; the gradient goes straight through to the float32 master."""
    if w.dim() < 2 or not w.is_floating_point():
        return w
    return w + (round_weights_torch(w, kind) - w).detach()


def fake_quant_tree_torch(tp, kind):
    import torch
    return tree_map(lambda v: fake_quant_torch(v, kind) if isinstance(v, torch.Tensor) else v, tp)


# ------------------------------------------------------------------------------------------------ NumPy
def round_weights(a, kind):
    """A float array rounded as the format stores it (float32 values; 1-D arrays - biases, norms - unchanged).

    apsi/lowbit.py:37-50; the rounding runs on the GPU and the result comes back as a NumPy array."""
    import torch
    a = np.asarray(a)
    if a.ndim < 2 or a.dtype.kind != "f":
        return a
    _kernel_format(kind)
    if not torch.cuda.is_available():
        raise LowbitError(LB_E_ARG, "round_weights runs on the GPU and no CUDA device is visible")
    t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()
    r = round_weights_torch(t, kind).cpu().numpy()
    return r.astype(a.dtype)


def round_tree(params, kind):
    return tree_map(lambda v: round_weights(v, kind) if isinstance(v, np.ndarray) else v, params)


# ---------------------------------------------------------------------- products
_HW = {"on": False, "why": None}


def fp8_matmul_available(dev):
    """True when this GPU and PyTorch can multiply in fp8 on tensor cores (compute capability 8.9 and up)."""
    import os
    import torch
    if os.environ.get("APSI_FP8_MATMUL", "1").strip().lower() in ("0", "false", "no"):
        return False
    if dev.type != "cuda" or not hasattr(torch, "_scaled_mm") or not hasattr(torch, "float8_e4m3fn"):
        return False
    try:
        return tuple(torch.cuda.get_device_capability(dev)) >= (8, 9)
    except Exception:                                   # noqa: BLE001
        return False


def _fp8_product(x2, w):
    """x2 @ w with both in fp8 E4M3 (one scale each) on the tensor cores, bfloat16 out (dense weights only)."""
    import torch
    xs = (x2.detach().abs().amax().float() / 448.0).clamp(min=1e-12)
    ws = (w.detach().abs().amax().float() / 448.0).clamp(min=1e-12)
    a = (x2.float() / xs).to(torch.float8_e4m3fn)
    b = (w.float() / ws).to(torch.float8_e4m3fn).t().contiguous().t()
    y = torch._scaled_mm(a, b, scale_a=xs, scale_b=ws, out_dtype=torch.bfloat16)
    return y[0] if isinstance(y, tuple) else y


def matmul(x, w):
    """x @ w.  A packed weight (precision.QTensor) runs the fused dequantise-and-matmul kernels; a dense one
    the ordinary product, or fp8 tensor cores when that is switched on and the shapes allow it."""
    from . import precision
    if isinstance(w, precision.QTensor):
        return precision.qmatmul(x, w)
    if not _HW["on"] or not x.is_cuda or w.dim() != 2 or x.shape[-1] % 16 or w.shape[1] % 16:
        return x @ w
    import torch
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    pad = (-M) % 16
    if pad:
        x2 = torch.cat([x2, x2.new_zeros((pad, K))])
    try:
        y = _fp8_product(x2.contiguous(), w)
    except Exception as e:                              # noqa: BLE001 - never fail a run over the fp8 path
        _HW["on"], _HW["why"] = False, f"{type(e).__name__}: {e}"
        return x @ w
    return y[:M].reshape(*x.shape[:-1], w.shape[1])
