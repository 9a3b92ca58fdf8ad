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
  runs the fused dequantise-and-matmul kernels.  A dense weight gives ``x @ w``, or, when ``_HW["on"]``, an fp8
  product on the library's fp8 kernels (w rounded to e4m3 per output column; backward in bfloat16).
  ``fp8_matmul_available`` answers the reference's question for this library.

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
# The dense-weight switch of the reference (apsi/lowbit.py:116): off unless a caller turns it on.  "why" stays
# for callers that read it; nothing here writes it (a failing fp8 product raises instead of switching off).
_HW = {"on": False, "why": None}


def fp8_matmul_available(dev):
    """Whether ``matmul`` can take dense weights through fp8 on this device (the reference's query,
    apsi/lowbit.py:119-131): a CUDA device of compute capability 10.x with this library loaded, unless the
    environment variable APSI_FP8_MATMUL is 0, false or no."""
    import os
    import torch
    if os.environ.get("APSI_FP8_MATMUL", "1").strip().lower() in ("0", "false", "no"):
        return False
    if getattr(dev, "type", None) != "cuda" or not torch.cuda.is_available():
        return False
    if torch.cuda.get_device_capability(dev)[0] != 10:
        return False
    from . import _lib
    try:
        _lib.load()
    except LowbitError:
        return False
    return True


_FP8 = {}


def _fp8_dense():
    """The autograd function of the dense fp8 product (built once, when torch is first needed).

    Forward: w [K, N] is rounded to fp8 e4m3 per output column (one float32 scale per column: the library's
    per-row minifloat quantiser on w^T) and multiplied with x in bfloat16 by the library's fused fp8 product
    (the codes become exact fp16 operands; float32 accumulation; bfloat16 out).  The reference instead rounds x
    and w to e4m3 with one scale each and calls cuBLASLt (apsi/lowbit.py:133-160); rounding only w, per column,
    keeps x exact and loses less.  Backward: in bfloat16 on the unrounded operands, as the reference's does:
    dx = g w^T, dw = x^T g."""
    if "fn" in _FP8:
        return _FP8["fn"]
    import torch
    from ._lib import FMT_FP8_E4M3

    class Fp8Dense(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x2, w):
            N = w.shape[1]
            codes, s32 = _k.quant_minifloat(w.detach().t().float().contiguous(), FMT_FP8_E4M3, per_row=True)
            y = _k.linear(FMT_FP8_E4M3, x2.detach().to(torch.bfloat16).contiguous(), codes, s32, N)
            ctx.save_for_backward(x2, w)
            return y

        @staticmethod
        def backward(ctx, g):
            x2, w = ctx.saved_tensors
            gb = g.to(torch.bfloat16)
            gx = gb @ w.to(torch.bfloat16).t()
            gw = x2.to(torch.bfloat16).t() @ gb
            return gx.to(x2.dtype), gw.to(w.dtype)

    _FP8["fn"] = Fp8Dense
    return Fp8Dense


def matmul(x, w):
    """x @ w.  A packed weight (precision.QTensor) runs the fused dequantise-and-matmul kernels.  A dense weight
    gives the ordinary product, or, when ``_HW["on"]`` and K is a multiple of 64, the fp8 product of
    ``_fp8_dense`` (bfloat16 out, with a gradient).  Errors of the fp8 path are raised, not hidden."""
    from . import precision
    if isinstance(w, precision.QTensor):
        return precision.qmatmul(x, w)
    if not _HW["on"] or not x.is_cuda or w.dim() != 2 or x.shape[-1] % 64:
        return x @ w
    K = x.shape[-1]
    y = _fp8_dense().apply(x.reshape(-1, K).contiguous(), w)
    return y.reshape(*x.shape[:-1], w.shape[1])
