"""A float32 device tensor with the surface of the reference's ``gpu_tensor`` for products, where ``@`` with a
quantised weight runs the fused low-bit kernels (apsi/gpu_tensor.py:229-263, ``GTensor.__matmul__``).

    a = gpu_tensor(x)                    # on cuda:0 (float32); gpu_tensor(x, "cpu") keeps an ordinary array
    y = a @ q + bias                     # q: a QTensor from quantize_linear / quantize(W, ..., axis=0)
    print(y.numpy())

The reference's ``GTensor`` multiplies dense float32 operands with its own GEMM and has no quantised product: a
QTensor right operand is not turned into a device array there.  Here a QTensor right operand goes to
``precision.qmatmul``: the activations are rounded to bfloat16 and multiplied by the codes on the decode GEMV
(M <= 16) or the tcgen05 GEMM, exactly as ``qmatmul`` does for a bfloat16 CUDA matrix, and the result comes back
as float32.  A 3-D ``[B, M, K]`` left operand is one product of ``B * M`` rows, as in the reference.  Dense
operands use torch's float32 matmul.  Element-wise ``+ - *`` with a tensor of the same shape, a row vector or a
number, and ``.T`` of a 2-D tensor, are kept on the device so ``a @ q + bias`` stays there.
"""
import numpy as np

from .precision import QTensor, qmatmul

__all__ = ["GTensor", "gpu_tensor"]


def _torch():
    import torch
    return torch


class GTensor:
    """A float32 tensor in a GPU's memory (a torch CUDA tensor), or with ``device="cpu"`` an ordinary array."""
    __array_priority__ = 1000

    def __init__(self, value, device):
        self.value = value              # torch.Tensor (float32, CUDA) or np.ndarray (float32) for "cpu"
        self.device = device

    # ------------------------------------------------------------ moving
    @staticmethod
    def of(x, device="cuda"):
        """``x`` (array, torch tensor, nested lists, number or GTensor) as a float32 tensor on ``device``."""
        if isinstance(x, GTensor):
            return x if x.device == str(device) else GTensor.of(x.numpy(), device)
        device = str(device)
        if device in ("cpu", "processor", "numpy"):
            if hasattr(x, "detach"):
                x = x.detach().float().cpu().numpy()
            return GTensor(np.ascontiguousarray(np.asarray(x, np.float32)), "cpu")
        if not (device == "cuda" or (device.startswith("cuda:") and device[5:].isdigit())):
            raise ValueError(f"unknown device {device!r}: 'cuda', 'cuda:<n>' or 'cpu'")
        torch = _torch()
        dev = torch.device("cuda", 0) if device == "cuda" else torch.device(device)
        t = x if isinstance(x, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(np.asarray(x, np.float32)))
        return GTensor(t.to(dev, torch.float32).contiguous(), device)

    def numpy(self):
        """The values as an ordinary float32 array."""
        if isinstance(self.value, np.ndarray):
            return self.value
        return self.value.detach().cpu().numpy()

    def __array__(self, dtype=None, copy=None):
        a = self.numpy()
        return a.astype(dtype) if dtype is not None else a

    def cpu(self):
        return self.numpy()

    def torch(self):
        """The underlying CUDA tensor (float32)."""
        if isinstance(self.value, np.ndarray):
            raise ValueError("a host GTensor has no device tensor")
        return self.value

    def __repr__(self):
        return f"gpu_tensor({list(self.shape)}, on {self.device})"

    @property
    def shape(self):
        return tuple(int(s) for s in self.value.shape)

    @property
    def ndim(self):
        return len(self.shape)

    @property
    def size(self):
        return int(np.prod(self.shape))

    @property
    def T(self):
        if self.ndim != 2:
            return GTensor(self.value.T if isinstance(self.value, np.ndarray) else self.value.permute(
                *range(self.ndim - 1, -1, -1)), self.device)
        return GTensor(self.value.T, self.device)

    def _wrap(self, v):
        return GTensor(v, self.device)

    # ------------------------------------------------------------ products
    def __matmul__(self, other):
        if isinstance(other, QTensor):
            # the fused low-bit kernels; the activations go in as bfloat16, the result comes back as float32
            if isinstance(self.value, np.ndarray):
                return GTensor(np.asarray(qmatmul(self.value, other), np.float32), self.device)
            torch = _torch()
            x = self.value.to(torch.bfloat16)
            if x.dim() == 2:
                x = x.contiguous()
            return self._wrap(qmatmul(x, other).float())
        y = other if isinstance(other, GTensor) else GTensor.of(other, self.device)
        if y.device != self.device:
            y = GTensor.of(y.numpy(), self.device)
        if self.ndim not in (2, 3) or y.ndim not in (2, 3) or (self.ndim == 2 and y.ndim == 3):
            raise ValueError(f"@: {list(self.shape)} @ {list(y.shape)}")
        if self.shape[-1] != y.shape[-2] or (y.ndim == 3 and y.shape[0] != self.shape[0]):
            raise ValueError(f"@: {list(self.shape)} @ {list(y.shape)}")
        return self._wrap(self.value @ y.value)

    def __rmatmul__(self, other):
        return GTensor.of(other, self.device) @ self

    # ------------------------------------------------------------ element-wise
    def _operand(self, other):
        if isinstance(other, GTensor):
            return other.value if other.device == self.device else GTensor.of(other.numpy(), self.device).value
        if np.ndim(other) == 0 and not hasattr(other, "detach"):
            return float(other)
        return GTensor.of(other, self.device).value

    def _binary(self, other, op, swap=False):
        o = self._operand(other)
        if not isinstance(o, float):
            if not (tuple(o.shape) == self.shape or (o.ndim == 1 and self.ndim >= 1 and o.shape[0] == self.shape[-1])):
                raise ValueError(f"{op}: shapes {list(self.shape)} and {list(o.shape)}")
        a, b = (o, self.value) if swap else (self.value, o)
        if op == "+":
            r = a + b
        elif op == "-":
            r = a - b
        else:
            r = a * b
        if isinstance(r, np.ndarray):
            r = r.astype(np.float32, copy=False)
        return self._wrap(r)

    def __add__(self, o):
        return self._binary(o, "+")

    def __radd__(self, o):
        return self._binary(o, "+", True)

    def __sub__(self, o):
        return self._binary(o, "-")

    def __rsub__(self, o):
        return self._binary(o, "-", True)

    def __mul__(self, o):
        return self._binary(o, "*")

    def __rmul__(self, o):
        return self._binary(o, "*", True)

    def __neg__(self):
        return self._wrap(-self.value)

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return self._wrap(self.value.reshape(shape))


def gpu_tensor(x, device="cuda"):
    """``x`` as a float32 tensor on the GPU (``device="cpu"``: an ordinary array with the same methods)."""
    return GTensor.of(x, device)
