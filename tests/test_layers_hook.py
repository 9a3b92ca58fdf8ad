"""The reference's model code picks the library up unchanged (apsi/layers.py:251-253 ``Linear.apply``: ``x @ p.W``,
and the attention / SwiGLU blocks of ``transformer_lm``, apsi/layers.py:1999-2008, which multiply the same way).

tests/golden/layers_trace_golden.npz was written by the reference's own ``transformer_lm`` forward with every
projection weight replaced by an object that, like ``apsi_b200.precision.QTensor``, makes NumPy defer ``x @ W``
to it (``__array_ufunc__ = None``): it recorded every call's input and output (the int4-g128 dequantised weight
multiplied in float64) and the weights' packed codes and fp16 scales.  Here the same calls go through QTensors
holding those codes on the GPU, as the forward would make them."""
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "layers_trace_golden.npz")


def test_numpy_defers_matmul_to_a_qtensor():
    from apsi_b200 import precision as P
    assert P.QTensor.__array_ufunc__ is None

    class Probe(P.QTensor):
        def __rmatmul__(self, x):
            return ("deferred", np.shape(x))
    q = Probe(np.zeros(8, np.uint8), None, P.get_format("int4"), (128, 1), 0, None, True,
              scale16=np.zeros((1, 1), np.float16), group=128, kn=True)
    assert (np.ones((3, 128), np.float32) @ q) == ("deferred", (3, 128))


@pytest.mark.gpu
def test_transformer_lm_call_sites_run_on_the_kernels(cuda):
    import torch
    from apsi_b200 import precision as P, kernels
    g = np.load(GOLD)
    names = [str(n) for n in g["call_names"]]
    qs = {}
    for n in set(names):
        packed, s16 = g[f"w_{n}_packed"], g[f"w_{n}_s16"].view(np.float16)
        out_, in_ = s16.shape[0], packed.shape[1] * 2
        qs[n] = P.QTensor(torch.from_numpy(packed).to(cuda), None, P.get_format("int4"), (in_, out_), 0, None, True,
                          scale16=torch.from_numpy(s16).to(cuda), group=128, kn=True)
    for i, n in enumerate(names):
        x, y_ref = g[f"call{i}_x"], g[f"call{i}_y"]
        y = x @ qs[n]                                  # the expression the reference's layers evaluate
        assert isinstance(y, np.ndarray) and y.shape == y_ref.shape and y.dtype == np.float32
        # against the reference's own output (float64 activations there, bfloat16 into the kernel here)
        assert O.max_abs_ratio(y, y_ref) <= 1e-2 and O.rel_frobenius(y, y_ref) <= 4e-3, n
        # against the product of the activations as the kernel takes them: the layer's bar
        Wd = O.dequant_int4_g128(g[f"w_{n}_packed"], g[f"w_{n}_s16"].view(np.float16))
        ref = O.linear_ref(O.bf16_round(x.reshape(-1, x.shape[-1])), Wd).reshape(y_ref.shape)
        assert O.max_abs_ratio(y, ref) <= 1e-2 and O.rel_frobenius(y, ref) <= 2e-3, n
    assert kernels.device_errors(cuda) == 0
