"""apsi_b200.gpu_tensor: the reference's device tensor surface (apsi/gpu_tensor.py:229-263) with ``@`` on a
quantised weight routed to the fused kernels.  CPU tests cover the dense host path and the shape errors; GPU
tests check ``GTensor @ QTensor`` bit for bit against ``precision.qmatmul`` on the same bfloat16 activations and
against the oracle's float32 product with the kernel tolerances (max-abs <= 1e-2 * max|y|, relative Frobenius
<= 2e-3)."""
import numpy as np
import pytest

import oracle as O
from apsi_b200.gpu_tensor import GTensor, gpu_tensor


def test_host_tensor_products_and_arithmetic():
    rng = np.random.default_rng(3)
    a = rng.standard_normal((4, 6)).astype(np.float32)
    w = rng.standard_normal((6, 5)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    g = gpu_tensor(a, "cpu")
    assert g.shape == (4, 6) and g.ndim == 2 and g.size == 24 and g.device == "cpu"
    y = g @ w + b
    assert isinstance(y, GTensor)
    assert np.allclose(y.numpy(), a @ w + b, rtol=1e-6, atol=1e-6)
    assert np.allclose((2.0 - g).numpy(), 2.0 - a) and np.allclose((g * g).numpy(), a * a)
    assert np.allclose((-g).numpy(), -a) and g.T.shape == (6, 4)
    assert np.allclose((w.T @ g.T).numpy(), w.T @ a.T, rtol=1e-6, atol=1e-6)     # __rmatmul__
    x3 = rng.standard_normal((2, 3, 6)).astype(np.float32)
    assert np.allclose((gpu_tensor(x3, "cpu") @ w).numpy(), x3 @ w, rtol=1e-6, atol=1e-6)
    assert np.asarray(g).dtype == np.float32


def test_shape_errors():
    g = gpu_tensor(np.ones((4, 6), np.float32), "cpu")
    with pytest.raises(ValueError):
        g @ np.ones((5, 2), np.float32)
    with pytest.raises(ValueError):
        g + np.ones((3,), np.float32)
    with pytest.raises(ValueError):
        gpu_tensor(np.ones(3), "tpu")


def _weights(N, K, seed, kind):
    x, W = O.make_config_inputs(4, N, K, seed=seed)
    if kind == "int4":
        codes, _, s16 = O.quant_int4_g128(W)
        Wd = O.dequant_int4_g128(codes, s16)
    else:
        codes, _, s16 = O.quant_int8_rows(W)
        Wd = O.dequant_int8_rows(codes, s16)
    return W, Wd


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["int4", "int8"])
@pytest.mark.parametrize("lead", [(1,), (8,), (64,), (300,), (2, 5)])
def test_gtensor_at_qtensor_runs_the_fused_kernels(cuda, kind, lead):
    import torch
    from apsi_b200 import precision as P
    N, K = 520, 1024
    W, Wd = _weights(N, K, seed=17 + len(lead), kind=kind)
    # quantize_linear takes the Apsi Linear orientation W[in, out] and multiplies as x @ W
    q = P.quantize_linear(torch.from_numpy(np.ascontiguousarray(W.T)).to(cuda), kind)
    rng = np.random.default_rng(int(np.prod(lead)))
    x = O.bf16_round(rng.standard_normal(lead + (K,)).astype(np.float32))
    g = gpu_tensor(x)
    assert g.device == "cuda" and g.torch().dtype == torch.float32
    y = g @ q
    assert isinstance(y, GTensor) and y.shape == lead + (N,) and y.torch().dtype == torch.float32
    xb = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    same = P.qmatmul(xb if xb.dim() == 2 else xb, q).float()
    assert torch.equal(y.torch(), same)
    ref = O.linear_ref(x.reshape(-1, K), Wd).reshape(lead + (N,))
    got = y.numpy()
    assert O.max_abs_ratio(got, ref) <= 1e-2 and O.rel_frobenius(got, ref) <= 2e-3
    # a @ q + bias stays on the device
    bias = rng.standard_normal(N).astype(np.float32)
    z = g @ q + bias
    assert z.device == "cuda" and np.allclose(z.numpy(), got + bias, rtol=0, atol=1e-6 * (1 + np.abs(got).max()))


@pytest.mark.gpu
def test_host_gtensor_at_qtensor_copies_through_the_kernels(cuda):
    import torch
    from apsi_b200 import precision as P
    N, K = 300, 512
    W, Wd = _weights(N, K, seed=5, kind="int4")
    q = P.quantize_linear(torch.from_numpy(np.ascontiguousarray(W.T)).to(cuda), "int4")
    x = O.bf16_round(np.random.default_rng(9).standard_normal((3, K)).astype(np.float32))
    y = gpu_tensor(x, "cpu") @ q
    assert y.device == "cpu" and y.numpy().dtype == np.float32
    dev = (gpu_tensor(x) @ q).numpy()
    assert np.array_equal(y.numpy(), dev)
