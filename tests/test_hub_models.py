"""The hub_gpu-style ops object (apsi_b200.hub) and the models entry points (apsi_b200.models).

CPU tests: names, runner() without a GPU, unsupported formats.  GPU tests: qmatrix codes bit-exact with the
oracle, linear / gemv / gemm / matmul and qlinear within the layer's tolerance of the oracle product, and the
RMSNorm prologue (linear(ln=...), rms) against the oracle's float32 RMSNorm."""
import numpy as np
import pytest

from apsi_b200 import hub, models, precision as P
from apsi_b200._lib import LowbitError
from oracle import lowbit_oracle as ora

TOL_REL_F, TOL_MAX_ABS = 2e-3, 1e-2


def _close(y, ref):
    return ora.rel_frobenius(y, ref) <= TOL_REL_F and ora.max_abs_ratio(y, ref) <= TOL_MAX_ABS


def test_runner_without_gpu_and_unknown_formats():
    import torch
    if not torch.cuda.is_available():
        ops, why = hub.runner("auto")
        assert ops is None and "CUDA" in why
    assert hub.runner("cpu") == (None, "device=cpu")
    with pytest.raises(LowbitError, match="no fused product"):
        hub._kind("fp4")
    assert hub._kind("w4g128") == ("int4", hub.FMT_INT4_G128)
    assert hub._kind("INT8") == ("int8", hub.FMT_INT8_ROW)


def test_dense_qlinear_keeps_the_reference_product():
    x = np.arange(6, dtype=np.float32).reshape(2, 3)
    W = np.ones((3, 4), np.float32)
    b = np.full(4, 0.5, np.float32)
    assert np.array_equal(models.qlinear(x, W, b), x @ W + b)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["int4", "int8"])
@pytest.mark.parametrize("T", [1, 5, 64])
def test_ops_qmatrix_and_linear(cuda, kind, T):
    rows, cols = 520, 1024
    x, W = ora.make_config_inputs(T, rows, cols, seed=31 + T)
    ops = hub.Ops(0)
    m = ops.qmatrix(W, kind)
    if kind == "int4":
        packed, _, s16 = ora.quant_int4_g128(W)
        assert np.array_equal(m.buf.cpu().numpy(), packed)
        Wd = ora.dequant_int4_g128(packed, s16)
    else:
        codes, _, s16 = ora.quant_int8_rows(W)
        assert np.array_equal(m.buf.cpu().numpy(), codes)
        Wd = ora.dequant_int8_rows(codes, s16)
    bias = np.random.default_rng(1).standard_normal(rows).astype(np.float32)
    X = ops.vec(x)
    Y = ops.alloc(T * rows)
    B = ops.vec(bias)
    ops.put(Y, np.zeros(T * rows, np.float32))
    ops.linear(m, X, Y, T, bias=B)
    y1 = ops.get(Y, T * rows).reshape(T, rows)
    ref_b = ora.linear_ref(x, Wd, ora.bf16_round(bias))
    assert _close(y1, ref_b)
    ops.linear(m, X, Y, T, acc=True)                       # Y += X @ W.T
    y2 = ops.get(Y, T * rows).reshape(T, rows)
    assert _close(y2, ora.linear_ref(x, Wd, None, y0=y1))
    assert _close(ops.matmul(x, m), ora.linear_ref(x, Wd))
    ops.close()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["int4", "w8"])
@pytest.mark.parametrize("M", [1, 40])
def test_qlinear_on_a_quantized_model(cuda, dtype, M):
    import torch
    K, N = 1024, 768
    x, W = ora.make_config_inputs(M, N, K, seed=7 + M)
    params = {"proj": {"W": W.T.copy(), "b": np.linspace(-1, 1, N).astype(np.float32)},
              "norm": np.ones(K, np.float32), "small": np.ones((4, 4), np.float32)}
    q = models.quantize_model(params, dtype)
    assert isinstance(q["proj"]["W"], P.QTensor) and q["small"] is params["small"] and q["norm"] is params["norm"]
    assert models.model_size(q) < models.model_size(params)
    y = models.qlinear(x, q["proj"]["W"], q["proj"]["b"])            # NumPy in, float32 out
    Wd = P.dequantize(q["proj"]["W"]).T                               # [N, K] as stored
    ref = ora.linear_ref(x, Wd, ora.bf16_round(params["proj"]["b"]))
    assert y.shape == (M, N) and _close(y, ref)
    xd = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    yd = models.qlinear(xd, q["proj"]["W"], torch.from_numpy(params["proj"]["b"]).to(cuda))
    assert yd.is_cuda and _close(yd.float().cpu().numpy(), ref)
    back = models.dequantize_model(q)
    assert back["proj"]["W"].shape == (K, N)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 3, 40])
def test_ops_linear_with_rmsnorm_prologue(cuda, T):
    """linear(ln=...) normalises each row first (hub_gpu.py:1305-1315): the result equals the product of the
    bf16-rounded RMSNorm (oracle, hub_gpu.py:1690-1693) within the layer's tolerance, and rms() alone is
    within one bf16 rounding of the float32 oracle."""
    rows, cols = 384, 1024
    x, W = ora.make_config_inputs(T, rows, cols, seed=5 + T)
    g = np.random.default_rng(3).standard_normal(cols).astype(np.float32) * 0.1 + 1.0
    ops = hub.Ops(0)
    m = ops.qmatrix(W, "int4")
    packed, _, s16 = ora.quant_int4_g128(W)
    Wd = ora.dequant_int4_g128(packed, s16)
    X, LN = ops.vec(x), ops.vec(g)
    Y = ops.alloc(T * rows)
    ops.linear(m, X, Y, T, ln=LN, eps=1e-5, off=0.0)
    xb = ora.bf16_round(x)
    xn = ora.bf16_round(ora.rms_norm(xb, g, eps=1e-5))                    # float32 norm weights (vec)
    assert _close(ops.get(Y, T * rows).reshape(T, rows), ora.linear_ref(xn, Wd))
    Z = ops.alloc(T * cols)
    ops.rms(X, Z, LN, T, cols, 1e-5, 0.5)
    z = ops.get(Z, T * cols).reshape(T, cols)
    ref = ora.rms_norm(xb, g, eps=1e-5, off=0.5)
    assert np.all(np.abs(z - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-30)
    ops.close()
