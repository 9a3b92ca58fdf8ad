"""apsi_b200.lowbit: the reference's lowbit entry points.  CPU tests check names, aliases and the loud failures;
GPU tests check the rounding against the reference's own round_weights (golden vectors) bit for bit."""
import numpy as np
import pytest

from apsi_b200 import lowbit
from apsi_b200._lib import LowbitError
from oracle import lowbit_oracle as ora


def test_kinds_aliases_and_parse_keep_the_reference_names():
    assert lowbit.KINDS == ("fp8", "fp6", "fp6_e2m3", "fp4", "int8", "int4")
    assert lowbit.BLOCK == 32
    assert lowbit.parse("Q4") == "int4" and lowbit.parse("mxint8") == "int8" and lowbit.parse("e2m1") == "fp4"
    assert lowbit.parse("bf16") is None and lowbit.parse(None) is None
    assert lowbit.parse_linear("w4g128") == "int4_g128" and lowbit.parse_linear("W8") == "int8_row"
    assert lowbit.parse_linear("int4") is None


def test_tree_map_and_non_weights_pass_through():
    t = {"a": [1, (2, 3)], "b": {"c": 4}}
    assert lowbit.tree_map(lambda v: v * 10, t) == {"a": [10, (20, 30)], "b": {"c": 40}}
    bias = np.arange(5, dtype=np.float32)
    assert lowbit.round_weights(bias, "int4") is not None
    assert np.array_equal(lowbit.round_weights(bias, "int4"), bias)        # 1-D arrays unchanged


def test_unsupported_and_host_inputs_fail_loudly():
    import torch
    with pytest.raises(LowbitError, match="minifloat"):
        lowbit.round_weights(np.ones((64, 4), np.float32), "fp4")
    with pytest.raises(LowbitError, match="unknown"):
        lowbit.round_weights(np.ones((64, 4), np.float32), "int3")
    with pytest.raises(LowbitError, match="CUDA"):
        lowbit.round_weights_torch(torch.ones((64, 4)), "int8")


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["int8", "int4"])
def test_round_weights_bit_exact_with_reference_golden(cuda, golden, kind):
    import torch
    got = lowbit.round_weights(golden["rw_in"], kind)
    assert np.array_equal(got.view(np.uint32), golden[f"rw_{kind}"].view(np.uint32))
    t = torch.from_numpy(golden["rw_in"]).to(cuda)
    got_t = lowbit.round_weights_torch(t, kind).cpu().numpy()
    assert np.array_equal(got_t.view(np.uint32), golden[f"rw_{kind}"].view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("kind", ["int8", "int4"])
@pytest.mark.parametrize("shape", [(4096, 512), (3, 100, 64), (33, 7)])
def test_round_weights_torch_matches_oracle_random(cuda, kind, shape):
    import torch
    rng = np.random.default_rng(sum(shape))
    w = (rng.standard_normal(shape) * rng.choice([1e-3, 0.02, 3.0])).astype(np.float32)
    w.reshape(-1)[::97] = 0.0
    got = lowbit.round_weights_torch(torch.from_numpy(w).to(cuda), kind).cpu().numpy()
    ref = ora.round_weights_g32(w, kind)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.gpu
def test_fake_quant_forward_rounds_and_gradient_passes_straight_through(cuda):
    import torch
    w = (torch.randn((256, 96), device=cuda) * 0.02).requires_grad_(True)
    y = lowbit.fake_quant_torch(w, "int4")
    assert torch.equal(y.detach(), lowbit.round_weights_torch(w.detach(), "int4"))
    (y * 3.0).sum().backward()
    assert torch.equal(w.grad, torch.full_like(w, 3.0))
    tree = lowbit.fake_quant_tree_torch({"W": w, "b": torch.zeros(96, device=cuda)}, "int8")
    assert torch.equal(tree["b"], torch.zeros(96, device=cuda))


@pytest.mark.gpu
def test_matmul_dispatches_packed_weights_to_the_fused_kernels(cuda):
    import torch
    from apsi_b200 import precision as P
    K, N = 1024, 640
    x, W = ora.make_config_inputs(2, N, K, seed=21)
    qt = P.quantize_linear(torch.from_numpy(W.T.copy()).to(cuda), "int4")     # Apsi Linear stores [in, out]
    xd = torch.from_numpy(x).to(cuda).to(torch.bfloat16)
    y = lowbit.matmul(xd, qt)
    assert torch.equal(y, P.qmatmul(xd, qt))
    dense = torch.randn((K, 8), device=cuda)
    assert torch.equal(lowbit.matmul(xd.float(), dense), xd.float() @ dense)


@pytest.mark.gpu
def test_dense_fp8_matmul_rounds_w_per_column_and_has_a_gradient(cuda):
    """lowbit.matmul on a dense weight with the fp8 switch on: w rounded to e4m3 per output column (the oracle's
    per-row minifloat quantiser on w^T), x exact in bfloat16; the bfloat16 backward of the reference."""
    import torch
    assert lowbit.fp8_matmul_available(cuda)
    K, N, M = 512, 192, 5
    x, Wt = ora.make_config_inputs(M, N, K, seed=31)          # Wt: [N, K]
    codes, s = ora.quant_minifloat(Wt, "fp8_e4m3", axis=0)
    ref = ora.linear_ref(x, ora.dequant_minifloat(codes, "fp8_e4m3", Wt.shape, s))
    xd = torch.from_numpy(x).to(cuda).requires_grad_(True)
    w = torch.from_numpy(Wt.T.copy()).to(cuda).requires_grad_(True)
    old = lowbit._HW["on"]
    lowbit._HW["on"] = True
    try:
        y = lowbit.matmul(xd, w)
    finally:
        lowbit._HW["on"] = old
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    yn = y.detach().float().cpu().numpy()
    assert ora.rel_frobenius(yn, ref) <= 2e-3 and ora.max_abs_ratio(yn, ref) <= 1e-2
    g = torch.randn((M, N), device=cuda)
    y.backward(g)
    gb = g.to(torch.bfloat16)
    assert torch.equal(xd.grad, (gb @ w.detach().to(torch.bfloat16).t()).float())
    assert torch.equal(w.grad, (xd.detach().to(torch.bfloat16).t() @ gb).float())
    # off: the ordinary product
    assert torch.equal(lowbit.matmul(xd.detach(), w.detach()), xd.detach() @ w.detach())


def test_fp8_matmul_available_honours_the_switch(monkeypatch):
    import torch
    monkeypatch.setenv("APSI_FP8_MATMUL", "0")
    assert lowbit.fp8_matmul_available(torch.device("cuda", 0)) is False
    monkeypatch.setenv("APSI_FP8_MATMUL", "1")
    assert lowbit.fp8_matmul_available(torch.device("cpu")) is False
