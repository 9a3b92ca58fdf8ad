"""Minifloat formats on the GPU (fp8 e4m3 / e5m2, fp6 e3m2 / e2m3, fp4 e2m1): codes, scales and dequantised
values bit-exact with the reference's golden vectors (precision.quantize / dequantize) and with the oracle."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

NAMES = ("fp8_e4m3", "fp8_e5m2", "fp6_e3m2", "fp6_e2m3", "fp4_e2m1")


def _same_f32(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    na, nb = np.isnan(a), np.isnan(b)
    return a.shape == b.shape and np.array_equal(na, nb) and np.array_equal(a.view(np.uint32)[~na],
                                                                              b.view(np.uint32)[~nb])


@pytest.mark.parametrize("name", NAMES)
def test_rows_bit_exact_with_reference_golden(cuda, golden, name):
    """axis=0: ties to the even code, saturation, a NaN row (scale 1.0), an inf row, signed zeros."""
    from apsi_b200 import precision as P
    W = golden[f"mf_{name}_w"]
    q = P.quantize(W, name, axis=0)
    np.testing.assert_array_equal(np.asarray(q.codes).reshape(-1), golden[f"mf_{name}_codes"])
    np.testing.assert_array_equal(np.asarray(q.scale).reshape(-1), golden[f"mf_{name}_scale"])
    assert np.asarray(q.scale).shape == (W.shape[0], 1)
    assert _same_f32(P.dequantize(q), golden[f"mf_{name}_deq"])


@pytest.mark.parametrize("name", NAMES)
def test_tensor_scale_bit_exact_with_reference_golden(cuda, golden, name):
    """axis=None: one float64 scale; packing runs across rows of an odd-sized array."""
    from apsi_b200 import precision as P
    W = golden[f"mf_{name}_t_w"]
    q = P.quantize(W, name)
    np.testing.assert_array_equal(np.asarray(q.codes).reshape(-1), golden[f"mf_{name}_t_codes"])
    assert q.scale == float(golden[f"mf_{name}_t_scale"][0])
    assert _same_f32(P.dequantize(q), golden[f"mf_{name}_t_deq"])


@pytest.mark.parametrize("name", NAMES)
@pytest.mark.parametrize("shape,std", [((257, 1000), 0.02), ((64, 4096), 1.5), ((3, 7), 100.0)])
def test_random_matches_oracle(cuda, name, shape, std):
    import torch
    from apsi_b200 import kernels as K
    from apsi_b200._lib import MINIFLOAT_FMT
    rng = np.random.default_rng(shape[0] + shape[1])
    w = (rng.standard_normal(shape) * std).astype(np.float32)
    w.reshape(-1)[::97] = -0.0
    fmt = MINIFLOAT_FMT[name]
    wt = torch.from_numpy(w).to(cuda)
    for per_row in (True, False):
        codes, aux = K.quant_minifloat(wt, fmt, per_row)
        ref_codes, ref_s = O.quant_minifloat(w, name, 0 if per_row else None)
        np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes)
        if per_row:
            np.testing.assert_array_equal(aux.cpu().numpy(), ref_s.reshape(-1))
            sc = aux
        else:
            m = float(aux.cpu().numpy()[0])
            assert m == float(np.max(np.abs(w)))
            sc = ref_s
        d = K.dequant_minifloat(fmt, codes, shape[0], shape[1], sc)
        assert _same_f32(d.cpu().numpy(), O.dequant_minifloat(ref_codes, name, shape, ref_s))
        db = K.dequant_minifloat(fmt, codes, shape[0], shape[1], sc, out_dtype=torch.bfloat16)
        np.testing.assert_array_equal(db.float().cpu().numpy(), O.bf16_round(d.cpu().numpy()))


def test_bfloat16_input_rounds_like_its_float32_value(cuda):
    import torch
    from apsi_b200 import kernels as K
    from apsi_b200._lib import MINIFLOAT_FMT
    rng = np.random.default_rng(5)
    w = torch.from_numpy((rng.standard_normal((33, 260)) * 0.3).astype(np.float32)).to(cuda).to(torch.bfloat16)
    codes, s = K.quant_minifloat(w, MINIFLOAT_FMT["fp8_e4m3"], True)
    ref_codes, ref_s = O.quant_minifloat(w.float().cpu().numpy(), "fp8_e4m3", 0)
    np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes)
    np.testing.assert_array_equal(s.cpu().numpy(), ref_s.reshape(-1))


@pytest.mark.parametrize("name", ["fp8_e4m3", "fp8_e5m2"])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (5, 300, 1024), (16, 520, 2048), (64, 1000, 512),
                                   (300, 768, 1024)])
def test_fp8_fused_product_matches_oracle(cuda, name, M, N, K):
    """Per-row fp8 weights through lb_linear (decode GEMV for M <= 16, tcgen05 GEMM above), against the
    float64 product of the oracle's dequantised weights: max-abs <= 1e-2 * max|y|, rel. Frobenius <= 2e-3."""
    import torch
    from apsi_b200 import precision as P
    rng = np.random.default_rng(M * 131 + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = P.quantize(W, name, axis=0)
    codes, s = O.quant_minifloat(W, name, 0)
    Wd = O.dequant_minifloat(codes, name, (N, K), s).astype(np.float64)
    xb = O.bf16_round(x)
    ref = xb.astype(np.float64) @ Wd.T
    y = P.qmatmul(torch.from_numpy(xb).to(cuda).to(torch.bfloat16), q).float().cpu().numpy()
    assert O.max_abs_ratio(y, ref) <= 1e-2
    assert O.rel_frobenius(y, ref) <= 2e-3


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (2, 11008, 4096), (5, 300, 1024), (8, 4096, 11008),
                                   (16, 520, 2048), (12, 1000, 16384), (64, 1000, 512), (17, 300, 1024),
                                   (300, 768, 1024), (2048, 1024, 2048)])
def test_fp4_fused_product_matches_oracle(cuda, M, N, K):
    """Per-row fp4 e2m1 weights: the fused decode GEMV for M <= 16 (codes to exact fp16 through the hardware
    e2m1 conversion; one K range and the cluster split over several), the tcgen05 GEMM above, both against the
    float64 product of the oracle's dequantised weights with the layer tolerance."""
    import torch
    from apsi_b200 import precision as P
    rng = np.random.default_rng(M * 7 + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = P.quantize(W, "fp4_e2m1", axis=0)
    codes, s = O.quant_minifloat(W, "fp4_e2m1", 0)
    Wd = O.dequant_minifloat(codes, "fp4_e2m1", (N, K), s).astype(np.float64)
    xb = O.bf16_round(x)
    ref = xb.astype(np.float64) @ Wd.T
    y = P.qmatmul(torch.from_numpy(xb).to(cuda).to(torch.bfloat16), q).float().cpu().numpy()
    assert O.max_abs_ratio(y, ref) <= 1e-2
    assert O.rel_frobenius(y, ref) <= 2e-3


def test_fp4_through_the_c_abi(cuda):
    """lb_linear with LB_FMT_FP4_E2M1 codes straight from lb_quant_minifloat, on the GEMV and on the GEMM, and
    the GEMM's column shards bit-identical to the full product."""
    import torch
    from apsi_b200 import kernels as K
    from apsi_b200._lib import FMT_FP4_E2M1
    g = torch.Generator(device=cuda)
    g.manual_seed(4)
    N, Kd = 640, 2048
    W = torch.randn((N, Kd), generator=g, device=cuda) * 0.03
    codes, s32 = K.quant_minifloat(W, FMT_FP4_E2M1, True)
    Wd = K.dequant_minifloat(FMT_FP4_E2M1, codes, N, Kd, s32)
    for M in (4, 100):
        x = torch.randn((M, Kd), generator=g, device=cuda).to(torch.bfloat16)
        y = K.linear(FMT_FP4_E2M1, x, codes, s32, N)
        ref = x.float() @ Wd.t()
        assert float((y.float() - ref).abs().max()) <= 1e-2 * float(ref.abs().max())
        half = N // 2
        cv = codes.view(N, Kd // 2)
        for r in range(2):
            part = K.linear(FMT_FP4_E2M1, x, cv[r * half:(r + 1) * half].contiguous(),
                            s32[r * half:(r + 1) * half].contiguous(), half)
            assert torch.equal(part, y[:, r * half:(r + 1) * half])


@pytest.mark.parametrize("name", ["fp6_e3m2", "fp6_e2m3"])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (3, 300, 1040), (8, 1000, 11008), (16, 520, 2048),
                                   (1, 77, 16), (64, 300, 512), (17, 520, 1024), (300, 1000, 4096),
                                   (2048, 1536, 4096), (40, 260, 1040)])
def test_fp6_fused_product_matches_oracle(cuda, name, M, N, K):
    """Per-row fp6 weights: the fused decode product for M <= 16 (four codes per three bytes, exact fp16
    through the hardware conversion, float32 accumulation on the CUDA cores), the tcgen05 GEMM above (codes to
    exact fp16 in the dequantising warps; K % 64 == 0) and dequantise-then-GEMM for other K; all against the
    float64 product of the oracle's dequantised weights with the layer tolerance."""
    import torch
    from apsi_b200 import precision as P
    rng = np.random.default_rng(M * 5 + N + K)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    q = P.quantize(W, name, axis=0)
    codes, s = O.quant_minifloat(W, name, 0)
    Wd = O.dequant_minifloat(codes, name, (N, K), s).astype(np.float64)
    xb = O.bf16_round(x)
    ref = xb.astype(np.float64) @ Wd.T
    y = P.qmatmul(torch.from_numpy(xb).to(cuda).to(torch.bfloat16), q).float().cpu().numpy()
    assert O.max_abs_ratio(y, ref) <= 1e-2
    assert O.rel_frobenius(y, ref) <= 2e-3


@pytest.mark.parametrize("name", ["fp6_e3m2", "fp6_e2m3"])
def test_fp6_through_the_c_abi(cuda, name):
    """lb_linear on fp6 codes straight from lb_quant_minifloat, with bias and accumulation; column shards are
    bit-identical to the full product, on the decode product and on the tcgen05 GEMM; repeated calls give the same
    bits; M > 16 with K % 64 != 0 is LB_E_UNSUPPORTED."""
    import torch
    from apsi_b200 import kernels as K
    from apsi_b200._lib import MINIFLOAT_FMT, LB_E_UNSUPPORTED, LowbitError
    f = MINIFLOAT_FMT[name]
    g = torch.Generator(device=cuda)
    g.manual_seed(8)
    N, Kd, M = 640, 2048, 5
    W = torch.randn((N, Kd), generator=g, device=cuda) * 0.03
    codes, s32 = K.quant_minifloat(W, f, True)
    Wd = K.dequant_minifloat(f, codes, N, Kd, s32)
    x = torch.randn((M, Kd), generator=g, device=cuda).to(torch.bfloat16)
    bias = torch.randn(N, generator=g, device=cuda).to(torch.bfloat16)
    y0 = torch.randn((M, N), generator=g, device=cuda).to(torch.bfloat16)
    y = K.linear(f, x, codes, s32, N, bias=bias, out=y0.clone(), accumulate=True)
    ref = x.float() @ Wd.t() + bias.float() + y0.float()
    assert float((y.float() - ref).abs().max()) <= 1e-2 * float(ref.abs().max())
    full = K.linear(f, x, codes, s32, N)
    assert torch.equal(full, K.linear(f, x, codes, s32, N))
    rb = Kd // 4 * 3
    cv = codes.view(N, rb)
    half = N // 2
    for r in range(2):
        part = K.linear(f, x, cv[r * half:(r + 1) * half].contiguous(), s32[r * half:(r + 1) * half].contiguous(),
                        half)
        assert torch.equal(part, full[:, r * half:(r + 1) * half])
    xg = torch.randn((300, Kd), generator=g, device=cuda).to(torch.bfloat16)    # the tcgen05 GEMM
    yg = K.linear(f, xg, codes, s32, N)
    refg = xg.float() @ Wd.t()
    assert float((yg.float() - refg).abs().max()) <= 1e-2 * float(refg.abs().max())
    for r in range(2):
        part = K.linear(f, xg, cv[r * half:(r + 1) * half].contiguous(), s32[r * half:(r + 1) * half].contiguous(),
                        half)
        assert torch.equal(part, yg[:, r * half:(r + 1) * half])
    K2 = 1040                                                                    # K % 64 != 0: no GEMM
    c2, s2 = K.quant_minifloat(torch.randn((N, K2), generator=g, device=cuda), f, True)
    with pytest.raises(LowbitError) as e:
        K.linear(f, torch.zeros((17, K2), dtype=torch.bfloat16, device=cuda), c2, s2, N)
    assert e.value.code == LB_E_UNSUPPORTED


@pytest.mark.parametrize("name", ["fp8_e4m3", "fp6_e3m2", "fp6_e2m3", "fp4_e2m1"])
def test_tensor_scaled_and_packed_products(cuda, name):
    """axis=None weights and the fp6 / fp4 formats: same tolerance against the oracle's product."""
    import torch
    from apsi_b200 import precision as P
    rng = np.random.default_rng(17)
    N, K, M = 200, 384, 3
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    x = O.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    for axis in (0, None):
        q = P.quantize(W, name, axis=axis)
        codes, s = O.quant_minifloat(W, name, axis)
        ref = x.astype(np.float64) @ O.dequant_minifloat(codes, name, (N, K), s).astype(np.float64).T
        y = P.qmatmul(torch.from_numpy(x).to(cuda).to(torch.bfloat16), q).float().cpu().numpy()
        assert O.max_abs_ratio(y, ref) <= 1e-2, axis
        assert O.rel_frobenius(y, ref) <= 2e-3, axis
