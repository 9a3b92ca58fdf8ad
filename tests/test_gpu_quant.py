"""Quantisation kernels on the GPU, bit-exact against the reference's golden vectors and the oracle."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def test_int4_g128_bit_exact_with_reference_golden(cuda, golden):
    from apsi_b200 import kernels as K
    packed, s16, s32 = K.quant_int4_g128(_t(golden["w4"], cuda))
    np.testing.assert_array_equal(packed.cpu().numpy(), golden["w4_packed"])
    np.testing.assert_array_equal(s32.cpu().numpy(), golden["w4_scale32"])
    np.testing.assert_array_equal(s16.cpu().numpy(), golden["w4_scale32"].astype(np.float16))


def test_int8_rows_bit_exact_with_reference_golden(cuda, golden):
    from apsi_b200 import kernels as K
    codes, s16, s32 = K.quant_int8_rows(_t(golden["w8"], cuda))
    np.testing.assert_array_equal(codes.cpu().numpy(), golden["w8_codes"])
    np.testing.assert_array_equal(s32.cpu().numpy(), golden["w8_scale32"])
    np.testing.assert_array_equal(s16.cpu().numpy(), golden["w8_scale32"].astype(np.float16))


@pytest.mark.parametrize("shape,std", [((64, 4096), 0.02), ((11008, 4096), 0.02), ((96, 1280), 3.0),
                                       ((7, 128), 1e-3), ((300, 11008), 0.015)])
def test_int4_g128_matches_oracle_random(cuda, shape, std):
    from apsi_b200 import kernels as K
    rng = np.random.default_rng(shape[0] * 7 + shape[1])
    w = (rng.standard_normal(shape) * std).astype(np.float32)
    # plant exact ties and all-zero groups
    w[0, :128] = 0.0
    w[1, :128] = np.resize((np.arange(-7, 7) + 0.5) * 0.25, 128)
    w[1, 0] = 1.75
    packed, s16, s32 = K.quant_int4_g128(_t(w, cuda))
    rp, r32, r16 = O.quant_int4_g128(w)
    np.testing.assert_array_equal(packed.cpu().numpy(), rp)
    np.testing.assert_array_equal(s32.cpu().numpy(), r32)
    np.testing.assert_array_equal(s16.cpu().numpy(), r16)


@pytest.mark.parametrize("shape", [(4096, 4096), (33, 392), (5, 11008)])
def test_int8_rows_matches_oracle_random(cuda, shape):
    from apsi_b200 import kernels as K
    rng = np.random.default_rng(shape[1])
    w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
    w[0] = 0.0
    codes, s16, s32 = K.quant_int8_rows(_t(w, cuda))
    rc, r32, r16 = O.quant_int8_rows(w)
    np.testing.assert_array_equal(codes.cpu().numpy(), rc)
    np.testing.assert_array_equal(s32.cpu().numpy(), r32)


def test_bf16_input_quantises_the_bf16_values(cuda):
    import torch
    from apsi_b200 import kernels as K
    rng = np.random.default_rng(5)
    w = O.bf16_round((rng.standard_normal((48, 512)) * 0.05).astype(np.float32))
    wb = _t(w, cuda).to(torch.bfloat16)
    packed, s16, s32 = K.quant_int4_g128(wb)
    rp, r32, _ = O.quant_int4_g128(w)
    np.testing.assert_array_equal(packed.cpu().numpy(), rp)
    np.testing.assert_array_equal(s32.cpu().numpy(), r32)


@pytest.mark.parametrize("kind", ["int8", "int4"])
def test_g32_words_match_hub_gpu_qnumpy(cuda, golden, kind):
    from apsi_b200 import kernels as K
    w = golden["wg"]
    with np.errstate(over="ignore", invalid="ignore"):
        q, sc = O.qnumpy_g32(w, kind)
    ok = np.isfinite(q).all(axis=1)                 # rows whose reference codes are NaN (subnormal scale) excluded
    w, q, sc = w[ok], q[ok], sc[ok]
    if kind == "int8":
        words, s32 = K.quant_q8_0_g32(_t(w, cuda))
        ref = O.pack_q8_0_words(q)
    else:
        words, s32 = K.quant_q4_0_g32(_t(w, cuda))
        ref = O.pack_q4_0_words(q)
    np.testing.assert_array_equal(words.cpu().numpy().view(np.uint32), ref)
    np.testing.assert_array_equal(s32.cpu().numpy(), sc)


def test_dequant_matches_reference_bits(cuda, golden):
    import torch
    from apsi_b200 import kernels as K
    from apsi_b200._lib import FMT_INT4_G128, FMT_INT8_ROW
    n, k = golden["w4"].shape
    out = K.dequant(FMT_INT4_G128, _t(golden["w4_packed"], cuda), _t(golden["w4_scale32"], cuda), n, k)
    np.testing.assert_array_equal(out.cpu().numpy(), golden["w4_deq32"])
    n8, k8 = golden["w8"].shape
    out8 = K.dequant(FMT_INT8_ROW, _t(golden["w8_codes"], cuda), _t(golden["w8_scale32"], cuda), n8, k8)
    np.testing.assert_array_equal(out8.cpu().numpy(), golden["w8_deq32"])
    s16 = _t(golden["w4_scale32"].astype(np.float16), cuda)
    outb = K.dequant(FMT_INT4_G128, _t(golden["w4_packed"], cuda), s16, n, k, out_dtype=torch.bfloat16)
    ref = O.bf16_round(O.dequant_int4_g128(golden["w4_packed"], golden["w4_scale32"].astype(np.float16)))
    np.testing.assert_array_equal(outb.float().cpu().numpy(), ref)
