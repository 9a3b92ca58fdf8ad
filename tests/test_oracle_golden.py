"""The oracle against golden vectors written by the reference itself (tests/golden/make_golden.py):
int4 groups of 128, int8 rows, ggml-style g32 blocks, dequantisation, the quantized product, the minifloat
formats and the GGUF Q8_0 / Q4_0 blocks."""
import numpy as np

import oracle as O


def test_int4_g128_codes_and_scales_match_reference(golden):
    packed, s32, s16 = O.quant_int4_g128(golden["w4"])
    np.testing.assert_array_equal(packed, golden["w4_packed"])
    np.testing.assert_array_equal(s32, golden["w4_scale32"])
    np.testing.assert_array_equal(s16, golden["w4_scale32"].astype(np.float16))


def test_int4_dequant_with_fp32_scale_matches_reference(golden):
    packed, s32, _ = O.quant_int4_g128(golden["w4"])
    n, k = golden["w4"].shape
    codes = O.unpack4(packed, n * k).reshape(n, k // 128, 128).astype(np.float32)
    np.testing.assert_array_equal((codes * s32[:, :, None]).reshape(n, k), golden["w4_deq32"])


def test_int8_rows_match_reference(golden):
    codes, s32, s16 = O.quant_int8_rows(golden["w8"])
    np.testing.assert_array_equal(codes, golden["w8_codes"])
    np.testing.assert_array_equal(s32, golden["w8_scale32"])
    np.testing.assert_array_equal(codes.astype(np.float32) * s32[:, None], golden["w8_deq32"])


def test_g32_blocks_match_hub_gpu_qnumpy(golden):
    with np.errstate(over="ignore", invalid="ignore"):
        for kind in ("int8", "int4"):
            q, sc = O.qnumpy_g32(golden["wg"], kind)
            np.testing.assert_array_equal(q, golden[f"wg_{kind}_q"])
            np.testing.assert_array_equal(sc, golden[f"wg_{kind}_scale"])


def test_quantized_product_matches_reference_qmatmul(golden):
    x, w = golden["mm_x"], golden["mm_w"]
    packed, s32, _ = O.quant_int4_g128(w)
    n, k = w.shape
    wd = (O.unpack4(packed, n * k).reshape(n, k // 128, 128).astype(np.float32) * s32[:, :, None]).reshape(n, k)
    np.testing.assert_allclose(x @ wd.T, golden["mm_y_qmatmul"], rtol=1e-5, atol=1e-6)


def test_pack4_layout_low_nibble_is_even_element():
    codes = np.array([1, -1, 7, -8, 0, 3], np.int8)
    p = O.pack4(codes)
    assert p.tolist() == [0xF1, 0x87, 0x30]
    np.testing.assert_array_equal(O.unpack4(p, 6), codes)


def test_g32_word_layouts():
    q = np.arange(-8, 8, dtype=np.float32)
    q = np.concatenate([q, q])[None, :]
    w4 = O.pack_q4_0_words(q)
    assert w4.shape == (1, 4)
    assert int(w4[0, 0]) & 0xF == 0 and (int(w4[0, 0]) >> 28) == 7        # q + 8, value j in nibble j
    w8 = O.pack_q8_0_words(q)
    assert (int(w8[0, 0]) & 0xFF) == 0xF8                                 # two's complement bytes


def test_error_metrics():
    ref = np.array([[1.0, -2.0, 4.0]])
    assert O.rel_frobenius(ref, ref) == 0.0
    assert abs(O.max_abs_ratio(ref + np.array([[0, 0, 0.04]]), ref) - 0.01) < 1e-12


def test_round_weights_matches_reference_lowbit(golden):
    for kind in ("int8", "int4"):
        got = O.round_weights_g32(golden["rw_in"], kind)
        assert np.array_equal(got.view(np.uint32), golden[f"rw_{kind}"].view(np.uint32)), kind


MINIFLOAT_NAMES = ("fp8_e4m3", "fp8_e5m2", "fp6_e3m2", "fp6_e2m3", "fp4_e2m1")


def test_minifloat_rows_match_reference(golden):
    """Per-row scales (axis=0): ties to the even code, saturation, NaN / inf rows, signed zeros."""
    for name in MINIFLOAT_NAMES:
        W = golden[f"mf_{name}_w"]
        codes, s = O.quant_minifloat(W, name, 0)
        np.testing.assert_array_equal(codes, golden[f"mf_{name}_codes"], err_msg=name)
        np.testing.assert_array_equal(s.reshape(-1), golden[f"mf_{name}_scale"], err_msg=name)
        d = O.dequant_minifloat(codes, name, W.shape, s)
        assert np.array_equal(d.view(np.uint32)[~np.isnan(d)], golden[f"mf_{name}_deq"].view(np.uint32)[~np.isnan(d)])
        np.testing.assert_array_equal(np.isnan(d), np.isnan(golden[f"mf_{name}_deq"]))


def test_minifloat_tensor_scale_matches_reference(golden):
    """One float64 scale for the tensor (axis=None); packing runs across rows for odd sizes."""
    for name in MINIFLOAT_NAMES:
        W = golden[f"mf_{name}_t_w"]
        codes, s = O.quant_minifloat(W, name, None)
        np.testing.assert_array_equal(codes, golden[f"mf_{name}_t_codes"], err_msg=name)
        assert s == float(golden[f"mf_{name}_t_scale"][0])
        d = O.dequant_minifloat(codes, name, W.shape, s)
        assert np.array_equal(d.view(np.uint32), golden[f"mf_{name}_t_deq"].view(np.uint32)), name


def test_minifloat_tables_and_pack6():
    assert [O.minifloat_max(n) for n in MINIFLOAT_NAMES] == [448.0, 57344.0, 28.0, 7.5, 6.0]
    t = O.minifloat_table("fp8_e4m3")
    assert np.isnan(t[0x7F]) and t[1] == 2.0 ** -9 and t[0x08] == 2.0 ** -6
    c = np.array([1, 2, 3, 63, 5], np.uint8)
    p = O.pack6(c)
    assert p.size == 6 and p[0] == (1 | (2 << 6)) & 0xFF
    np.testing.assert_array_equal(O.unpack6(p, 5), c)


def test_gguf_blocks_match_reference(golden):
    G = golden["gguf_w"]
    np.testing.assert_array_equal(O.gguf_q8_0(G), golden["gguf_q8_0"])
    np.testing.assert_array_equal(O.gguf_q4_0(G), golden["gguf_q4_0"])
    np.testing.assert_array_equal(O.gguf_dequant(golden["gguf_q8_0"], "q8_0", G.size), golden["gguf_dq8_0"])
    np.testing.assert_array_equal(O.gguf_dequant(golden["gguf_q4_0"], "q4_0", G.size), golden["gguf_dq4_0"])
