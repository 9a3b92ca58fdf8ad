"""The oracle against golden vectors written by the reference itself (tests/golden/make_golden.py):
int4 groups of 128, int8 rows, ggml-style g32 blocks, dequantisation and the quantized product."""
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
