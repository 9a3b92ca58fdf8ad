"""The C ABI: the library loads, exports every entry point include/apsi_lowbit.h declares, and rejects bad
arguments before touching a device (no compute call is made here)."""
import ctypes
import os
import re

import pytest

from apsi_b200 import _lib, build

HEADER = os.path.join(build.ROOT, "include", "apsi_lowbit.h")


def declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(lb_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported_and_bound(lib):
    names = declared()
    assert len(names) >= 12
    bound = {n for n, _, _ in _lib.SIGNATURES}
    for n in names:
        assert hasattr(lib, n), n
        assert n in bound, f"{n} has no ctypes signature"


def test_version_matches_header(lib):
    v = int(re.search(r"#define LB_VERSION (\d+)", open(HEADER).read()).group(1))
    assert lib.lb_version() == v


def test_constants_match_header():
    text = open(HEADER).read()
    for name, val in (("LB_E_ARG", _lib.LB_E_ARG), ("LB_E_UNSUPPORTED", _lib.LB_E_UNSUPPORTED),
                      ("LB_FMT_INT4_G128", _lib.FMT_INT4_G128), ("LB_FMT_INT8_ROW", _lib.FMT_INT8_ROW),
                      ("LB_DT_F16", _lib.DT_F16), ("LB_FMT_FP8_E4M3", _lib.FMT_FP8_E4M3),
                      ("LB_FMT_FP4_E2M1", _lib.FMT_FP4_E2M1)):
        m = re.search(rf"#define {name} \(?(-?\d+)\)?", text)
        assert int(m.group(1)) == val, name


def test_bad_arguments_are_rejected_before_launch(lib):
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(1 << 20)            # never dereferenced: the checks fail first
    assert lib.lb_quant_int4_g128(null, 0, 4, 128, fake, fake, null, null) == _lib.LB_E_ARG
    assert lib.lb_quant_int4_g128(fake, 0, 4, 100, fake, fake, null, null) == _lib.LB_E_ARG     # K % 128
    assert b"multiple of 128" in lib.lb_last_error()
    assert lib.lb_quant_int4_g128(fake, 7, 4, 128, fake, fake, null, null) == _lib.LB_E_ARG     # dtype
    assert lib.lb_quant_int8_rows(fake, 0, 0, 64, fake, fake, null, null) == _lib.LB_E_ARG      # N = 0
    assert lib.lb_linear(3, fake, 1, 128, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_UNSUPPORTED
    assert lib.lb_linear(7, fake, 32, 80, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_UNSUPPORTED
    assert lib.lb_linear(7, fake, 32, 128, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_WORKSPACE
    assert lib.lb_linear(8, fake, 1, 40, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_ARG  # K % 16
    assert lib.lb_linear(2, fake, 1, 100, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_ARG
    assert lib.lb_linear(2, fake, 1, 128, fake, fake, 8, null, 0, fake, 4, null, 0, null) == _lib.LB_E_ARG  # ldy
    odd = ctypes.c_void_p((1 << 20) + 2)
    assert lib.lb_linear(2, odd, 1, 128, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_ALIGN
    assert lib.lb_dequant(2, fake, fake, 5, 4, 128, fake, 0, null) == _lib.LB_E_ARG             # scale dtype
    assert lib.lb_dequant(3, fake, fake, _lib.DT_F16, 4, 128, fake, 0, null) == _lib.LB_E_ARG    # g32 needs f32
    assert lib.lb_quant_minifloat(2, fake, 0, 4, 8, 1, fake, fake, null, null) == _lib.LB_E_ARG  # not a minifloat
    assert lib.lb_quant_minifloat(5, fake, 0, 4, 8, 1, fake, null, null, null) == _lib.LB_E_ARG  # per row: scale32
    assert lib.lb_quant_minifloat(5, fake, 0, 4, 8, 0, fake, null, null, null) == _lib.LB_E_ARG  # tensor: absmax
    assert lib.lb_quant_minifloat(5, odd, 0, 4, 8, 1, fake, fake, null, null) == _lib.LB_E_ALIGN
    assert lib.lb_dequant_minifloat(5, fake, 4, 8, 1, null, 1.0, fake, 0, null) == _lib.LB_E_ARG
    assert lib.lb_dequant_minifloat(9, fake, 4, 8, 0, null, 1.0, fake, 7, null) == _lib.LB_E_ARG  # out dtype
    assert [lib.lb_minifloat_bytes(f, 7) for f in (5, 6, 7, 8, 9, 2)] == [7, 7, 6, 6, 4, -1]
    assert lib.lb_linear(9, fake, 32, 128, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_WORKSPACE
    assert lib.lb_linear(9, fake, 1, 64, fake, fake, 4, null, 0, fake, 4, null, 0, null) == _lib.LB_E_ARG  # K % 128
    f = ctypes.c_float(1e-6)
    assert lib.lb_linear_rms(2, fake, 1, 128, null, 1, f, f, fake, fake, 4, null, 0, fake, 4, null, 0, 0,
                             null) == _lib.LB_E_ARG                                             # no ln weights
    assert lib.lb_linear_rms(2, fake, 1, 128, fake, 7, f, f, fake, fake, 4, null, 0, fake, 4, null, 0, 0,
                             null) == _lib.LB_E_ARG                                             # ln dtype
    assert lib.lb_linear_rms(2, fake, 1, 128, odd, _lib.DT_F32, f, f, fake, fake, 4, null, 0, fake, 4, null, 0, 0,
                             null) == _lib.LB_E_ALIGN
    assert lib.lb_linear_rms(2, fake, 32, 128, fake, _lib.DT_F32, f, f, fake, fake, 4, null, 0, fake, 4, null, 0, 0,
                             null) == _lib.LB_E_WORKSPACE                                       # prefill: workspace


def test_prepared_weight_arguments_are_checked_before_the_device(lib):
    null = ctypes.c_void_p(0)
    fake = ctypes.c_void_p(1 << 20)
    odd = ctypes.c_void_p((1 << 20) + 8)
    h = ctypes.c_void_p()
    assert lib.lb_weight_create(2, fake, fake, 4, 128, None) == _lib.LB_E_ARG                   # no out
    assert lib.lb_weight_create(3, fake, fake, 4, 128, ctypes.byref(h)) == _lib.LB_E_UNSUPPORTED  # g32 words
    assert lib.lb_weight_create(2, null, fake, 4, 128, ctypes.byref(h)) == _lib.LB_E_ARG
    assert lib.lb_weight_create(2, fake, fake, 0, 128, ctypes.byref(h)) == _lib.LB_E_ARG
    assert lib.lb_weight_create(2, fake, fake, 4, 100, ctypes.byref(h)) == _lib.LB_E_ARG        # K % 128
    assert lib.lb_weight_create(1, fake, fake, 4, 96, ctypes.byref(h)) == _lib.LB_E_ARG         # K % 64
    assert lib.lb_weight_create(2, odd, fake, 4, 128, ctypes.byref(h)) == _lib.LB_E_ALIGN
    assert h.value is None
    assert lib.lb_weight_linear(null, fake, 1, fake, 4, 0, null) == _lib.LB_E_ARG
    assert lib.lb_weight_destroy(null) == 0


def test_workspace_query(lib):
    n = ctypes.c_size_t(123)
    assert lib.lb_linear_workspace_size(2, 1, 4096, 4096, ctypes.byref(n)) == 0
    assert n.value == 0                                         # the decode GEMV needs no workspace
    assert lib.lb_linear_workspace_size(2, 2048, 4096, 4096, ctypes.byref(n)) == 0
    assert n.value >= 2048 * 4096 * 2                           # fp16 activations of the GEMM
    assert lib.lb_linear_workspace_size(4, 1, 4, 128, ctypes.byref(n)) == _lib.LB_E_UNSUPPORTED
    assert lib.lb_linear_workspace_size(9, 16, 4, 128, ctypes.byref(n)) == 0 and n.value == 0   # fp4: decode GEMV
    assert lib.lb_linear_workspace_size(9, 17, 4, 128, ctypes.byref(n)) == 0 and n.value > 0    # fp4: GEMM
    assert lib.lb_linear_workspace_size(7, 16, 4, 128, ctypes.byref(n)) == 0 and n.value == 0   # fp6: decode
    assert lib.lb_linear_workspace_size(8, 17, 4, 128, ctypes.byref(n)) == 0 and n.value > 0    # fp6: GEMM
    assert lib.lb_linear_workspace_size(8, 17, 4, 80, ctypes.byref(n)) == _lib.LB_E_UNSUPPORTED   # K % 64
    assert lib.lb_linear_rms_workspace_size(2, 16, 4096, 4096, ctypes.byref(n)) == 0 and n.value == 0
    g = ctypes.c_size_t(0)
    assert lib.lb_linear_workspace_size(2, 2048, 4096, 4096, ctypes.byref(g)) == 0
    assert lib.lb_linear_rms_workspace_size(2, 2048, 4096, 4096, ctypes.byref(n)) == 0
    assert n.value == g.value + 2048 * 4096 * 2                 # the normalised rows, then the GEMM's own


def test_python_layer_raises_loudly_without_a_device():
    import torch
    from apsi_b200 import kernels
    if torch.cuda.is_available():
        pytest.skip("a device is present")
    with pytest.raises(_lib.LowbitError):
        kernels.quant_int4_g128(torch.zeros(4, 128))
    x = torch.zeros(2, 128, dtype=torch.bfloat16)
    codes, s16 = torch.zeros(4, 64, dtype=torch.uint8), torch.zeros(4, 1, dtype=torch.float16)
    for call in (lambda: kernels.linear(_lib.FMT_INT4_G128, x, codes, s16, 4),
                 lambda: kernels.linear(_lib.FMT_FP4_E2M1, x, codes, torch.zeros(4), 4),
                 lambda: kernels.linear_rms(_lib.FMT_INT4_G128, x, torch.ones(128), codes, s16, 4),
                 lambda: kernels.rmsnorm(x, torch.ones(128)),
                 lambda: kernels.act_mul(torch.zeros(2, 256, dtype=torch.bfloat16), 128)):
        with pytest.raises(_lib.LowbitError):      # host tensors: refused, never computed on the CPU
            call()


def test_product_operand_checks_reject_short_or_wrong_outputs():
    """kernels._check_product, run on host tensors: an output with too few rows or columns, the wrong dtype or a
    column stride, and codes / scales / bias smaller than the format needs are rejected before any call."""
    import torch
    from apsi_b200 import kernels as Kn
    M, N, K = 3, 64, 256
    x = torch.zeros((M, K), dtype=torch.bfloat16)
    codes = torch.zeros((N, K // 2), dtype=torch.uint8)
    s16 = torch.zeros((N, K // 128), dtype=torch.float16)
    ok = torch.zeros((M, N), dtype=torch.bfloat16)
    Kn._check_product(_lib.FMT_INT4_G128, x, M, K, codes, s16, N, None, ok)            # fits
    Kn._check_product(_lib.FMT_INT4_G128, x, M, K, codes, s16, N, None,
                      torch.zeros((M, 2 * N), dtype=torch.bfloat16)[:, :N])              # strided rows: fine
    bad_outs = [torch.zeros((M - 1, N), dtype=torch.bfloat16),                          # too few rows
                torch.zeros((M, N - 1), dtype=torch.bfloat16),                          # too few columns
                torch.zeros((M, N), dtype=torch.float32),                               # wrong dtype
                torch.zeros((N, M), dtype=torch.bfloat16).t()]                          # column stride != 1
    for out in bad_outs:
        with pytest.raises(_lib.LowbitError) as e:
            Kn._check_product(_lib.FMT_INT4_G128, x, M, K, codes, s16, N, None, out)
        assert e.value.code == _lib.LB_E_ARG
    with pytest.raises(_lib.LowbitError, match="codes holds"):
        Kn._check_product(_lib.FMT_INT4_G128, x, M, K, codes[:-1], s16, N, None, ok)
    with pytest.raises(_lib.LowbitError, match="scales holds"):
        Kn._check_product(_lib.FMT_INT8_ROW, x, M, K, torch.zeros((N, K), dtype=torch.int8),
                          torch.zeros((N - 1,), dtype=torch.float16), N, None, ok)
    with pytest.raises(_lib.LowbitError, match="bias"):
        Kn._check_product(_lib.FMT_INT4_G128, x, M, K, codes, s16, N, torch.zeros((N - 1,), dtype=torch.bfloat16),
                          ok)
