"""lb_linear_noalloc: the product through the C ABI with the library's fixed device scratch instead of a
workspace.  The file name sorts last so these run after every other test (and they also pass alone)."""
import ctypes

import numpy as np
import pytest

from apsi_b200 import _lib, build

TOL_REL_F = 2e-3      # relative Frobenius error of the layer
TOL_MAX_ABS = 1e-2    # max-abs error as a fraction of max |y|


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_noalloc_rejects_shapes_beyond_the_scratch(lib):
    fake = ctypes.c_void_p(1 << 20)    # never dereferenced: the size check fails first
    null = ctypes.c_void_p(0)
    M, K = 4096, 4096                   # 32 MiB of fp16 activations > LB_NOALLOC_SCRATCH_BYTES
    rc = lib.lb_linear_noalloc(_lib.FMT_INT4_G128, fake, M, K, fake, fake, 256, null, 0, fake, 256, null)
    assert rc == _lib.LB_E_WORKSPACE
    assert b"scratch" in lib.lb_last_error()
    rc = lib.lb_linear_noalloc(3, fake, 1, 128, fake, fake, 4, null, 0, fake, 4, null)    # g32: no product
    assert rc == _lib.LB_E_UNSUPPORTED
    rc = lib.lb_linear_noalloc(7, fake, 17, 80, fake, fake, 4, null, 0, fake, 4, null)    # fp6 above M = 16:
    assert rc == _lib.LB_E_UNSUPPORTED                                                    # K % 64 == 0 only


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", [_lib.FMT_INT4_G128, _lib.FMT_INT8_ROW])
@pytest.mark.parametrize("M", [256, 2048, 1])
def test_noalloc_matches_lb_linear_twice_in_a_row(lib, cuda, fmt, M):
    """Two calls in a row: the output is the same bits as lb_linear with a caller workspace (both run the same
    kernels on the same inputs), within the product tolerance of the oracle's float64 product, and the device's
    free memory does not move across the no-allocation call."""
    import torch
    from apsi_b200 import kernels
    from oracle import lowbit_oracle as ora

    N, K = 1024, 4096
    rng = np.random.default_rng(11 + M + fmt)
    Wn = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    W = torch.from_numpy(Wn).to(cuda)
    if fmt == _lib.FMT_INT4_G128:
        codes, s16, _ = kernels.quant_int4_g128(W, want_scale32=False)
        Wd = ora.dequant_int4_g128(codes.cpu().numpy(), s16.cpu().numpy())
    else:
        codes, s16, _ = kernels.quant_int8_rows(W, want_scale32=False)
        Wd = ora.dequant_int8_rows(codes.cpu().numpy(), s16.cpu().numpy())
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    nbytes = kernels.linear_workspace_bytes(fmt, M, N, K)
    ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=cuda) if nbytes else None
    for call in range(2):   # two calls in a row reuse the same scratch
        xn = ora.bf16_round(rng.standard_normal((M, K)).astype(np.float32))
        x = torch.from_numpy(xn).to(cuda).to(torch.bfloat16)
        y_ref = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        _lib.check(lib.lb_linear(fmt, _ptr(x), M, K, _ptr(codes), _ptr(s16), N, None, 0, _ptr(y_ref), N,
                                 _ptr(ws), nbytes, stream))
        torch.cuda.synchronize(cuda)
        free0 = torch.cuda.mem_get_info(cuda)[0]
        _lib.check(lib.lb_linear_noalloc(fmt, _ptr(x), M, K, _ptr(codes), _ptr(s16), N, None, 0, _ptr(y), N,
                                         stream))
        torch.cuda.synchronize(cuda)
        free1 = torch.cuda.mem_get_info(cuda)[0]
        assert free1 == free0, f"call {call}: free device memory moved by {free0 - free1} bytes"
        assert torch.equal(y, y_ref), f"call {call}: lb_linear_noalloc and lb_linear differ"
        a = y.float().cpu().numpy().astype(np.float64)
        ref = ora.linear_ref(xn, Wd)
        assert np.isfinite(a).all(), f"call {call}: unwritten outputs"
        rel, mab = ora.rel_frobenius(a, ref), ora.max_abs_ratio(a, ref)
        assert rel <= TOL_REL_F and mab <= TOL_MAX_ABS, f"call {call}: relF {rel:.3e} maxabs {mab:.3e}"
    assert kernels.device_errors(cuda) == 0
