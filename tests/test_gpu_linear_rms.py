"""The normalised projection ``lb_linear_rms`` (the reference's ``_Base.linear(x, W, ln=...)`` and its gemvq*n
kernels, apsi/hub_gpu.py:1305-1315, 837-870): for M <= 16 the RMSNorm runs inside the decode GEMV's activation
staging, above it ``lb_rmsnorm`` precedes the GEMM.  Either way the result is bit-identical to ``lb_rmsnorm``
followed by ``lb_linear``, and within the layer tolerance of the oracle's float32 RMSNorm + product."""
import numpy as np
import pytest

import oracle as O
from oracle import lowbit_oracle as ora

pytestmark = pytest.mark.gpu


def _weights(torch, cuda, N, K, fmt, seed):
    from apsi_b200 import kernels as Kn
    from apsi_b200._lib import FMT_INT4_G128, FMT_INT8_ROW
    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    W = torch.randn((N, K), generator=g, device=cuda) * 0.02
    if fmt == "int4":
        codes, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
        return FMT_INT4_G128, codes, s16
    if fmt == "int8":
        codes, s16, _ = Kn.quant_int8_rows(W, want_scale32=False)
        return FMT_INT8_ROW, codes, s16
    from apsi_b200._lib import MINIFLOAT_FMT       # fp8 / fp4 rows: float32 row scales
    f = MINIFLOAT_FMT[fmt]
    codes, s32 = Kn.quant_minifloat(W, f, True)
    return f, codes, s32


@pytest.mark.parametrize("M,N,K", [(1, 11008, 4096), (8, 6144, 4096), (8, 22016, 4096), (3, 520, 1024),
                                   (12, 300, 2048), (16, 1000, 4096), (5, 4096, 11008), (1, 256, 16384),
                                   (40, 520, 2048), (300, 1024, 4096)])
@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("ln_dtype", ["bf16", "f32"])
def test_fused_norm_is_bit_identical_to_norm_then_linear(cuda, M, N, K, fmt, ln_dtype):
    import torch
    from apsi_b200 import kernels as Kn
    f, codes, s16 = _weights(torch, cuda, N, K, fmt, seed=M + N + K)
    g = torch.Generator(device=cuda)
    g.manual_seed(7 * M + K)
    x = (torch.randn((M, K), generator=g, device=cuda) * 3.0).to(torch.bfloat16)
    ln = torch.randn(K, generator=g, device=cuda) * 0.2 + 1.0
    ln = ln.to(torch.bfloat16) if ln_dtype == "bf16" else ln
    for eps, off in ((1e-5, 0.0), (1e-6, 1.0)):
        ref = Kn.linear(f, Kn.rmsnorm(x, ln, eps=eps, off=off), codes, s16, N)
        got = Kn.linear_rms(f, x, ln, codes, s16, N, eps=eps, off=off)
        torch.cuda.synchronize()
        assert Kn.device_errors() == 0
        assert torch.equal(got, ref), (eps, off)


@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (8, 1000, 2048), (5, 640, 11008), (40, 520, 2048)])
@pytest.mark.parametrize("fmt", ["fp8_e4m3", "fp8_e5m2", "fp4_e2m1"])
def test_fused_norm_on_minifloat_rows(cuda, M, N, K, fmt):
    """The norm prologue on the fp16-staged formats (fp8, fp4 rows): the same bits as the norm followed by the
    product, on the GEMV (one K range and several) and on the GEMM."""
    import torch
    from apsi_b200 import kernels as Kn
    f, codes, sc = _weights(torch, cuda, N, K, fmt, seed=M * 3 + N + K)
    g = torch.Generator(device=cuda)
    g.manual_seed(M + 2 * K)
    x = (torch.randn((M, K), generator=g, device=cuda) * 2.0).to(torch.bfloat16)
    ln = (torch.randn(K, generator=g, device=cuda) * 0.2 + 1.0).to(torch.bfloat16)
    ref = Kn.linear(f, Kn.rmsnorm(x, ln, eps=1e-5, off=0.5), codes, sc, N)
    got = Kn.linear_rms(f, x, ln, codes, sc, N, eps=1e-5, off=0.5)
    torch.cuda.synchronize()
    assert Kn.device_errors() == 0
    assert torch.equal(got, ref)


def test_fused_norm_with_bias_accumulate_static_and_unaligned_weights(cuda):
    import torch
    from apsi_b200 import kernels as Kn
    M, N, K = 6, 1000, 4096
    f, codes, s16 = _weights(torch, cuda, N, K, "int4", seed=5)
    g = torch.Generator(device=cuda)
    g.manual_seed(9)
    x = torch.randn((M, K), generator=g, device=cuda).to(torch.bfloat16)
    base = (torch.randn(K + 1, generator=g, device=cuda) * 0.1 + 1.0).to(torch.bfloat16)
    ln = base[1:]                                        # 2-byte aligned only: the scalar weight loads
    bias = torch.randn(N, generator=g, device=cuda).to(torch.bfloat16)
    y0 = torch.randn((M, N), generator=g, device=cuda).to(torch.bfloat16)
    ref = Kn.linear(f, Kn.rmsnorm(x, ln.contiguous(), eps=1e-5), codes, s16, N, bias=bias, out=y0.clone(),
                    accumulate=True)
    got = Kn.linear_rms(f, x, ln, codes, s16, N, eps=1e-5, bias=bias, out=y0.clone(), accumulate=True,
                        static_weights=True)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)
    x0 = x.clone()
    Kn.linear_rms(f, x, ln, codes, s16, N, eps=1e-5)
    assert torch.equal(x, x0)                           # the fused path does not write x


def test_fused_norm_matches_the_oracle(cuda):
    import torch
    from apsi_b200 import kernels as Kn
    from apsi_b200._lib import FMT_INT4_G128
    M, N, K = 4, 384, 2048
    x, W = O.make_config_inputs(M, N, K, seed=17)
    g = (np.random.default_rng(2).standard_normal(K) * 0.1 + 1.0).astype(np.float32)
    packed, _, s16 = O.quant_int4_g128(W)
    Wd = O.dequant_int4_g128(packed, s16)
    xb = O.bf16_round(x)
    xn = O.bf16_round(ora.rms_norm(xb, O.bf16_round(g), eps=1e-5))
    ref = O.linear_ref(xn, Wd)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    y = Kn.linear_rms(FMT_INT4_G128, t(x).to(torch.bfloat16), t(g).to(torch.bfloat16), t(packed), t(s16), N,
                      eps=1e-5)
    y = y.float().cpu().numpy()
    assert O.max_abs_ratio(y, ref) <= 1e-2 and O.rel_frobenius(y, ref) <= 2e-3


@pytest.mark.parametrize("K", [4096, 1000, 13])
def test_rmsnorm_vector_and_scalar_loads_agree(cuda, K):
    """lb_rmsnorm gives the same bits with 16-byte loads (aligned rows, K % 8 == 0) and element loads."""
    import torch
    from apsi_b200 import kernels as Kn
    g = torch.Generator(device=cuda)
    g.manual_seed(K)
    M = 5
    x = (torch.randn((M, K), generator=g, device=cuda) * 2).to(torch.bfloat16)
    w = torch.randn(K, generator=g, device=cuda) * 0.1 + 1.0
    a = Kn.rmsnorm(x, w, eps=1e-6, off=0.25)
    buf = torch.empty(M * K + 1, dtype=torch.bfloat16, device=cuda)
    xs = buf[1:].view(M, K)                              # 2-byte aligned rows
    xs.copy_(x)
    b = Kn.rmsnorm(xs, w, eps=1e-6, off=0.25)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    ref = ora.rms_norm(x.float().cpu().numpy(), w.cpu().numpy(), eps=1e-6, off=0.25)
    got = a.float().cpu().numpy()
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -8 + 1e-30)

