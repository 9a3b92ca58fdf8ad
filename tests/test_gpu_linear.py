"""The fused dequantise-and-matmul kernels against the oracle: max-abs error <= 1e-2 * max|y| and relative
Frobenius error <= 2e-3 (float32 accumulation, bfloat16 output), on the decode GEMV (M <= 16, persistent and
cluster paths) and the tcgen05 GEMM (M > 16), with bias and accumulation, and the column-sharding invariant
(outputs of a row slice of W are bit-identical to the same rows of the full product)."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
MAXABS, RELF = 1e-2, 2e-3


def _t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _case(M, N, K, seed, fmt, outliers=0.0):
    x, W = O.make_config_inputs(M, N, K, seed=seed, outliers=outliers)
    if fmt == "int4":
        codes, _, s16 = O.quant_int4_g128(W)
        Wd = O.dequant_int4_g128(codes, s16)
    else:
        codes, _, s16 = O.quant_int8_rows(W)
        Wd = O.dequant_int8_rows(codes, s16)
    return x, codes, s16, Wd


def _run(cuda, fmt, x, codes, s16, N, bias=None, y0=None):
    import torch
    from apsi_b200 import kernels as K
    from apsi_b200._lib import FMT_INT4_G128, FMT_INT8_ROW
    f = FMT_INT4_G128 if fmt == "int4" else FMT_INT8_ROW
    xt = _t(x, cuda).to(torch.bfloat16)
    bt = _t(bias, cuda).to(torch.bfloat16) if bias is not None else None
    out = _t(y0, cuda).to(torch.bfloat16) if y0 is not None else None
    y = K.linear(f, xt, _t(codes, cuda), _t(s16, cuda), N, bias=bt, out=out, accumulate=y0 is not None)
    torch.cuda.synchronize()
    assert K.device_errors() == 0
    return y.float().cpu().numpy()


def _check(y, ref):
    assert np.isfinite(y).all()
    assert O.max_abs_ratio(y, ref) <= MAXABS, O.max_abs_ratio(y, ref)
    assert O.rel_frobenius(y, ref) <= RELF, O.rel_frobenius(y, ref)


SHAPES = [
    (1, 11008, 4096), (4, 11008, 4096), (16, 11008, 4096),      # configs[1] up projection
    (1, 4096, 11008), (4, 4096, 11008), (16, 4096, 11008),      # configs[1] down projection
    (1, 4096, 4096),                                            # configs[0] shape
    (1, 300, 512), (3, 96, 1024), (5, 520, 1280), (9, 200, 384), (2, 17, 128), (1, 1, 256),   # ragged
    (8, 2400, 2048), (13, 3000, 6144), (6, 1000, 11008), (8, 4096, 11008),
    (17, 300, 1024), (40, 520, 2048), (64, 1000, 4096), (130, 257, 512), (256, 1024, 1024),  # GEMM
    (300, 520, 2048), (2048, 12288, 4096),                      # configs[2]
    (64, 1000, 16384), (100, 520, 28672), (128, 384, 14336), (17, 256, 20480),   # K split over CTAs (M <= 128)
]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("fmt", ["int4", "int8"])
def test_linear_matches_oracle(cuda, M, N, K, fmt):
    if fmt == "int8" and K % 64:
        pytest.skip("int8 rows need K % 64 == 0")
    x, codes, s16, Wd = _case(M, N, K, seed=M * 131 + N + K, fmt=fmt, outliers=0.001 if M == 2048 else 0.0)
    y = _run(cuda, fmt, x, codes, s16, N)
    _check(y, O.linear_ref(x, Wd))


@pytest.mark.parametrize("M,N,K", [(1, 520, 1024), (6, 300, 2048), (48, 400, 1024)])
def test_bias_and_accumulate(cuda, M, N, K):
    rng = np.random.default_rng(11)
    x, codes, s16, Wd = _case(M, N, K, seed=3, fmt="int4")
    bias = O.bf16_round(rng.standard_normal(N).astype(np.float32))
    y0 = O.bf16_round(rng.standard_normal((M, N)).astype(np.float32))
    y = _run(cuda, "int4", x, codes, s16, N, bias=bias, y0=y0)
    _check(y, O.linear_ref(x, Wd, bias=bias, y0=y0))


@pytest.mark.parametrize("M,N,K", [(1, 11008, 4096), (4, 4096, 11008), (1, 8192, 28672), (16, 2048, 4096),
                                   (2, 1376, 4096), (1, 28672, 8192), (8, 4096, 11008), (300, 12288, 1024),
                                   (2048, 12288, 4096), (64, 8192, 28672), (100, 2048, 16384)])
@pytest.mark.parametrize("shards", [2, 8])
def test_column_shards_are_bit_identical(cuda, M, N, K, shards):
    """Each shard of rows computed alone (the multi-GPU layout) gives exactly the full product's columns,
    even when the shard runs on a different execution path (cluster split vs persistent GEMV; whole tiles vs
    the token-cut tiles of a GEMM's last wave)."""
    import torch
    from apsi_b200 import kernels as Kn
    from apsi_b200._lib import FMT_INT4_G128
    g = torch.Generator(device=cuda)
    g.manual_seed(M + N + K)
    W = torch.randn((N, K), generator=g, device=cuda) * 0.02
    codes, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
    x = torch.randn((M, K), generator=g, device=cuda).to(torch.bfloat16)
    full = Kn.linear(FMT_INT4_G128, x, codes, s16, N)
    nl = N // shards
    for r in range(shards):
        part = Kn.linear(FMT_INT4_G128, x, codes[r * nl:(r + 1) * nl].contiguous(),
                         s16[r * nl:(r + 1) * nl].contiguous(), nl)
        assert torch.equal(part, full[:, r * nl:(r + 1) * nl]), (r, nl)


@pytest.mark.parametrize("N,K", [(28672, 8192), (8192, 28672)])
@pytest.mark.parametrize("M", [1, 64, 2048])
def test_configs4_rows_match_oracle(cuda, M, N, K):
    """configs[4] (the 70B MLP: gate/up [28672, 8192], down [8192, 28672], W ~ N(0, 0.015)) at the sizes the
    bench reports.  The whole matrix is quantised and multiplied on the device; three 512-row slices (first,
    middle, last) are then (1) quantised by the oracle bit for bit as the device did, (2) multiplied alone and
    found bit-identical to the same columns of the full product (the reduction depends only on K, whatever
    path the slice takes), and (3) within the layer's tolerance of the oracle's float64 product.  So the full
    product's columns are pinned to the oracle through exact equalities."""
    import torch
    from apsi_b200 import kernels as Kn
    from apsi_b200._lib import FMT_INT4_G128
    g = torch.Generator(device=cuda)
    g.manual_seed(M * 7 + N)
    W = torch.randn((N, K), generator=g, device=cuda) * 0.015
    codes, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
    xf = torch.randn((M, K), generator=g, device=cuda)
    if M == 2048:                                        # configs[2]-style outliers in the prefill activations
        xf = torch.where(torch.rand((M, K), generator=g, device=cuda) < 1e-3, xf * 20, xf)
    x = xf.to(torch.bfloat16)
    full = Kn.linear(FMT_INT4_G128, x, codes, s16, N)
    torch.cuda.synchronize()
    xn = x.float().cpu().numpy()
    R = 512
    for r0 in (0, (N // 2 // 128) * 128, N - R):
        rows = W[r0:r0 + R].cpu().numpy()
        o_codes, _, o_s16 = O.quant_int4_g128(rows)
        c_rows, s_rows = codes[r0:r0 + R].contiguous(), s16[r0:r0 + R].contiguous()
        assert np.array_equal(c_rows.cpu().numpy(), o_codes), r0
        assert np.array_equal(s_rows.cpu().numpy().view(np.uint16), o_s16.view(np.uint16)), r0
        part = Kn.linear(FMT_INT4_G128, x, c_rows, s_rows, R)
        assert torch.equal(part, full[:, r0:r0 + R]), r0
        _check(part.float().cpu().numpy(), O.linear_ref(xn, O.dequant_int4_g128(o_codes, o_s16)))
    assert Kn.device_errors() == 0


def test_repeat_calls_are_deterministic(cuda):
    x, codes, s16, _ = _case(16, 3000, 8192, seed=9, fmt="int4")
    a = _run(cuda, "int4", x, codes, s16, 3000)
    b = _run(cuda, "int4", x, codes, s16, 3000)
    np.testing.assert_array_equal(a, b)


def test_large_activation_rows_are_exact_after_power_of_two_rescale(cuda):
    """Rows far outside the fp16 range (and tiny rows) go through the power-of-two rescale exactly."""
    M, N, K = 20, 256, 1024
    x, codes, s16, Wd = _case(M, N, K, seed=2, fmt="int4")
    x[0] *= 2.0 ** 40
    x[1] *= 2.0 ** -40
    x = O.bf16_round(x)
    y = _run(cuda, "int4", x, codes, s16, N)
    ref = O.linear_ref(x, Wd)
    for r in range(M):
        _check(y[r:r + 1], ref[r:r + 1])
    xg = x[:4]
    yg = _run(cuda, "int4", xg, codes, s16, N)                 # the same rows through the GEMV
    ref = O.linear_ref(xg, Wd)
    for r in range(4):
        _check(yg[r:r + 1], ref[r:r + 1])


def test_static_weight_overlap_waits_for_the_activations(cuda):
    """With LB_LINEAR_STATIC_WEIGHTS the GEMV starts streaming weights before the previous kernel ends; the
    activations written by that previous kernel must still be the ones used."""
    import torch
    from apsi_b200 import kernels as Kn
    from apsi_b200._lib import FMT_INT4_G128
    g = torch.Generator(device=cuda)
    g.manual_seed(21)
    N, K = 11008, 4096
    W = torch.randn((N, K), generator=g, device=cuda) * 0.02
    codes, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
    base = torch.randn((4, K), generator=g, device=cuda)
    ref = []
    for i in range(4):
        x = (base[i:i + 1] * (i + 1)).to(torch.bfloat16)
        ref.append(Kn.linear(FMT_INT4_G128, x, codes, s16, N))
    torch.cuda.synchronize()
    xs = torch.empty((1, K), dtype=torch.bfloat16, device=cuda)
    outs = []
    for i in range(4):
        torch.mul(base[i:i + 1], i + 1, out=xs.float()) if False else xs.copy_((base[i:i + 1] * (i + 1)))
        outs.append(Kn.linear(FMT_INT4_G128, xs, codes, s16, N, static_weights=True))
    torch.cuda.synchronize()
    for a, b in zip(ref, outs):
        assert torch.equal(a, b)


def test_qmatmul_fast_path_matches_general_path(cuda):
    """precision.qmatmul's per-call fast path (a contiguous bf16 CUDA matrix, M <= 16) gives the same bits as
    the general path (a 3-D input), with and without ``out``, and follows a replaced codes tensor."""
    import torch
    from apsi_b200 import precision as P
    rng = np.random.default_rng(44)
    W = torch.from_numpy((rng.standard_normal((1000, 1024)) * 0.02).astype(np.float32)).to(cuda)
    q = P.quantize(W, "int4", axis=0, group=128)
    x = torch.from_numpy(rng.standard_normal((5, 1024)).astype(np.float32)).to(cuda).to(torch.bfloat16)
    y_fast = P.qmatmul(x, q)
    y_gen = P.qmatmul(x.unsqueeze(0), q)[0]
    assert torch.equal(y_fast, y_gen)
    out = torch.empty((5, 1000), dtype=torch.bfloat16, device=cuda)
    assert P.qmatmul(x, q, out=out) is out and torch.equal(out, y_gen)
    q2 = P.quantize(W * 2, "int4", axis=0, group=128)
    q.codes, q.scale16 = q2.codes, q2.scale16                # replaced tensors: the cached spec is rebuilt
    assert torch.equal(P.qmatmul(x, q), P.qmatmul(x.unsqueeze(0), q2)[0])


def test_prepared_weight_gives_the_bits_of_linear_ex(cuda):
    """lb_weight_linear (a weight checked once, tensor maps encoded once) against lb_linear_ex on the same
    inputs: identical bits for int4 (box and row-copy paths) and int8, with and without static weights; M above
    16 is refused."""
    import torch
    from apsi_b200 import kernels as Kn, _lib
    from apsi_b200._lib import FMT_INT4_G128, FMT_INT8_ROW
    g = torch.Generator(device=cuda)
    g.manual_seed(8)
    for fmt, N, K in [(FMT_INT4_G128, 1000, 1024), (FMT_INT4_G128, 11008, 4096), (FMT_INT4_G128, 300, 11008),
                      (FMT_INT8_ROW, 520, 1024)]:
        W = torch.randn((N, K), generator=g, device=cuda) * 0.02
        codes, s16, _ = (Kn.quant_int4_g128 if fmt == FMT_INT4_G128 else Kn.quant_int8_rows)(W, want_scale32=False)
        pw = Kn.PreparedWeight(fmt, codes.data_ptr(), s16.data_ptr(), N, K, cuda.index or 0)
        for M in (1, 2, 3, 8, 16):
            x = torch.randn((M, K), generator=g, device=cuda).to(torch.bfloat16)
            ref = Kn.linear(fmt, x, codes, s16, N)
            for static in (False, True):
                spec = (fmt, codes.data_ptr(), s16.data_ptr(), N, K, cuda.index or 0, pw)
                y = Kn.linear_spec(spec, x, None, static)
                torch.cuda.synchronize()
                assert torch.equal(y, ref), (fmt, N, K, M, static)
        x = torch.randn((17, K), generator=g, device=cuda).to(torch.bfloat16)
        y = torch.empty((17, N), dtype=torch.bfloat16, device=cuda)
        rc = _lib.load().lb_weight_linear(pw.ptr, x.data_ptr(), 17, y.data_ptr(), N, 0,
                                          torch.cuda.current_stream(cuda).cuda_stream)
        assert rc == _lib.LB_E_UNSUPPORTED
    assert Kn.device_errors() == 0


def test_qmatmul_streams_settled_weights_early(cuda):
    """From a QTensor's second decode product on, precision.qmatmul launches with static weights (the weight
    stream starts before the previous kernel ends): same bits as the first, plain launch; after an in-place
    rewrite of the weights, touch() makes the next product wait for the writer again."""
    import torch
    from apsi_b200 import precision as P
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    W1 = torch.randn((3000, 4096), generator=g, device=cuda) * 0.02
    W2 = torch.randn((3000, 4096), generator=g, device=cuda) * 0.02
    x = torch.randn((2, 4096), generator=g, device=cuda).to(torch.bfloat16)
    q = P.quantize(W1, "int4", axis=0, group=128)
    assert not q._settled
    y1 = P.qmatmul(x, q)
    assert q._settled
    assert torch.equal(P.qmatmul(x, q), y1)
    q2 = P.quantize(W2, "int4", axis=0, group=128)
    q.codes.copy_(q2.codes)
    q.scale16.copy_(q2.scale16)
    q.touch()
    y2 = P.qmatmul(x, q)
    assert torch.equal(y2, P.qmatmul(x, q2))
