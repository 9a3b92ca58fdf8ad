"""Size-independent properties of the oracle's restatements, beside the golden vectors that pin them: the
minifloat grids are fixed points of encode / decode, every value rounds to a grid neighbour, the fp4 / fp6 /
int4 packings round-trip, and the GGUF blocks reproduce their values within their step.  These are
checked on the CPU, for every format."""
import numpy as np
import pytest

from oracle import lowbit_oracle as ora

NAMES = ("fp8_e4m3", "fp8_e5m2", "fp6_e3m2", "fp6_e2m3", "fp4_e2m1")


@pytest.mark.parametrize("name", NAMES)
def test_every_finite_grid_value_is_a_fixed_point(name):
    t = ora.minifloat_table(name)
    eb, mb = ora.MINIFLOATS[name][:2]
    for sign in (1.0, -1.0):
        mags = np.flatnonzero(np.isfinite(t))
        codes = ora.minifloat_encode(name, sign * t[mags])
        back = ora.minifloat_decode(name, codes)
        assert np.array_equal(back, (sign * t[mags]).astype(np.float32))
        assert np.all(((codes.astype(np.int64) >> (eb + mb)) & 1) == (1 if sign < 0 else 0))


@pytest.mark.parametrize("name", NAMES)
def test_encode_picks_a_nearest_grid_value(name):
    rng = np.random.default_rng(len(name))
    mx = ora.minifloat_max(name)
    y = rng.uniform(-1.2 * mx, 1.2 * mx, 20000)
    v = ora.minifloat_decode(name, ora.minifloat_encode(name, y)).astype(np.float64)
    grid = np.sort(np.unique(np.abs(ora.minifloat_table(name)[np.isfinite(ora.minifloat_table(name))])))
    a = np.minimum(np.abs(y), mx)                          # saturation above the largest finite value
    i = np.clip(np.searchsorted(grid, a), 1, grid.size - 1)
    best = np.minimum(np.abs(grid[i] - a), np.abs(grid[i - 1] - a))
    assert np.all(np.abs(np.abs(v) - a) <= best + 1e-12)
    assert np.all((np.sign(v) == np.sign(y)) | (v == 0))


@pytest.mark.parametrize("n", [1, 3, 4, 5, 64, 1001])
def test_fp6_and_int4_packings_round_trip(n):
    rng = np.random.default_rng(n)
    c6 = rng.integers(0, 64, n).astype(np.uint8)
    p6 = ora.pack6(c6)
    assert p6.size == 3 * ((n + 3) // 4)
    assert np.array_equal(ora.unpack6(p6, n), c6)
    c4 = rng.integers(-8, 8, n).astype(np.int8)
    p4 = ora.pack4(c4)
    assert p4.size == (n + 1) // 2
    assert np.array_equal(ora.unpack4(p4, n), c4)


@pytest.mark.parametrize("std", [1e-3, 0.02, 3.0])
def test_gguf_blocks_reproduce_values_within_their_step(std):
    """Q8_0 rounds to the nearest of 255 steps of amax / 127 (half a step of error); Q4_0 uses steps of amax / 8
    with codes clipped at 15, so values near +amax opposite a negative maximum lose up to a whole step.  Both
    carry the binary16 rounding of the block scale times the largest code."""
    rng = np.random.default_rng(int(std * 1000) + 1)
    x = (rng.standard_normal(32 * 64) * std).astype(np.float32)
    for kind, enc, steps, frac in (("q8_0", ora.gguf_q8_0, 127.0, 0.5), ("q4_0", ora.gguf_q4_0, 8.0, 1.0)):
        buf = enc(x)
        assert buf.size == 64 * (34 if kind == "q8_0" else 18)
        y = ora.gguf_dequant(buf, kind, x.size).reshape(-1, 32)
        amax = np.abs(x.reshape(-1, 32)).max(axis=1, keepdims=True)
        step = amax / steps
        tol = frac * step + amax * 2.0 ** -9 + 1e-30
        assert np.all(np.abs(y - x.reshape(-1, 32)) <= tol), kind
        assert np.all(np.abs(y).max(axis=1) <= amax[:, 0] * (1 + 2.0 ** -9)), kind


def test_int4_g128_codes_and_scales_bound_the_weights():
    rng = np.random.default_rng(5)
    W = (rng.standard_normal((16, 512)) * 0.05).astype(np.float32)
    packed, s32, s16 = ora.quant_int4_g128(W)
    codes = ora.unpack4(packed.reshape(-1), W.size).reshape(16, 512)
    assert codes.min() >= -8 and codes.max() <= 7
    g = np.abs(W.reshape(16, 4, 128)).max(axis=2)
    assert np.allclose(s32, g / 7.0, rtol=1e-6)
    d = ora.dequant_int4_g128(packed, s16)
    assert np.all(np.abs(d - W) <= np.repeat(s16.astype(np.float32), 128, axis=1) * 0.5 + 1e-3 * g.max())
