"""precision.round_to, quant_error, format_info and module (apsi/precision.py:278-339) against values the
reference computed (tests/golden/precision_api_golden.npz, written by tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

from apsi_b200 import precision as P

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "precision_api_golden.npz")


@pytest.fixture(scope="module")
def gold():
    return dict(np.load(GOLD))


def test_format_info_matches_the_reference_table(gold):
    for name, row in zip(gold["format_info_names"], gold["format_info"]):
        info = P.format_info(str(name))
        bits, mx, eps, tiny, values = row
        assert info["name"] == str(name)
        assert info["bits"] == bits and info["max"] == mx and info["eps"] == eps and info["tiny"] == tiny, name
        if values >= 0:
            assert info["values"] == values, name
        else:
            assert "values" not in info
    assert P.format_info("fp8")["name"] == "fp8_e4m3" and P.format_info("bf8")["name"] == "fp8_e5m2"


def test_module_exposes_the_reference_functions(gold):
    mod = P.module()
    for name in gold["module_functions"]:
        assert callable(mod[str(name)]), name
    assert mod["quantize_linear"] is P.quantize_linear


def test_unknown_format_raises_the_reference_error():
    with pytest.raises(P.RuntimeErr, match="unknown numeric format"):
        P.format_info("int3")
    with pytest.raises(P.RuntimeErr, match="not on the B200 low-bit path"):
        P.round_to(np.ones((4, 8), np.float32), "bf16")


CASES = [("int8", 0), ("fp8_e4m3", 0), ("fp8_e5m2", 0), ("fp6_e3m2", 0), ("fp6_e2m3", 0), ("fp4_e2m1", 0),
         ("fp8_e4m3", None), ("fp4_e2m1", None)]


@pytest.mark.gpu
@pytest.mark.parametrize("fmt,axis", CASES)
def test_round_to_and_quant_error_match_the_reference(cuda, gold, fmt, axis):
    tag = f"{fmt}_{'row' if axis == 0 else 'tensor'}"
    x = gold["x"]
    r = P.round_to(x, fmt, "auto", axis)
    assert r.dtype == np.float64 and r.shape == x.shape
    assert np.array_equal(r, gold["round_to_" + tag]), tag
    e = P.quant_error(x, fmt, axis)
    assert e == pytest.approx(float(gold["quant_error_" + tag]), rel=1e-12, abs=0.0)


@pytest.mark.gpu
def test_round_to_and_quant_error_int4_groups_match_the_reference(cuda, gold):
    x = gold["x"]
    g = x.reshape(-1, 128)
    r = P.round_to(g, "int4", "auto", 0).reshape(x.shape)
    assert np.array_equal(r, gold["round_to_int4_g128"])
    assert np.array_equal(P.round_to(x, "int4", "auto", 0, group=128), gold["round_to_int4_g128"])
    assert P.quant_error(g, "int4", 0) == pytest.approx(float(gold["quant_error_int4_g128"]), rel=1e-12, abs=0.0)


@pytest.mark.gpu
def test_nbytes_counts_codes_and_scales(cuda, gold):
    x = gold["x"]
    q = P.quantize(x, "int4", axis=0, group=128)
    assert P.nbytes(q) == q.nbytes and P.nbytes(x) == x.nbytes
