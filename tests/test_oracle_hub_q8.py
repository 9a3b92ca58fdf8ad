"""The C restatement of the reference's fastest CPU product (oracle/hub_q8.c: hub_cpu's Q8_0 GEMV on all cores)
against outputs the reference itself wrote (tests/golden/hub_q8_golden.npz, from apsi.hub_cpu): Q8_0 codes and
scales bit for bit, products to float32 rounding.  bench.py times this restatement as the CPU baseline."""
import os

import numpy as np
import pytest

from oracle import hub_q8

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "hub_q8_golden.npz")


@pytest.fixture(scope="module")
def gold():
    hub_q8.build()
    return dict(np.load(GOLD))


def test_q8_codes_and_scales_match_the_reference(gold):
    w = (gold["a_wbits"].astype(np.uint32) << np.uint32(16)).view(np.float32)
    codes, scales = hub_q8.q8_from_weights(w)
    assert np.array_equal(codes, gold["a_codes"])
    assert np.array_equal(scales.view(np.uint32), gold["a_scales"].view(np.uint32))


@pytest.mark.parametrize("tag", ["a", "b", "c"])
@pytest.mark.parametrize("threads", [1, 3, 0])
def test_q8_product_matches_the_reference(gold, tag, threads):
    y = hub_q8.matmul(gold[f"{tag}_x"], gold[f"{tag}_codes"], gold[f"{tag}_scales"], threads)
    ref = gold[f"{tag}_y"]
    assert y.shape == ref.shape
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()


def test_q8_product_runs_the_widest_kernel_the_cpu_has():
    isa = hub_q8.load().hub_q8_isa()
    assert isa in (0, 256, 512)
