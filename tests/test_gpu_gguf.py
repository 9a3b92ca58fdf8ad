"""GGUF Q8_0 / Q4_0 block bytes on the GPU, byte for byte against the reference's own writer (golden vectors
from apsi.modelio._q8_0 / _q4_0) and against the oracle on seeded inputs with ties."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def test_blocks_match_reference_golden(cuda, golden):
    from apsi_b200 import modelio as MIO
    G = golden["gguf_w"]
    assert np.array_equal(np.frombuffer(MIO.gguf_q8_0(G), np.uint8), golden["gguf_q8_0"])
    assert np.array_equal(np.frombuffer(MIO.gguf_q4_0(G), np.uint8), golden["gguf_q4_0"])
    np.testing.assert_array_equal(MIO.gguf_dequant(golden["gguf_q8_0"].tobytes(), "q8_0", G.size), golden["gguf_dq8_0"])
    np.testing.assert_array_equal(MIO.gguf_dequant(golden["gguf_q4_0"].tobytes(), "q4_0", G.size), golden["gguf_dq4_0"])


@pytest.mark.parametrize("n,std", [(32 * 1000, 0.05), (32 * 37, 3.0), (32, 1e-3)])
def test_random_blocks_match_oracle(cuda, n, std):
    import torch
    from apsi_b200 import kernels as K
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * std).astype(np.float32)
    x[:32] = 0.0                                                   # an all-zero block (d = 0, inverse 0)
    if n >= 96:
        x[32:64] = np.float32(0.25) * (np.arange(32, dtype=np.float32) - 16)   # scaled values on half-integers
        x[64:96] = -x[64:96]
    xt = torch.from_numpy(x).to(cuda)
    for kind, fn in ((8, O.gguf_q8_0), (4, O.gguf_q4_0)):
        b = K.gguf_encode(xt, kind)
        ref = fn(x)
        np.testing.assert_array_equal(b.cpu().numpy(), ref)
        d = K.gguf_decode(b, kind, n).cpu().numpy()
        np.testing.assert_array_equal(d, O.gguf_dequant(ref, "q8_0" if kind == 8 else "q4_0", n))
