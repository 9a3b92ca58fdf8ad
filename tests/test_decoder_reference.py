"""The decoder on this library's kernels against logits the reference's own decoder computed.

tests/golden/decoder_golden.npz holds the logits of ``apsi.hub_models.Decoder.forward`` (the reference's
Llama-family decoder, apsi/hub_models.py:1150-1200) for a prompt and for four tokens fed one at a time through
its cache, on the weights of tests/golden/tiny_decoder.py.  Those projections are exactly int4 with one scale
per 128 values, so ``QuantDecoder.from_weights`` (int4-g128 kernels for every projection, the library's RMSNorm,
RoPE/cache and SwiGLU kernels) multiplies the same weights; the difference is the bfloat16 activations and
cache against the reference's float32.  Bound: max-abs error <= 2e-2 * max|logit| per position, and the same
top token wherever the reference's top two logits are more than that apart."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import tiny_decoder as TD  # noqa: E402

GOLD = os.path.join(HERE, "golden", "decoder_golden.npz")
TOL = 2e-2


def test_the_weight_generator_matches_the_golden_run():
    g = np.load(GOLD)
    assert np.array_equal(g["ids"], TD.token_ids())
    assert float(g["checksum"]) == TD.checksum(TD.weights())


def _close(got, ref, what):
    for j in range(ref.shape[0]):
        err = np.abs(got[j] - ref[j]).max()
        assert err <= TOL * np.abs(ref[j]).max(), f"{what} position {j}: max error {err:.3e}"
        top2 = np.sort(ref[j])[-2:]
        if top2[1] - top2[0] > 2 * TOL * np.abs(ref[j]).max():
            assert int(np.argmax(got[j])) == int(np.argmax(ref[j])), f"{what} position {j}: top token differs"


@pytest.mark.gpu
def test_quant_decoder_matches_the_reference_decoder(cuda):
    import torch
    from apsi_b200 import kernels
    from apsi_b200.decoder import QuantDecoder
    g = np.load(GOLD)
    model = QuantDecoder.from_weights(TD.CFG, TD.weights(), device=cuda, fmt="int4")
    # the int4-g128 codes of every projection reproduce the weights exactly
    W = TD.weights()
    wq = torch.from_numpy(W["model.layers.0.self_attn.o_proj.weight"]).to(cuda)
    assert torch.equal(model.layers[0]["o"].dequantized().float(), wq)
    ids = torch.from_numpy(g["ids"]).to(cuda).view(1, -1)
    P = TD.PROMPT
    cache = model.new_cache(1, P + TD.DECODE)
    logits = model.prefill(ids[:, :P], cache, all_positions=True)[0].float().cpu().numpy()
    _close(logits, g["prompt_logits"], "prompt")
    steps = []
    for j in range(P, P + TD.DECODE):
        pos = torch.full((1,), j, dtype=torch.int64, device=cuda)
        steps.append(model.decode_step(ids[:, j], cache, pos)[0].float().cpu().numpy())
    _close(np.stack(steps), g["decode_logits"], "decode")
    assert kernels.device_errors(cuda) == 0
