"""The quantized decoder (apsi_b200.decoder): every projection on the library's kernels, checked against a
float32 torch restatement of the same network on the dequantised weights, and the cached decode step checked
against a prefill of the longer sequence.  A small configuration; configs[3] itself is timed by bench.py."""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

SMALL = dict(H=256, L=2, nh=4, kvh=2, dh=64, I=512, V=1000)


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm())


def _reference_logits(model, ids):
    """float32 restatement: the same blocks with dequantised weights, no bf16 rounding of activations."""
    cfg = model.cfg
    B, T = ids.shape

    def rms(x, w):
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + cfg.eps) * w.float()

    def rope(t, pos):
        h = cfg.dh // 2
        ang = pos.float()[:, None] * model._inv
        cos, sin = torch.cos(ang)[None, :, None, :], torch.sin(ang)[None, :, None, :]
        a, b = t[..., :h], t[..., h:]
        return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)

    X = model.embed.index_select(0, ids.reshape(-1)).float().view(B, T, -1)
    pos = torch.arange(T, device=ids.device)
    for Ld in model.layers:
        qkv = rms(X, Ld["ln1"]) @ Ld["qkv"].dequantized().T
        q, k, v = qkv.split([cfg.nh * cfg.dh, cfg.kvh * cfg.dh, cfg.kvh * cfg.dh], dim=-1)
        q = rope(q.reshape(B, T, cfg.nh, cfg.dh), pos).transpose(1, 2)
        k = rope(k.reshape(B, T, cfg.kvh, cfg.dh), pos).transpose(1, 2)
        v = v.reshape(B, T, cfg.kvh, cfg.dh).transpose(1, 2)
        rep = cfg.nh // cfg.kvh
        k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        s = (q @ k.transpose(-1, -2)) / math.sqrt(cfg.dh)
        s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool, device=ids.device), 1), float("-inf"))
        o = (s.softmax(-1) @ v).transpose(1, 2).reshape(B, T, -1)
        X = X + o @ Ld["o"].dequantized().T
        gu = rms(X, Ld["ln2"]) @ Ld["gu"].dequantized().T
        g_, u_ = gu.split(cfg.I, dim=-1)
        X = X + (F.silu(g_) * u_) @ Ld["down"].dequantized().T
    return rms(X[:, -1], model.norm) @ model.head.dequantized().T


@pytest.mark.parametrize("fmt", ["int4", "int8", "fp8_e4m3", "fp4_e2m1"])
def test_prefill_matches_float32_restatement(cuda, fmt):
    from apsi_b200.decoder import QuantDecoder, DecoderConfig
    model = QuantDecoder(DecoderConfig(**SMALL), device=cuda, fmt=fmt, seed=3)
    ids = torch.randint(0, SMALL["V"], (3, 40), device=cuda, generator=torch.Generator(device=cuda).manual_seed(1))
    cache = model.new_cache(3, 48)
    got = model.prefill(ids, cache)
    ref = _reference_logits(model, ids)
    assert got.shape == (3, SMALL["V"])
    assert _rel(got, ref) < 3e-2


@pytest.mark.parametrize("fmt", ["int4", "fp4_e2m1"])
def test_cached_decode_matches_longer_prefill(cuda, fmt):
    from apsi_b200.decoder import QuantDecoder, DecoderConfig
    from apsi_b200 import kernels
    model = QuantDecoder(DecoderConfig(**SMALL), device=cuda, fmt=fmt, seed=4)
    ids = torch.randint(0, SMALL["V"], (2, 21), device=cuda, generator=torch.Generator(device=cuda).manual_seed(2))
    cache = model.new_cache(2, 32)
    model.prefill(ids[:, :20], cache)
    step = model.decode_step(ids[:, 20], cache, torch.tensor([20], device=cuda))
    full = model.prefill(ids, model.new_cache(2, 32))
    assert _rel(step, full) < 2e-2
    # greedy generation through the captured decode graph equals the uncaptured loop
    toks_g, _ = model.generate(ids[:, :8], 6, graph=True)
    toks_e, t = model.generate(ids[:, :8], 6, graph=False)
    assert torch.equal(toks_g, toks_e)
    assert t["decode_tokens"] == 12 and kernels.device_errors(cuda) == 0
