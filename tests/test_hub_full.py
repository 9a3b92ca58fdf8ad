"""The whole-decoder ops object (``apsi_b200.hub.Ops``, ``full = True``) driven through the call sequence of the
reference's GPU decoder pass (``hub_models.Decoder._forward_gpu``, apsi/hub_models.py:1018-1092, restated below
as test code), on the weights of tests/golden/tiny_decoder.py, against the logits the reference's decoder
computed for them (tests/golden/decoder_golden.npz).  The projections go through the int4-g128 kernels
(``qmatrix(w, "int4")``), the norms are float32 weights, the cache holds bfloat16: max-abs error
<= 2e-2 * max|logit| per position."""
import math
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import tiny_decoder as TD  # noqa: E402

GOLD = os.path.join(HERE, "golden", "decoder_golden.npz")
TOL = 2e-2


def _upload(r, W, cfg):
    """The reference's _upload_full for an int4 model (hub_models.py:807-836), restated."""
    layers = []
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        qkv = np.concatenate([W[p + f"self_attn.{x}_proj.weight"] for x in "qkv"], 0)
        layers.append({"qkv": r.qmatrix(qkv, "int4"), "o": r.qmatrix(W[p + "self_attn.o_proj.weight"], "int4"),
                       "gu": r.qmatrix(np.concatenate([W[p + "mlp.gate_proj.weight"], W[p + "mlp.up_proj.weight"]], 0),
                                       "int4"),
                       "down": r.qmatrix(W[p + "mlp.down_proj.weight"], "int4"),
                       "ln1": r.vec(W[p + "input_layernorm.weight"]), "ln2": r.vec(W[p + "post_attention_layernorm.weight"]),
                       "I": W[p + "mlp.down_proj.weight"].shape[1]})
    return layers, r.vec(W["model.norm.weight"]), r.qmatrix(W["lm_head.weight"], "int4")


class _Cache:
    """_GpuCache (hub_models.py:1389-1440) at a fixed capacity: K / V per layer and the RoPE tables."""

    def __init__(self, r, cfg, cap):
        H, nh = cfg["hidden_size"], cfg["num_attention_heads"]
        kvh, dh = cfg["num_key_value_heads"], H // nh
        self.cap = cap
        self.K = [r.alloc_kv(kvh * cap * dh, True) for _ in range(cfg["num_hidden_layers"])]
        self.V = [r.alloc_kv(kvh * cap * dh, True) for _ in range(cfg["num_hidden_layers"])]
        inv = 1.0 / cfg["rope_theta"] ** (np.arange(0, dh, 2, dtype=np.float64) / dh)
        f = np.outer(np.arange(cap), inv)
        self.cos, self.sin = r.alloc(f.size), r.alloc(f.size)
        r.put(self.cos, np.cos(f).astype(np.float32).reshape(-1))
        r.put(self.sin, np.sin(f).astype(np.float32).reshape(-1))


def _forward(r, W, cfg, layers, norm, head, cache, ids, s0, last):
    """One pass of _forward_gpu (hub_models.py:1044-1087) over ids at cache position s0."""
    H, nh = cfg["hidden_size"], cfg["num_attention_heads"]
    kvh, dh = cfg["num_key_value_heads"], H // nh
    width, eps, V = (nh + 2 * kvh) * dh, cfg["rms_norm_eps"], head.rows
    T = len(ids)
    X = r.ws("x", T * H)
    r.put(X, W["model.embed_tokens.weight"][ids].reshape(-1))
    QKV, Q, O = r.ws("qkv", T * width), r.ws("q", T * nh * dh), r.ws("o", T * nh * dh)
    S = r.ws("s", nh * T * (s0 + T))
    for i, Ld in enumerate(layers):
        I = Ld["I"]
        GU, M = r.ws("gu", T * 2 * I), r.ws("m", T * I)
        r.linear(Ld["qkv"], X, QKV, T, ln=Ld["ln1"], eps=eps, off=0.0)
        r.qkv_prep(QKV, Q, cache.K[i], cache.V[i], cache.cos, cache.sin, None, None, T, nh, kvh, dh, dh, s0,
                   cache.cap, eps, half=True)
        r.attention(Q, cache.K[i], cache.V[i], O, S, T, nh, kvh, dh, s0, cache.cap, None, 1.0 / math.sqrt(dh),
                    half=True)
        r.linear(Ld["o"], O, X, T, acc=True)
        r.linear(Ld["gu"], X, GU, T, ln=Ld["ln2"], eps=eps, off=0.0)
        r.act_mul(GU, M, T, I, 0)
        r.linear(Ld["down"], M, X, T, acc=True)
    rows, first = (1, T - 1) if last else (T, 0)
    LOG = r.ws("log", rows * V)
    r.linear(head, X, LOG, rows, ln=norm, eps=eps, off=0.0, xoff=first * H)
    return r.get(LOG, rows * V).reshape(rows, V)


def _close(got, ref, what):
    for j in range(ref.shape[0]):
        err = np.abs(got[j] - ref[j]).max()
        assert err <= TOL * np.abs(ref[j]).max(), f"{what} position {j}: max error {err:.3e}"


def test_ops_reports_the_whole_decoder_interface():
    from apsi_b200 import hub
    assert hub.Ops.full is True
    for name in ("qmatrix", "matrix", "upload", "linear", "rms", "embed", "qkv_prep", "attention", "act_mul",
                 "alloc", "alloc_kv", "copy_kv", "copy", "free", "put", "get", "ws", "vec", "begin", "close",
                 "sample_prep", "free_memory", "trim", "gemv", "gemm", "matmul", "matmul_rows"):
        assert callable(getattr(hub.Ops, name)), name


@pytest.mark.gpu
def test_ops_runs_the_reference_decoder_sequence(cuda):
    from apsi_b200 import hub, kernels
    g = np.load(GOLD)
    W, cfg = TD.weights(), TD.CFG
    r = hub.Ops(0)
    layers, norm, head = _upload(r, W, cfg)
    cache = _Cache(r, cfg, 64)
    ids = g["ids"]
    P = TD.PROMPT
    _close(_forward(r, W, cfg, layers, norm, head, cache, ids[:P], 0, last=False), g["prompt_logits"], "prompt")
    steps = [_forward(r, W, cfg, layers, norm, head, cache, ids[j:j + 1], j, last=True)[0]
             for j in range(P, P + TD.DECODE)]
    _close(np.stack(steps), g["decode_logits"], "decode")
    # sampling helper: the greedy candidate is the top logit
    LOG = r.ws("log", head.rows)
    SEEN = r.ws("seen", head.rows)
    r.put(SEEN, np.zeros(head.rows, np.float32))
    gmax, Z, cand, vals, count = r.sample_prep(LOG, SEEN, head.rows, 1.0, 1.0, 0.0, 8)
    assert count >= 1 and int(cand[0]) == int(np.argmax(steps[-1])) and Z >= 1.0
    # a tied head: the embedding table as a dense bf16 matrix, embed() gathers its rows
    emb = r.matrix(W["model.embed_tokens.weight"])
    X = r.ws("xe", 3 * cfg["hidden_size"])
    r.embed(emb, ids[:3], X)
    want = TD._bf16(W["model.embed_tokens.weight"][ids[:3]]).reshape(-1)
    assert np.array_equal(r.get(X, want.size), want)
    assert kernels.device_errors(cuda) == 0
    r.close()
