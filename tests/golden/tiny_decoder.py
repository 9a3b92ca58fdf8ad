"""A small Llama-style decoder whose projections are exactly representable in int4 with one power-of-two scale per
128 values (test infrastructure).

Every projection row is built group by group: codes q in [-7, 7] (each group holds a +7 or a -7) times 2^e, so
``quantize(W.reshape(-1, 128), "int4", axis=0)`` (the g128 layout) recovers q and 2^e exactly, and the same values
are exact in bfloat16.  The reference's decoder (``apsi.hub_models.Decoder``) multiplying W in float32 and this
library's int4 kernels multiplying the codes therefore use the same weights; only the activations' rounding
differs.  ``make_golden.decoder_logits`` runs the reference on these weights; ``tests/test_decoder_reference.py``
runs ``apsi_b200.decoder.QuantDecoder`` on them.
"""
import numpy as np

CFG = {"model_type": "llama", "hidden_size": 256, "num_attention_heads": 4, "num_key_value_heads": 2,
       "num_hidden_layers": 2, "intermediate_size": 512, "rms_norm_eps": 1e-6, "rope_theta": 10000.0,
       "max_position_embeddings": 64, "tie_word_embeddings": False, "hidden_act": "silu", "vocab_size": 384}
SEED = 20261202
PROMPT = 12          # prompt positions, then one token at a time
DECODE = 4


def _int4_exact(rng, n, k):
    q = rng.integers(-7, 8, size=(n, k // 128, 128))
    pick = rng.integers(0, 128, size=(n, k // 128))
    sign = np.where(rng.random((n, k // 128)) < 0.5, -7, 7)
    np.put_along_axis(q, pick[..., None], sign[..., None], axis=2)
    e = rng.integers(-10, -6, size=(n, k // 128, 1))
    return (q * np.exp2(e)).reshape(n, k).astype(np.float32)


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    u = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return u.view(np.float32)


def weights():
    """HF-named float32 weights of the decoder (projections int4-g128-exact, norms and embeddings bf16-exact)."""
    c = CFG
    rng = np.random.default_rng(SEED)
    H, nh, kvh, I, V = c["hidden_size"], c["num_attention_heads"], c["num_key_value_heads"], \
        c["intermediate_size"], c["vocab_size"]
    dh = H // nh
    W = {"model.embed_tokens.weight": _bf16(rng.standard_normal((V, H)) * 0.5),
         "model.norm.weight": _bf16(1 + rng.standard_normal(H) * 0.1),
         "lm_head.weight": _int4_exact(rng, V, H)}
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}."
        W[p + "input_layernorm.weight"] = _bf16(1 + rng.standard_normal(H) * 0.1)
        W[p + "post_attention_layernorm.weight"] = _bf16(1 + rng.standard_normal(H) * 0.1)
        W[p + "self_attn.q_proj.weight"] = _int4_exact(rng, nh * dh, H)
        W[p + "self_attn.k_proj.weight"] = _int4_exact(rng, kvh * dh, H)
        W[p + "self_attn.v_proj.weight"] = _int4_exact(rng, kvh * dh, H)
        W[p + "self_attn.o_proj.weight"] = _int4_exact(rng, H, nh * dh)
        W[p + "mlp.gate_proj.weight"] = _int4_exact(rng, I, H)
        W[p + "mlp.up_proj.weight"] = _int4_exact(rng, I, H)
        W[p + "mlp.down_proj.weight"] = _int4_exact(rng, H, I)
    return W


def token_ids():
    rng = np.random.default_rng(SEED + 1)
    return rng.integers(0, CFG["vocab_size"], size=PROMPT + DECODE)


def checksum(W):
    """A digest of the weights, stored with the golden logits so a drift of the generator is caught."""
    tot = np.float64(0)
    for k in sorted(W):
        a = W[k].astype(np.float64).reshape(-1)
        tot += np.dot(a, np.arange(1, a.size + 1, dtype=np.float64) % 97)
    return tot
