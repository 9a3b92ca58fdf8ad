"""A quantized decoder whose every projection runs on this library's kernels.

It follows the layer sequence of the reference's GPU decoder (``hub_models.Decoder._forward_gpu``,
apsi/hub_models.py:1018-1092), one block per layer:

    QKV  = linear(qkv, X, ln=ln1)            fused [(nh + 2 kvh) dh, H] projection after RMSNorm
    q, k, v = split(QKV); rope(q, k); write k, v into the cache        (qkv_prep)
    O    = attention(q, cache)                                           (attention)
    X   += linear(o, O)                                                  (o projection, residual add)
    GU   = linear(gu, X, ln=ln2)             fused [2 I, H] gate/up projection after RMSNorm
    X   += linear(down, silu(G) * U)                                     (act_mul, down projection)
    logits = linear(head, X_last, ln=final_norm)

All projections -- QKV, O, gate/up, down and the LM head -- are int4 group-128 (or int8, fp8 e4m3 or fp4 e2m1
per-row) weights in the library's packed layout, multiplied by ``kernels.linear``: the decode GEMV for up to 16 rows, the tcgen05
GEMM above; the residual adds are the kernels' accumulate epilogue.  The normalised projections (QKV,
gate/up, head) go through ``kernels.linear_rms``: for decode the RMSNorm runs inside the GEMV's activation
staging, for prefill ``lb_rmsnorm`` precedes the GEMM (the same bits either way).  The QKV split with rotary
embedding and the cache write (``lb_qkv_prep``) and the SwiGLU product (``lb_act_mul``) are the library's
kernels too.  Embedding lookup and attention over the KV cache are torch operations (attention is not
on the quantized-linear path this library rebuilds).  Activations are bf16; the KV cache is bf16.

Weights are random (seeded, N(0, 0.02) projections, unit norms), as configs[3] specifies; there is no
checkpoint.  ``generate`` prefills a batch of prompts and then decodes greedily, one CUDA-graph replay per
step (static shapes: attention over the whole cache capacity with a position mask).
"""
import math
import time
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import kernels as Kn
from ._lib import FMT_INT4_G128, FMT_INT8_ROW, FMT_FP8_E4M3, FMT_FP4_E2M1, LowbitError, LB_E_ARG

__all__ = ["DecoderConfig", "QuantDecoder", "KVCache"]


@dataclass
class DecoderConfig:
    """Llama-style shapes; the defaults are configs[3] (a 7B-class decoder)."""
    H: int = 4096          # hidden size
    L: int = 32            # layers
    nh: int = 32           # attention heads
    kvh: int = 8           # key/value heads
    dh: int = 128          # head size
    I: int = 11008         # SwiGLU width
    V: int = 32000         # vocabulary
    eps: float = 1e-5
    theta: float = 10000.0
    wstd: float = 0.02


class KVCache:
    """Keys and values of every layer: [L, B, kvh, cap, dh] bf16."""

    def __init__(self, cfg, batch, cap, device):
        self.cap, self.batch = cap, batch
        shape = (cfg.L, batch, cfg.kvh, cap, cfg.dh)
        self.k = torch.zeros(shape, dtype=torch.bfloat16, device=device)
        self.v = torch.zeros(shape, dtype=torch.bfloat16, device=device)


class _Proj:
    """One packed projection: codes and fp16 scales of [N, K] in the kernel layout."""
    __slots__ = ("fmt", "codes", "scales", "N", "K")

    def __init__(self, W, fmt):
        self.N, self.K = W.shape
        self.fmt = fmt
        if fmt == FMT_INT4_G128:
            self.codes, self.scales, _ = Kn.quant_int4_g128(W, want_scale32=False)
        elif fmt == FMT_INT8_ROW:
            self.codes, self.scales, _ = Kn.quant_int8_rows(W, want_scale32=False)
        else:                                    # fp8 / fp4 rows: float32 row scales
            self.codes, self.scales = Kn.quant_minifloat(W, fmt, True)

    def __call__(self, x, out=None, accumulate=False, static=False, ln=None, eps=1e-6):
        if ln is not None:                       # RMSNorm prologue (inside the decode GEMV for M <= 16)
            return Kn.linear_rms(self.fmt, x, ln, self.codes, self.scales, self.N, eps=eps, out=out,
                                 accumulate=accumulate, static_weights=static)
        return Kn.linear(self.fmt, x, self.codes, self.scales, self.N, out=out, accumulate=accumulate,
                         static_weights=static)

    def dequantized(self):
        if self.fmt in (FMT_INT4_G128, FMT_INT8_ROW):
            return Kn.dequant(self.fmt, self.codes, self.scales, self.N, self.K)
        return Kn.dequant_minifloat(self.fmt, self.codes, self.N, self.K, self.scales)


class QuantDecoder:
    """The decoder of configs[3] with packed low-bit projections (see the module docstring)."""

    _FMTS = {"int4": FMT_INT4_G128, "int8": FMT_INT8_ROW, "fp8_e4m3": FMT_FP8_E4M3, "fp4_e2m1": FMT_FP4_E2M1}

    def __init__(self, cfg=None, device="cuda", fmt="int4", seed=0, max_positions=8192):
        self._setup(cfg or DecoderConfig(), device, fmt, max_positions)
        cfg = self.cfg
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        width = (cfg.nh + 2 * cfg.kvh) * cfg.dh

        def proj(n, k):
            W = torch.randn((n, k), generator=g, device=self.dev) * cfg.wstd
            p = _Proj(W, self.fmt)
            del W
            return p

        self.embed = (torch.randn((cfg.V, cfg.H), generator=g, device=self.dev) * cfg.wstd * 50).to(torch.bfloat16)
        self.layers = []
        for _ in range(cfg.L):
            self.layers.append({
                "ln1": torch.ones(cfg.H, dtype=torch.bfloat16, device=self.dev),
                "qkv": proj(width, cfg.H),
                "o": proj(cfg.H, cfg.nh * cfg.dh),
                "ln2": torch.ones(cfg.H, dtype=torch.bfloat16, device=self.dev),
                "gu": proj(2 * cfg.I, cfg.H),
                "down": proj(cfg.H, cfg.I),
            })
        self.norm = torch.ones(cfg.H, dtype=torch.bfloat16, device=self.dev)
        self.head = proj(cfg.V, cfg.H)

    def _setup(self, cfg, device, fmt, max_positions):
        self.cfg = cfg
        self.dev = torch.device(device)
        if fmt not in self._FMTS:
            raise LowbitError(LB_E_ARG, f"projection format '{fmt}' is not one of {sorted(self._FMTS)}")
        self.fmt = self._FMTS[fmt]
        half = cfg.dh // 2
        inv = 1.0 / (cfg.theta ** (torch.arange(half, device=self.dev, dtype=torch.float64) / half))
        self._inv = inv.float()                                        # rotary frequencies
        ang = torch.arange(max_positions, device=self.dev, dtype=torch.float64)[:, None] * inv[None, :]
        self._cos = torch.cos(ang).float().contiguous()                # [positions, dh / 2]
        self._sin = torch.sin(ang).float().contiguous()
        self.max_positions = max_positions

    @classmethod
    def from_weights(cls, hf_cfg, W, device="cuda", fmt="int4", max_positions=None):
        """The decoder of a Llama-family checkpoint: ``hf_cfg`` its config.json as a dict, ``W`` its weights by
        Hugging Face name ([out, in] arrays or tensors), read as the reference's ``hub_models.Decoder`` reads
        them (apsi/hub_models.py:537-563; q/k/v and gate/up fused as its ``_groups``, :572-585).  The
        projections are quantised to ``fmt`` by this library's kernels; norms and embeddings are kept in
        bfloat16.  Variants the kernels here do not cover (Gemma's norm offset, q/k norms, projection biases,
        partial rotary, rope scaling, sliding windows, GPT-2) are refused."""
        import numpy as np
        c = dict(hf_cfg)
        t = c.get("model_type", "llama")
        unsupported = [k for k in ("rope_scaling", "sliding_window", "partial_rotary_factor") if c.get(k)]
        if t.startswith("gemma") or t == "gpt2" or unsupported:
            raise LowbitError(LB_E_ARG, f"decoder variant not covered: model_type {t} {unsupported}")
        if any(k.endswith(("q_norm.weight", "k_norm.weight", "_proj.bias")) for k in W):
            raise LowbitError(LB_E_ARG, "q/k norms and projection biases are not covered")
        H = int(c["hidden_size"])
        nh = int(c["num_attention_heads"])
        kvh = int(c.get("num_key_value_heads") or nh)
        dh = int(c.get("head_dim") or H // nh)
        emb = W["model.embed_tokens.weight"]
        cfg = DecoderConfig(H=H, L=int(c["num_hidden_layers"]), nh=nh, kvh=kvh, dh=dh,
                            I=int(c["intermediate_size"]), V=int(emb.shape[0]), eps=float(c.get("rms_norm_eps", 1e-6)),
                            theta=float(c.get("rope_theta", 10000.0)))
        self = cls.__new__(cls)
        self._setup(cfg, device, fmt, max_positions or int(c.get("max_position_embeddings", 4096)))

        def dev32(a):
            return torch.as_tensor(np.asarray(a, np.float32) if not isinstance(a, torch.Tensor) else a,
                                   dtype=torch.float32).to(self.dev).contiguous()

        def proj(*names):
            return _Proj(torch.cat([dev32(W[n]) for n in names], 0), self.fmt)

        def vec(n):
            return dev32(W[n]).to(torch.bfloat16)

        self.embed = dev32(emb).to(torch.bfloat16)
        self.layers = []
        for i in range(cfg.L):
            p = f"model.layers.{i}."
            self.layers.append({
                "ln1": vec(p + "input_layernorm.weight"),
                "qkv": proj(p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight"),
                "o": proj(p + "self_attn.o_proj.weight"),
                "ln2": vec(p + "post_attention_layernorm.weight"),
                "gu": proj(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"),
                "down": proj(p + "mlp.down_proj.weight"),
            })
        self.norm = vec("model.norm.weight")
        self.head = proj("lm_head.weight" if "lm_head.weight" in W else "model.embed_tokens.weight")
        return self

    # ------------------------------------------------------------------ pieces
    def weight_bytes(self):
        def nb(p):
            return p.codes.numel() * p.codes.element_size() + p.scales.numel() * p.scales.element_size()
        return sum(nb(p) for Ld in self.layers for p in (Ld["qkv"], Ld["o"], Ld["gu"], Ld["down"])) + nb(self.head)

    def new_cache(self, batch, cap):
        if cap > self.max_positions:
            raise LowbitError(LB_E_ARG, f"a cache of {cap} positions exceeds max_positions ({self.max_positions})")
        return KVCache(self.cfg, batch, cap, self.dev)

    def _block(self, i, X, B, T, cache, pos, start, mask):
        """One layer on X [B*T, H] (updated in place); pos [T] positions, start: first cache slot (int) or None
        when pos is a device tensor (decode, captured)."""
        cfg, Ld = self.cfg, self.layers[i]
        M = B * T
        static = M <= 16
        qkv = Ld["qkv"](X, static=static, ln=Ld["ln1"], eps=cfg.eps)
        kc, vc = cache.k[i], cache.v[i]                                # [B, kvh, cap, dh]
        q = torch.empty((B, cfg.nh, T, cfg.dh), dtype=torch.bfloat16, device=self.dev)
        Kn.qkv_prep(qkv, B, T, cfg.nh, cfg.kvh, cfg.dh, cfg.dh, self._cos, self._sin, q, kc, vc,
                    pos0=(pos if start is None else None), start=(start or 0))
        if start is not None:
            keys, vals = kc[:, :, :start + T], vc[:, :, :start + T]
            attn = F.scaled_dot_product_attention(q, keys, vals, is_causal=(start == 0 and T > 1), enable_gqa=True)
        else:                                                          # decode: T == 1, pos is a device tensor
            attn = F.scaled_dot_product_attention(q, kc, vc, attn_mask=mask, enable_gqa=True)
        o_in = attn.transpose(1, 2).reshape(M, cfg.nh * cfg.dh).contiguous()
        Ld["o"](o_in, out=X, accumulate=True, static=static)
        gu = Ld["gu"](X, static=static, ln=Ld["ln2"], eps=cfg.eps)
        m = Kn.act_mul(gu, cfg.I, 0)
        Ld["down"](m, out=X, accumulate=True, static=static)

    def _logits(self, X_last):
        return self.head(X_last.contiguous(), static=X_last.shape[0] <= 16, ln=self.norm, eps=self.cfg.eps)

    # ------------------------------------------------------------------ forward passes
    def prefill(self, ids, cache, all_positions=False):
        """ids [B, T] -> logits [B, V] of the last position (all_positions: [B, T, V]); fills cache slots
        [0, T)."""
        B, T = ids.shape
        X = self.embed.index_select(0, ids.reshape(-1)).contiguous()   # [B*T, H]
        pos = torch.arange(T, device=self.dev)
        for i in range(self.cfg.L):
            self._block(i, X, B, T, cache, pos, 0, None)
        if all_positions:
            return self._logits(X).view(B, T, -1)
        return self._logits(X.view(B, T, -1)[:, -1])

    def decode_step(self, tok, cache, pos_t):
        """tok [B] int64, pos_t [1] int64 (device) -> logits [B, V]; writes cache slot pos_t."""
        B = tok.shape[0]
        X = self.embed.index_select(0, tok).contiguous()
        # additive mask, built once per step (a boolean mask would be converted in every layer's attention)
        mask = torch.zeros((1, 1, 1, cache.cap), dtype=torch.bfloat16, device=self.dev)
        mask.masked_fill_(torch.arange(cache.cap, device=self.dev) > pos_t, float("-inf"))
        for i in range(self.cfg.L):
            self._block(i, X, B, 1, cache, pos_t, None, mask)
        return self._logits(X)

    def generate(self, ids, steps, graph=True):
        """Greedy decoding: prefill ids [B, T], then `steps` tokens.  Returns (tokens [B, steps], timings)."""
        B, T = ids.shape
        cache = self.new_cache(B, T + steps)
        torch.cuda.synchronize(self.dev)
        t0 = time.perf_counter()
        logits = self.prefill(ids, cache)
        tok = logits.float().argmax(-1)
        torch.cuda.synchronize(self.dev)
        t1 = time.perf_counter()
        out = torch.empty((B, steps), dtype=torch.int64, device=self.dev)
        tok_buf = tok.clone()
        pos_buf = torch.full((1,), T, dtype=torch.int64, device=self.dev)
        g = None
        if graph and steps > 0:
            s = torch.cuda.Stream(device=self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(s):                      # warm the kernels' lazy setup outside capture
                self.decode_step(tok_buf, self.new_cache(B, T + steps), pos_buf)
            torch.cuda.current_stream(self.dev).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                logits_buf = self.decode_step(tok_buf, cache, pos_buf)
                next_tok = logits_buf.float().argmax(-1)
        torch.cuda.synchronize(self.dev)
        t2 = time.perf_counter()
        for s_ in range(steps):
            if g is not None:
                g.replay()
                out[:, s_] = next_tok
                tok_buf.copy_(next_tok)
            else:
                lg = self.decode_step(tok_buf, cache, pos_buf)
                nt = lg.float().argmax(-1)
                out[:, s_] = nt
                tok_buf.copy_(nt)
            pos_buf += 1
        torch.cuda.synchronize(self.dev)
        t3 = time.perf_counter()
        del g
        return out, {"prefill_s": t1 - t0, "decode_s": t3 - t2, "capture_s": t2 - t1,
                     "prefill_tokens": B * T, "decode_tokens": B * steps}
