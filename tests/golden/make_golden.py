"""Write the golden vectors that pin the oracle and the kernels to the reference.

Run where the reference is importable; ``APSI_REF`` must name the directory that holds its ``apsi`` package:

    APSI_REF=<reference checkout> python tests/golden/make_golden.py

The outputs come from the reference's own functions -- ``apsi.precision.quantize`` / ``dequantize`` /
``qmatmul``, ``apsi.hub_gpu.qnumpy``, ``apsi.lowbit.round_weights`` and, for ``ref_packed.apsim``,
``apsi.modelio.save_model`` -- on seeded inputs, including adversarial ones (exact half-way ties,
near-ties one ulp either side, all-zero groups, signed zeros, subnormals, single outliers).  The arrays are
small so the fixture stays a few hundred KB.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _reference():
    root = os.environ.get("APSI_REF")
    if not root or not os.path.isdir(os.path.join(root, "apsi")):
        raise SystemExit("set APSI_REF to the directory that holds the reference's apsi package")
    sys.path.insert(0, root)
    from apsi import precision, hub_gpu  # noqa: E402
    return precision, hub_gpu


def _reference_lowbit():
    from apsi import lowbit  # noqa: E402  (after _reference() put the reference on the path)
    return lowbit


def _adversarial_rows(rng, K, qmax):
    """Rows whose quotients land exactly on, and one ulp beside, half-integers."""
    rows = []
    s = np.float32(2.0 ** -4)                      # a scale that is exact as m / qmax
    m = np.float32(s * qmax)
    # exact ties k + 0.5 for every k in range, plus the absmax
    ks = np.arange(-qmax, qmax, dtype=np.float64) + 0.5
    base = np.resize(ks * float(s), K).astype(np.float32)
    base[0] = m
    rows.append(base)
    up = np.nextafter(base, np.float32(np.inf))
    up[0] = m
    rows.append(up)
    dn = np.nextafter(base, np.float32(-np.inf))
    dn[0] = m
    rows.append(dn)
    rows.append(np.zeros(K, np.float32))                                         # all-zero -> scale 1.0
    z = np.zeros(K, np.float32)
    z[1::2] = -0.0
    z[5] = np.float32(3e-3)
    rows.append(z)                                                               # signed zeros + one value
    rows.append((rng.standard_normal(K) * 1e-41).astype(np.float32))             # subnormals
    rows.append((rng.standard_normal(K) * 1e-30).astype(np.float32))             # tiny normals
    o = (rng.standard_normal(K) * 0.02).astype(np.float32)
    o[::37] *= 300.0
    rows.append(o)                                                               # single outliers
    rows.append((rng.standard_normal(K) * 1e4).astype(np.float32))               # large values
    r = (rng.integers(-qmax, qmax + 1, K) * float(s)).astype(np.float32)
    r[0] = m
    rows.append(r)                                                               # exact multiples
    return np.stack(rows)


def main():
    precision, hub_gpu = _reference()
    rng = np.random.default_rng(20261201)
    out = {}

    # ---- int4 with groups of 128 (precision.quantize on [-1, 128] rows, axis=0)
    K4 = 512
    W4 = np.concatenate([(rng.standard_normal((24, K4)) * 0.02).astype(np.float32),
                         _adversarial_rows(rng, K4, 7)])
    q = precision.quantize(W4.reshape(-1, 128), "int4", axis=0)
    out["w4"] = W4
    out["w4_packed"] = np.asarray(q.codes, np.uint8).reshape(W4.shape[0], K4 // 2)
    out["w4_scale32"] = np.asarray(q.scale, np.float32).reshape(W4.shape[0], K4 // 128)
    out["w4_deq32"] = np.asarray(precision.dequantize(q), np.float32).reshape(W4.shape)

    # ---- int8 with one scale per output row (precision.quantize(W, "int8", axis=0))
    K8 = 384
    W8 = np.concatenate([(rng.standard_normal((24, K8)) * 0.02).astype(np.float32),
                         _adversarial_rows(rng, K8, 127)])
    q8 = precision.quantize(W8, "int8", axis=0)
    out["w8"] = W8
    out["w8_codes"] = np.asarray(q8.codes, np.uint8).view(np.int8).reshape(W8.shape)
    out["w8_scale32"] = np.asarray(q8.scale, np.float32).reshape(-1)
    out["w8_deq32"] = np.asarray(precision.dequantize(q8), np.float32)

    # ---- a product through the reference's own quantized matmul (dequantise + float32 matmul)
    x = rng.standard_normal((5, K4)).astype(np.float32)
    Wt = (rng.standard_normal((40, K4)) * 0.02).astype(np.float32)
    qt = precision.quantize(Wt.reshape(-1, 128), "int4", axis=0)
    out["mm_x"] = x
    out["mm_w"] = Wt
    out["mm_y_qmatmul"] = np.asarray(precision.qmatmul(x, precision.dequantize(qt).reshape(Wt.shape).T),
                                     np.float32)

    # ---- ggml-style blocks of 32 (hub_gpu.qnumpy), both kinds
    Wg = np.concatenate([(rng.standard_normal((16, 256)) * 0.05).astype(np.float32),
                         _adversarial_rows(rng, 256, 7)])
    out["wg"] = Wg
    for kind in ("int8", "int4"):
        qv, sc = hub_gpu.qnumpy(Wg, kind)
        out[f"wg_{kind}_q"] = np.asarray(qv, np.float32)
        out[f"wg_{kind}_scale"] = np.asarray(sc, np.float32)

    # ---- lowbit.round_weights (rows = outputs, blocks of 32 along the inputs, padded) on an [in, out] weight
    # whose input size is not a multiple of 32, with tiny, zero and exactly representable columns
    lowbit = _reference_lowbit()
    n_in, n_out = 70, 24
    Wr = (rng.standard_normal((n_in, n_out)) * 0.05).astype(np.float32)
    Wr[:, 3] *= 1e-4
    Wr[:, 5] = 0.0
    Wr[:, 7] = np.tile(np.array([0.5, -0.25, 1.75, 7.0, -8.0], np.float32), 14)[:n_in]
    out["rw_in"] = Wr
    for kind in ("int8", "int4"):
        out[f"rw_{kind}"] = np.asarray(lowbit.round_weights(Wr, kind), np.float32)

    # ---- a checkpoint written by the reference's own save_model (apsi/modelio.py:417-463): an int4
    # group-128 layer stored the reference's way (W.reshape(-1, 128), axis 0), an int8 per-row layer, a bias
    # and a norm vector.  The source arrays go into the npz so the loaded codes can be checked bit for bit.
    from apsi import modelio  # noqa: E402
    w4 = (rng.standard_normal((48, 384)) * 0.02).astype(np.float32)
    w8 = (rng.standard_normal((40, 256)) * 0.02).astype(np.float32)
    b4 = (rng.standard_normal(48) * 0.1).astype(np.float32)
    nv = np.ones(384, np.float32)
    out["apsim_w4"], out["apsim_w8"], out["apsim_b4"], out["apsim_norm"] = w4, w8, b4, nv
    tree = {"proj": {"W": precision.quantize(w4.reshape(-1, 128), "int4", axis=0), "b": b4},
            "down": {"W": precision.quantize(w8, "int8", axis=0)}, "norm": nv}
    apsim = os.path.join(HERE, "ref_packed.apsim")
    modelio.save_model(apsim, tree, metadata={"written_by": "apsi.modelio.save_model"})
    print("wrote", apsim)

    # ---- minifloat formats (precision.quantize with scale="auto"): per row (axis=0) and per tensor (axis=None).
    # Rows whose absmax is the format's largest value are quantised with scale 1.0 exactly, so they carry exact
    # grid midpoints (ties), values one float32 ulp beside them, subnormal-range values and signed zeros; a row
    # with a NaN (scale 1.0, other values saturate), a row with an infinity (scale inf), an all-zero row, and
    # seeded normal rows.
    for name in ("fp8_e4m3", "fp8_e5m2", "fp6_e3m2", "fp6_e2m3", "fp4_e2m1"):
        f = precision.get_format(name)
        vals = np.asarray(f.sorted_vals, np.float64)
        mids = (vals[:-1] + vals[1:]) / 2.0
        C = 96
        rows = []
        for arr in (mids, np.nextafter(mids.astype(np.float32), np.float32(np.inf)),
                    np.nextafter(mids.astype(np.float32), np.float32(-np.inf)), vals):
            r = np.resize(np.asarray(arr, np.float64), C)
            r[1::3] *= -1.0
            r[0] = f.max
            rows.append(r.astype(np.float32))
        z = np.zeros(C, np.float32)
        z[1::2] = -0.0
        z[0] = f.max
        z[3] = np.float32(vals[1] / 3.0)                    # below half the smallest subnormal
        z[4] = np.float32(vals[1] / 2.0)                    # exactly half of it (tie with zero)
        rows.append(z)
        nanrow = (rng.standard_normal(C) * 3 * f.max).astype(np.float32)
        nanrow[7] = np.nan
        rows.append(nanrow)
        infrow = (rng.standard_normal(C)).astype(np.float32)
        infrow[11] = -np.inf
        rows.append(infrow)
        rows.append(np.zeros(C, np.float32))
        for _ in range(6):
            rows.append((rng.standard_normal(C) * 0.02).astype(np.float32))
        o = (rng.standard_normal(C) * 0.02).astype(np.float32)
        o[::17] *= 200.0
        rows.append(o)
        Wm = np.stack(rows)
        q = precision.quantize(Wm, name, axis=0)
        out[f"mf_{name}_w"] = Wm
        out[f"mf_{name}_codes"] = np.asarray(q.codes, np.uint8).reshape(-1)
        out[f"mf_{name}_scale"] = np.asarray(q.scale, np.float32).reshape(-1)
        out[f"mf_{name}_deq"] = np.asarray(precision.dequantize(q), np.float32)
        Wt = (rng.standard_normal((7, 37)) * 0.3).astype(np.float32)          # odd sizes: packing runs across rows
        Wt[2, 5] = -0.0
        qt = precision.quantize(Wt, name)
        out[f"mf_{name}_t_w"] = Wt
        out[f"mf_{name}_t_codes"] = np.asarray(qt.codes, np.uint8).reshape(-1)
        out[f"mf_{name}_t_scale"] = np.asarray([qt.scale], np.float64)
        out[f"mf_{name}_t_deq"] = np.asarray(precision.dequantize(qt), np.float32)

    # ---- GGUF Q8_0 / Q4_0 block bytes (apsi/modelio.py:56-95): seeded blocks, ties at half-integers of the
    # scaled values, an all-zero block, a block whose largest magnitude is negative
    from apsi import modelio as _mio  # noqa: E402
    G = (rng.standard_normal((6, 128)) * 0.05).astype(np.float32)
    G[1, :32] = 0.0
    G[2, :32] = np.linspace(-1.0, 0.5, 32, dtype=np.float32)
    G[3, 32:64] = (np.arange(32, dtype=np.float32) - 16.0) * np.float32(0.125) + np.float32(0.0625)
    out["gguf_w"] = G
    out["gguf_q8_0"] = np.frombuffer(_mio._q8_0(G), np.uint8).copy()
    out["gguf_q4_0"] = np.frombuffer(_mio._q4_0(G), np.uint8).copy()
    out["gguf_dq8_0"] = np.asarray(_mio._dq8_0(out["gguf_q8_0"].tobytes(), G.size), np.float32)
    out["gguf_dq4_0"] = np.asarray(_mio._dq4_0(out["gguf_q4_0"].tobytes(), G.size), np.float32)

    path = os.path.join(HERE, "lowbit_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items()})


def precision_api(precision, path=None):
    """Golden values of the precision module's metrics and tables (``round_to``, ``quant_error``,
    ``format_info``, ``module``; apsi/precision.py:278-339) on seeded inputs, in precision_api_golden.npz."""
    rng = np.random.default_rng(20261202)
    x = (rng.standard_normal((24, 256)) * 0.05).astype(np.float32)
    x[3, :] = 0.0                                        # an all-zero row (scale 1.0)
    x[5, 17] = 2.5                                       # an outlier
    out = {"x": x}
    cases = [("int8", 0), ("fp8_e4m3", 0), ("fp8_e5m2", 0), ("fp6_e3m2", 0), ("fp6_e2m3", 0), ("fp4_e2m1", 0),
             ("fp8_e4m3", None), ("fp4_e2m1", None)]
    for fmt, axis in cases:
        tag = f"{fmt}_{'row' if axis == 0 else 'tensor'}"
        out["round_to_" + tag] = np.asarray(precision.round_to(x, fmt, "auto", axis), np.float64)
        out["quant_error_" + tag] = np.float64(precision.quant_error(x, fmt, axis))
    g = x.reshape(-1, 128)                               # int4 in groups of 128: the reference's own spelling
    out["round_to_int4_g128"] = np.asarray(precision.round_to(g, "int4", "auto", 0), np.float64).reshape(x.shape)
    out["quant_error_int4_g128"] = np.float64(precision.quant_error(g, "int4", 0))
    names = ["int8", "int4", "fp8_e4m3", "fp8_e5m2", "fp6_e3m2", "fp6_e2m3", "fp4_e2m1", "f64", "f32", "f16",
             "bf16", "uint8"]
    info = np.zeros((len(names), 5), np.float64)
    for i, n in enumerate(names):
        r = precision.format_info(n)
        info[i] = [r.bits, r.max, r.eps, r.tiny, getattr(r, "values", -1)]
    out["format_info_names"] = np.array(names)
    out["format_info"] = info
    funcs = [k for k, v in precision.module().items() if callable(v) and k in
             ("quantize", "dequantize", "round_to", "qmatmul", "nbytes", "quant_error", "format_info")]
    out["module_functions"] = np.array(sorted(funcs))
    path = path or os.path.join(HERE, "precision_api_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


def hub_cpu_q8(path=None):
    """Golden outputs of the reference's fastest CPU product (``apsi.hub_cpu``: ``Q8.from_bf16`` and ``matmul``
    on a Q8, apsi/hub_cpu.py:170-194, 474-534) on seeded bfloat16 weights, in hub_q8_golden.npz.  They pin
    the C restatement ``oracle/hub_q8.c`` that bench.py times as the CPU baseline."""
    from apsi import hub_cpu  # noqa: E402  (after _reference() put the reference on the path)
    if not hub_cpu.q8_available():
        raise SystemExit("the reference's native Q8 product is not available here")
    rng = np.random.default_rng(3202)
    out = {}
    for tag, (O, I, T) in {"a": (300, 512, 3), "b": (256, 1024, 1), "c": (64, 2048, 16)}.items():
        W = (rng.standard_normal((O, I)) * 0.02).astype(np.float32)
        W[7, :64] = 0.0                                  # an all-zero block (scale 0, codes 0)
        bits = (W.view(np.uint32) >> np.uint32(16)).astype(np.uint16)       # bfloat16 by truncation
        q = hub_cpu.Q8.from_bf16(bits)
        x = rng.standard_normal((T, I)).astype(np.float32)
        if tag == "a":                                   # the quantiser's input, for the Q8_0 code check
            out[f"{tag}_wbits"] = bits
        out[f"{tag}_codes"], out[f"{tag}_scales"] = q.codes, q.scales
        out[f"{tag}_x"] = x
        out[f"{tag}_y"] = np.asarray(hub_cpu.matmul(x, q), np.float32)
    path = path or os.path.join(HERE, "hub_q8_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


def decoder_logits(path=None):
    """Golden logits of the reference's decoder (``apsi.hub_models.Decoder.forward`` on its processor path,
    apsi/hub_models.py:1150-1200, the layer sequence its GPU path runs too) on the int4-g128-exact weights of
    tiny_decoder.py: the logits of a prompt, then of four tokens fed one at a time through the cache, in
    decoder_golden.npz with a checksum of the weights."""
    from apsi import hub_models  # noqa: E402  (after _reference() put the reference on the path)
    sys.path.insert(0, HERE)
    import tiny_decoder as TD
    W = TD.weights()
    dec = hub_models.Decoder(dict(TD.CFG), W)
    ids = TD.token_ids()
    cache = dec.new_cache()
    out = {"ids": ids, "checksum": np.float64(TD.checksum(W)),
           "prompt_logits": np.asarray(dec.forward(np.array([ids[:TD.PROMPT]]), cache, 0)[0], np.float32)}
    steps = []
    for j in range(TD.PROMPT, TD.PROMPT + TD.DECODE):
        steps.append(np.asarray(dec.forward(np.array([[ids[j]]]), cache, j, last=True)[0, -1], np.float32))
    out["decode_logits"] = np.stack(steps)
    path = path or os.path.join(HERE, "decoder_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


def layers_trace(path=None):
    """The reference's transformer_lm forward (apsi/layers.py:1999-2008; Linear.apply and the attention / SwiGLU
    blocks all multiply as ``x @ W``) with every projection weight replaced by its int4-g128 dequantisation
    (the oracle's quantisation of W.T: rows = outputs, groups of 128 along the inputs).  Each weight is wrapped
    so that the forward's own ``x @ W`` expressions defer to it (``__array_ufunc__ = None``, the hook this
    library's QTensor uses); every call's input and output is recorded, in call order, with the packed codes and
    fp16 scales of its weight and the final logits, in layers_trace_golden.npz."""
    from apsi import layers as Ly  # noqa: E402  (after _reference() put the reference on the path)
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    import oracle as O
    model = Ly.transformer_lm(256, d=128, heads=4, layers=1, context=16, rope=True, norm="rms", ffn="swiglu",
                              ff=256)
    params = model.init(0)
    calls = []

    class Traced:
        __array_ufunc__ = None

        def __init__(self, W, name):
            packed, _, s16 = O.quant_int4_g128(np.ascontiguousarray(np.asarray(W, np.float32).T))
            self.name, self.packed, self.s16 = name, packed, s16
            self.Wd = O.dequant_int4_g128(packed, s16).T.astype(np.float64)      # [in, out]
            self.shape, self.ndim = self.Wd.shape, 2

        def __rmatmul__(self, x):
            y = np.asarray(x) @ self.Wd
            calls.append((self.name, np.asarray(x, np.float32), np.asarray(y, np.float32)))
            return y

    out = {}
    blk = params[1][0]
    targets = [(blk.attn.inner.fields, k) for k in ("Wq", "Wk", "Wv", "Wo")] + \
              [(blk.mlp.inner.fields, k) for k in ("Wg", "Wu", "Wd")] + [(params[2].fields, "W")]
    for f, k in targets:
        t = Traced(f[k], "head" if k == "W" else k)
        f[k] = t
        out[f"w_{t.name}_packed"], out[f"w_{t.name}_s16"] = t.packed, t.s16.view(np.uint16)
    ids = np.random.default_rng(5).integers(0, 256, size=(2, 8))
    out["ids"] = ids
    out["logits"] = np.asarray(model(params, ids, train=False), np.float32)
    out["call_names"] = np.array([c[0] for c in calls])
    for i, (_, x, y) in enumerate(calls):
        out[f"call{i}_x"], out[f"call{i}_y"] = x, y
    path = path or os.path.join(HERE, "layers_trace_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, len(calls), "calls")


if __name__ == "__main__":
    main()
    precision_api(_reference()[0])
    hub_cpu_q8()
    decoder_logits()
    layers_trace()
