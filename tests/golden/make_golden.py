"""Write the golden vectors that pin the oracle and the kernels to the reference.

Run in a container where the reference is importable (its ``apsi`` package on ``APSI_REF`` or
``/root/reference``):

    python tests/golden/make_golden.py

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
    root = os.environ.get("APSI_REF", "/root/reference")
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

    path = os.path.join(HERE, "lowbit_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
