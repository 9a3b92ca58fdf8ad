#!/usr/bin/env python
"""Benchmark of the B200 low-bit linear layer (the contract of this repository's bench).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Metric: int4-g128 weight-only GEMV weight GB/s at M=1, on configs[1] (x bf16 [1, 4096],
W [11008, 4096] ~ N(0, 0.02) quantised to int4 with fp16 absmax/7 scales per 128 values).

A step is one decode token through LAYERS = 128 resident, distinct int4-g128 weight matrices of that shape
(2.98 GB of packed weights -- the weight bytes of one decode step of the 7B-class decoder in configs[3]), so
every GEMV streams its weights from HBM (inputs are larger than L2; nothing is flushed).  The step is one
CUDA-graph replay of 128 GEMV launches.  ``value`` is packed weight bytes per second over all ranks.

N > 1 (torchrun): each rank holds the column shards of 128 layers that are N times as wide (weak scaling:
[11008, 4096] per rank per layer).  The gather is fused into the GEMVs: every rank's GEMV stores its columns
into every rank's full output over NVLink (CUDA IPC peer buffers), and one flag barrier ends the step, all
inside the timed CUDA graph.  An NCCL all-gather of the same outputs is timed on its own for comparison.

Also reported: the GEMV's live roofline (CUDA events on the launching stream), ``e2e`` through the public API
(``apsi_b200.precision.qmatmul``) from pinned host memory and back, the reference's fastest CPU path (hub_cpu's
Q8_0 GEMV on all host cores, restated in ``oracle/hub_q8.c``) as ``cpu_baseline``, the prefill GEMM of configs[2] (M=2048, N=12288, K=4096), and
``mlp70b``: the 70B-shaped MLP of configs[4] column-sharded over all ranks (strong scaling) at M = 1, 64 and
2048, with the per-rank products, the NCCL all-gathers and both together timed separately.
"""
import argparse
import json
import os
import re
import sys
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

METRIC = "int4-g128 W-only GEMV weight GB/s (M=1) & GEMM TFLOP/s (M=2048) vs roofline, 1–8 GPU"
M1, N1, K1 = 1, 11008, 4096          # configs[1]
LAYERS = 128
GM, GN, GK = 2048, 12288, 4096       # configs[2]
MLP_N, MLP_K = 28672, 8192           # configs[4]: gate/up [28672, 8192], down [8192, 28672]
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM, FALLBACK_TF = 6650.0, 1590.0


def gemv_bytes(M, N, K):
    """Algorithmic bytes of one int4-g128 GEMV: packed codes + fp16 scales + x + y."""
    return N * K // 2 + N * (K // 128) * 2 + M * K * 2 + M * N * 2


def weight_bytes(N, K):
    return N * K // 2 + N * (K // 128) * 2


def read_peaks():
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM, FALLBACK_TF, "fallback"


def read_traffic(name):
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) recorded by an ncu capture in
    profiles/<name>.md as a line 'traffic_bytes_per_launch: N' (None when absent)."""
    try:
        with open(os.path.join(HERE, "profiles", name + ".md")) as fh:
            m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)", fh.read())
        return float(m.group(1)) if m else None
    except OSError:
        return None


# ------------------------------------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML every `period` seconds in a thread."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting"}

    def __init__(self, index, period=0.002):
        self.samples = []
        self.period = period
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:                      # noqa: BLE001 - no NVML: report no clocks
            self.max_mhz = None
        self._stop = threading.Event()
        self._t = None

    def _sample(self):
        nv = self.nv
        try:
            sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
            try:
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:                  # noqa: BLE001
                rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
            self.samples.append((time.perf_counter(), sm, rs))
        except Exception:                      # noqa: BLE001
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()

    def summary(self, t0, t1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        if not win:                            # region shorter than the period: nearest samples
            win = sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
        mhz = [s[1] for s in win]
        bits = 0
        for s in win:
            bits |= s[2]
        reasons = [n for b, n in self.REASONS.items() if bits & b]
        return {"sm_mhz": float(np.median(mhz)) if mhz else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(win)}


# ------------------------------------------------------------------------------------------------ CPU baseline
def _q8_layer(M, seed=0):
    """configs[1]'s layer in the reference's Q8_0 CPU layout (bfloat16-rounded weights ~ N(0, 0.02)) and M
    float32 tokens."""
    import oracle as O
    from oracle import hub_q8
    rng = np.random.default_rng(seed)
    W = O.bf16_round((rng.standard_normal((N1, K1)) * 0.02).astype(np.float32))
    codes, scales = hub_q8.q8_from_weights(W)
    x = O.bf16_round(rng.standard_normal((M, K1)).astype(np.float32))
    return codes, scales, x


Q8_COPIES = 6          # distinct Q8_0 copies of the layer (6 x 50.7 MB): products stream from DRAM, not the L3


def _q8_layers(M):
    """Q8_COPIES distinct copies of configs[1]'s layer in Q8_0 (a decode step reads each layer once, so the
    CPU product must not be served from the host's last-level cache) and M tokens."""
    layers = [_q8_layer(M, seed=s)[:2] for s in range(Q8_COPIES)]
    return layers, _q8_layer(M)[2]


def time_hub_q8(M, reps, warmup=2, threads=0):
    """The reference's fastest CPU product (hub_cpu.matmul on Q8_0 weights, all cores), restated in
    oracle/hub_q8.c, on configs[1]'s [11008, 4096] layer at M tokens, rotating over Q8_COPIES copies: seconds
    per product (median of `reps`)."""
    from oracle import hub_q8
    layers, x = _q8_layers(M)
    for i in range(warmup):
        hub_q8.matmul(x, *layers[i % Q8_COPIES], threads)
    ts = []
    for i in range(reps):
        c, s_ = layers[i % Q8_COPIES]
        t0 = time.perf_counter()
        hub_q8.matmul(x, c, s_, threads)
        ts.append(time.perf_counter() - t0)
    return float(np.median(ts)), layers[0][0].nbytes + layers[0][1].nbytes


def cpu_baseline_sample():
    """cpu_baseline of our arm: the reference's fastest CPU path (hub_cpu's Q8_0 GEMV on all host cores,
    restated in C) on configs[1]'s layer at M=1, as configs[1]-layer-equivalent GB/s (the int4-g128 bytes of the
    same [11008, 4096] layer per second of the CPU product), plus the NumPy port of precision.qmatmul."""
    from oracle import hub_q8
    threads = hub_q8.host_threads()
    dt, q8_bytes = time_hub_q8(1, reps=200, threads=threads)
    import oracle as O
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((N1, K1)) * 0.02).astype(np.float32)
    packed, _, s16 = O.quant_int4_g128(W)
    x = O.bf16_round(rng.standard_normal((M1, K1)).astype(np.float32))
    O.qmatmul_dequant_reference(x, packed, s16, "int4_g128")        # warm
    t0 = time.perf_counter()
    O.qmatmul_dequant_reference(x, packed, s16, "int4_g128")
    dn = time.perf_counter() - t0
    return {"value": round(weight_bytes(N1, K1) / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"200 products of configs[1]'s [11008,4096] layer at M=1, rotating over {Q8_COPIES} distinct "
                      f"Q8_0 copies (weights from DRAM), through oracle/hub_q8.c, the C restatement of "
                      f"hub_cpu.matmul on Q8_0 weights (the reference's fastest CPU path; its thread team over "
                      f"{threads} threads): {dt * 1e3:.3f} ms per product, "
                      f"{q8_bytes / dt / 1e9:.1f} GB/s of Q8_0 bytes; value = int4-g128 bytes of the same layer "
                      f"per second",
            "numpy_qmatmul": {"ms_per_product": round(dn * 1e3, 1),
                              "value": round(weight_bytes(N1, K1) / dn / 1e9, 4),
                              "what": "oracle port of precision.qmatmul (dequantise + float32 BLAS), 1 product"}}


def run_reference(args, rank):
    """The reference arm: the reference's fastest CPU product for this layer -- hub_cpu.matmul on Q8_0 weights
    over all host cores (restated in oracle/hub_q8.c; the reference's own code cannot run on the GPU machines) --
    on configs[1]'s [11008, 4096] layer at M=1, one product per step.  ``value`` is configs[1]-layer-equivalent
    GB/s (the int4-g128 bytes of the same layer per second), so the ratio of the two arms is the ratio of their
    times per product; the Q8_0 byte rate is reported beside it, with M = 4 and 16."""
    if rank != 0:
        return 0
    from oracle import hub_q8
    threads = hub_q8.host_threads()
    layers, x = _q8_layers(M1)
    for i in range(max(args.warmup, 1)):
        hub_q8.matmul(x, *layers[i % Q8_COPIES], threads)
    ts = []
    for i in range(args.steps):
        c, s_ = layers[i % Q8_COPIES]
        t0 = time.perf_counter()
        hub_q8.matmul(x, c, s_, threads)
        ts.append(time.perf_counter() - t0)
    dt = float(np.sum(ts)) / args.steps
    val = weight_bytes(N1, K1) / dt / 1e9
    q8b = layers[0][0].nbytes + layers[0][1].nbytes
    per_m = {}
    for M in (4, 16):
        dm, _ = time_hub_q8(M, reps=max(5, args.steps // 4), threads=threads)
        per_m[f"M={M}"] = {"ms_per_product": round(dm * 1e3, 4), "value": round(weight_bytes(N1, K1) / dm / 1e9, 3),
                           "q8_weight_GB_per_s": round(q8b / dm / 1e9, 2)}
    sample = (f"one product of configs[1]'s [11008,4096] layer per step at M=1 (rotating over {Q8_COPIES} distinct "
              f"Q8_0 copies, so the weights come from DRAM) through oracle/hub_q8.c, the C restatement of "
              f"hub_cpu.matmul on Q8_0 weights with its thread team over {threads} threads")
    out = {"impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "GB/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int8xf32->f32", "data": "synthetic",
           "config": {"workload": "configs[1]: decode product M=1 of the [11008,4096] layer, one per step "
                                  "(value: int4-g128 bytes of that layer per second of the CPU product)",
                      "M": M1, "N": N1, "K": K1,
                      "path": "hub_cpu.matmul on Q8_0 (apsi/hub_cpu.py:96-194, 404-534), restated in C",
                      "q8_weight_GB_per_s": round(q8b / dt / 1e9, 2), "per_M": per_m},
           "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                            "sample": sample},
           "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)
    return 0


# ------------------------------------------------------------------------------------------------ our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from apsi_b200 import kernels as Kn
    from apsi_b200 import precision as P
    from apsi_b200 import sharded as S
    from apsi_b200._lib import FMT_INT4_G128

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    hbm_peak, tf_peak, peak_kind = read_peaks()

    # ---- resident inputs: LAYERS distinct weight shards, quantised on the device (not timed)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    packed, scales = [], []
    for _ in range(LAYERS):
        W = torch.randn((N1, K1), generator=gen, device=dev) * 0.02
        p, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
        packed.append(p)
        scales.append(s16)
        del W
    x = torch.randn((M1, K1), generator=gen, device=dev).to(torch.bfloat16)
    ys = torch.empty((LAYERS, M1, N1), dtype=torch.bfloat16, device=dev)
    gathered = torch.empty((world, LAYERS * M1, N1), dtype=torch.bfloat16, device=dev) if world > 1 else None
    # N > 1: every rank's full outputs [LAYERS * M1, N1 * world], written by all ranks' GEMVs (fused gather)
    peers = S.PeerOutputs(N1 * world, LAYERS * M1, dev) if world > 1 else None

    def sweep():
        if peers is None:
            for i in range(LAYERS):
                Kn.linear(FMT_INT4_G128, x, packed[i], scales[i], N1, out=ys[i], static_weights=True)
            return
        ldy = N1 * world
        for i in range(LAYERS):
            ptrs = [q + i * M1 * ldy * 2 for q in peers.ptrs[0]]
            Kn.linear_sharded(FMT_INT4_G128, x, packed[i], scales[i], N1, ptrs, rank, ldy, static_weights=True)
        Kn.rank_barrier(peers.ptrs[2], rank, 0, dev)       # epoch from the device counter: graph-safe

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        sweep()                                            # first use (device init, lazy setup) outside capture
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        sweep()
    torch.cuda.synchronize(dev)

    ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]

    def step(i=None):
        with torch.cuda.stream(stream):
            if i is not None:
                ev_a[i].record(stream)
            graph.replay()
            if i is not None:
                ev_b[i].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    clk = ClockSampler(local_rank)
    clk.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    t_start.record(stream)
    for i in range(args.steps):
        step(i)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    w1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    clk.stop()
    elapsed = t_start.elapsed_time(t_end)                  # ms
    gemv_ms = sum(a.elapsed_time(b) for a, b in zip(ev_a, ev_b))
    tt = torch.tensor([elapsed, gemv_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    elapsed, gemv_ms = float(tt[0]), float(tt[1])
    errs = Kn.device_errors(dev)

    wb_step = LAYERS * weight_bytes(N1, K1) * world
    value = wb_step * args.steps / (elapsed * 1e-3) / 1e9
    launch_s = gemv_ms * 1e-3 / (args.steps * LAYERS)
    achieved = gemv_bytes(M1, N1, K1) / launch_s / 1e9
    traffic = read_traffic("gemv_int4_m1_11008x4096")

    out = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(elapsed / args.steps, 5), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "int4xbf16->f32", "data": "synthetic",
           "config": {"workload": "configs[1]: int4-g128 decode GEMV, M=1, W[11008,4096] per rank, "
                                  f"{LAYERS} distinct resident weight matrices per step",
                      "M": M1, "N": N1 * world, "N_per_rank": N1, "K": K1, "layers_per_step": LAYERS,
                      "weight_bytes_per_step": wb_step, "l2": "inputs larger than L2 (no flush)",
                      "parallelism": f"column-shard x{world}" + (" + gather fused into the GEMVs (peer stores over "
                                                                 "NVLink) + flag barrier" if world > 1 else ""),
                      "graph": "one CUDA graph replay of the GEMV launches per step"},
           "roofline": {"kernel": "gemv_kernel<int4,1>", "bound": "hbm", "achieved": round(achieved, 1),
                        "peak": hbm_peak, "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                        "traffic": traffic, "peak_source": f"{peak_kind} hbm_gbs",
                        "algorithmic_bytes_per_launch": gemv_bytes(M1, N1, K1),
                        "avg_launch_us": round(launch_s * 1e6, 3)},
           "gpu_launches": args.steps * (LAYERS + (1 if world > 1 else 0)),
           "device_error_bits": errs}
    out["clocks"] = clk.summary(w0, w1)

    # ---- NCCL all-gather of the same outputs, alone (N > 1; the unfused alternative)
    if world > 1:
        torch.cuda.synchronize(dev)
        dist.barrier()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(5, args.steps)
        with torch.cuda.stream(stream):
            a0.record(stream)
            for _ in range(reps):
                dist.all_gather_into_tensor(gathered.view(-1), ys.view(-1))
            a1.record(stream)
        torch.cuda.synchronize(dev)
        ag = torch.tensor([a0.elapsed_time(a1) / reps], dtype=torch.float64, device=dev)
        dist.all_reduce(ag, op=dist.ReduceOp.MAX)
        per_rank = ys.numel() * 2 * (world - 1)
        out["allgather"] = {"what": "NCCL all_gather_into_tensor of one step's outputs (not on the timed path)",
                            "ms": round(float(ag), 4), "bytes_received_per_rank": per_rank,
                            "GB_per_s_per_rank": round(per_rank / (float(ag) * 1e-3) / 1e9, 2)}

    if world > 1:                          # layer 0's fused gather against an NCCL all-gather of the shards
        out["gather_bitexact"] = gather_check(
            torch, Kn, FMT_INT4_G128, dev, rank, world, [(packed[0], scales[0], N1, K1)], {K1: x}, [ys[0]],
            [torch.empty((world, M1, N1), dtype=torch.bfloat16, device=dev)],
            [(peers.ptrs[0], peers.ptrs[2], N1 * world, peers.view0(M1))], M1)

    # ---- e2e through the public API: pinned host x in, every layer's y back to pinned host memory
    qts = []
    for i in range(LAYERS):
        q = P.QTensor(packed[i], None, P.get_format("int4"), (N1, K1), 0, None, True, scale16=scales[i], group=128)
        qts.append(q)
    x_host = x.cpu().pin_memory()
    y_host = torch.empty((LAYERS, M1, N1), dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, min(args.steps, 20))

    def e2e_step():
        xd = x_host.to(dev, non_blocking=True)
        for i in range(LAYERS):
            P.qmatmul(xd, qts[i], out=ys[i])
        y_host.copy_(ys, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    et = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_s = float(et)
    out["e2e"] = {"value": round(wb_step / e2e_s / 1e9, 2), "unit": "GB/s",
                  "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": y_host.numel() * 2,
                  "api": "apsi_b200.precision.qmatmul per layer (one launch each, no graph)",
                  "ms_per_step": round(e2e_s * 1e3, 3)}

    # ---- prefill GEMM, configs[2] (rank 0 reports)
    out["gemm"] = gemm_measure(torch, Kn, FMT_INT4_G128, dev, tf_peak, peak_kind)

    # ---- the quantise / pack kernel (bandwidth-bound), configs[1]'s weight
    out["quant"] = quant_measure(torch, Kn, dev, hbm_peak, peak_kind)

    # ---- the 70B-shaped MLP, column-sharded over all ranks (strong scaling)
    out["mlp70b"] = mlp70b_measure(torch, Kn, FMT_INT4_G128, dev, rank, world, stream, hbm_peak, tf_peak, peak_kind)

    if world == 1:
        try:
            out["decoder"] = decoder_measure(torch, dev, hbm_peak)
        except Exception as e:               # noqa: BLE001
            out["decoder"] = {"error": f"{type(e).__name__}: {e}"}

    if rank == 0 and world == 1:
        try:
            out["cpu_baseline"] = cpu_baseline_sample()
        except Exception as e:               # noqa: BLE001
            out["cpu_baseline"] = {"value": None, "unit": "GB/s", "cores": None, "kind": "port",
                                   "sample": f"failed: {type(e).__name__}: {e}"}
    del graph
    if peers is not None:
        peers.close()
    if rank == 0:
        print(json.dumps(out), flush=True)
    return 0


def quant_measure(torch, Kn, dev, hbm_peak, peak_kind, reps=20):
    """lb_quant_int4_g128 on configs[1]'s [11008, 4096] weight from float32 and from bfloat16, rotating over
    weight copies larger than L2 together: algorithmic bytes (read the weight, write codes + fp16 scales) per
    second against the HBM peak.  The float32 scales are not requested (as the layer stores fp16 scales)."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    res = {"workload": f"configs[1] weight [{N1},{K1}] -> int4-g128 codes + fp16 scales"}
    for name, dt, esize in (("f32", torch.float32, 4), ("bf16", torch.bfloat16, 2)):
        copies = max(2, -(-2 * L2_BYTES // (N1 * K1 * esize)))
        ws = [(torch.randn((N1, K1), generator=gen, device=dev) * 0.02).to(dt) for _ in range(copies)]
        outs = [Kn.quant_int4_g128(w, want_scale32=False) for w in ws]            # warm; allocates outputs
        del outs
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for i in range(reps):
            Kn.quant_int4_g128(ws[i % copies], want_scale32=False)
        b.record()
        torch.cuda.synchronize(dev)
        s_ = a.elapsed_time(b) * 1e-3 / reps
        nbytes = N1 * K1 * esize + weight_bytes(N1, K1)
        gbs = nbytes / s_ / 1e9
        res[name] = {"us_per_call": round(s_ * 1e6, 2), "GB_per_s": round(gbs, 1),
                     "roofline": {"kernel": "quant_int4_g128_kernel", "bound": "hbm", "achieved": round(gbs, 1),
                                  "peak": hbm_peak, "unit": "GB/s", "frac": round(gbs / hbm_peak, 4),
                                  "peak_source": f"{peak_kind} hbm_gbs",
                                  "algorithmic_bytes_per_launch": nbytes}}
        del ws
    return res


def gemm_measure(torch, Kn, fmt, dev, tf_peak, peak_kind, reps=20):
    gen = torch.Generator(device=dev)
    gen.manual_seed(99)
    W = torch.randn((GN, GK), generator=gen, device=dev) * 0.02
    p, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
    del W
    x = torch.randn((GM, GK), generator=gen, device=dev)
    hit = torch.rand((GM, GK), generator=gen, device=dev) < 0.001
    x = torch.where(hit, x * 20, x).to(torch.bfloat16)
    y = torch.empty((GM, GN), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        Kn.linear(fmt, x, p, s16, GN, out=y)
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        Kn.linear(fmt, x, p, s16, GN, out=y)
    b.record()
    torch.cuda.synchronize(dev)
    s = a.elapsed_time(b) * 1e-3 / reps
    flops = 2 * GM * GN * GK
    tf = flops / s / 1e12
    return {"workload": "configs[2]: int4-g128 GEMM M=2048 N=12288 K=4096, x with 0.1% outliers x20",
            "us_per_call": round(s * 1e6, 2), "TFLOP_per_s": round(tf, 1),
            "roofline": {"kernel": "gemm_kernel<int4,256> (+prep_x_kernel)", "bound": "tensor",
                         "achieved": round(tf, 1), "peak": tf_peak, "unit": "TFLOP/s", "frac": round(tf / tf_peak, 4),
                         "peak_source": f"{peak_kind} bf16_tflops (burst)",
                         "traffic": read_traffic("gemm_int4_m2048_12288x4096")}}


def mlp70b_measure(torch, Kn, fmt, dev, rank, world, stream, hbm_peak, tf_peak, peak_kind, reps=5):
    """gate and up [28672, 8192] and down [8192, 28672], int4-g128, each column-sharded over the
    `world` ranks (rank r holds rows [r N / world, (r + 1) N / world)); strong scaling.  For M in {1, 64, 2048}:
    the per-rank products of one MLP (three matrices, as a CUDA graph for M = 1); with several ranks also the
    three NCCL all-gathers plus interleaves on their own, products and all-gathers together, and the products
    with the gather fused in (peer stores over NVLink + one flag barrier per matrix).  Each rank keeps enough
    distinct weight copies to stream more than twice the L2 per MLP pass, so nothing is served from L2.  Times
    are the max over ranks."""
    import torch.distributed as dist
    from apsi_b200 import sharded as S
    shapes = [("gate", MLP_N, MLP_K), ("up", MLP_N, MLP_K), ("down", MLP_K, MLP_N)]
    per_rank = sum(weight_bytes(n // world, k) for _, n, k in shapes)
    copies = max(1, -(-2 * L2_BYTES // per_rank))
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242 + rank)
    mats = []
    for _ in range(copies):
        lst = []
        for _, n, k in shapes:
            W = torch.randn((n // world, k), generator=gen, device=dev) * 0.015
            p, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
            del W
            lst.append((p, s16, n // world, k))
        mats.append(lst)
    total_w = sum(weight_bytes(n, k) for _, n, k in shapes)
    flops_per_token = 2 * sum(n * k for _, n, k in shapes)
    # world > 1: the whole (unsharded) MLP on each GPU alone, the 1-GPU time the strong-scaling efficiency of
    # this run is computed against (363 MB of weights, more than twice the L2: one copy suffices)
    full_mats = []
    if world > 1:
        for _, n, k in shapes:
            W = torch.randn((n, k), generator=gen, device=dev) * 0.015
            p, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
            del W
            full_mats.append((p, s16, n, k))

    def maxed(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    peers = [S.PeerOutputs(n, 2048, dev) for _, n, _ in shapes] if world > 1 else None
    res = {"workload": f"configs[4]: 70B MLP gate/up [{MLP_N},{MLP_K}], down [{MLP_K},{MLP_N}], int4-g128, "
                       f"column-sharded x{world}" + (" (gather fused into the products, or NCCL all-gather + "
                                                    "interleave)" if world > 1 else ""),
           "weight_bytes_per_mlp": total_w, "weight_copies_per_rank": copies, "scaling": "strong"}
    for M in (1, 64, 2048):
        xs = {k: torch.randn((M, k), generator=gen, device=dev).to(torch.bfloat16) for k in (MLP_K, MLP_N)}
        ys = [torch.empty((M, nl), dtype=torch.bfloat16, device=dev) for (_, _, nl, _) in mats[0]]
        gath = [torch.empty((world, M, nl), dtype=torch.bfloat16, device=dev) for (_, _, nl, _) in mats[0]] \
            if world > 1 else None

        def compute(c):
            for j, (p, s16, nl, k) in enumerate(mats[c]):
                Kn.linear(fmt, xs[k], p, s16, nl, out=ys[j], static_weights=(M <= 16))

        yfull = [torch.empty((M, n), dtype=torch.bfloat16, device=dev) for (_, _, n, _) in full_mats]

        def single():
            for j, (p, s16, n, k) in enumerate(full_mats):
                Kn.linear(fmt, xs[k], p, s16, n, out=yfull[j], static_weights=(M <= 16))

        def gather():
            for j in range(3):
                dist.all_gather_into_tensor(gath[j].view(-1), ys[j].view(-1))
                Kn.interleave_cols(gath[j], world, M, ys[j].shape[1])

        def fused(c):
            for j, (p, s16, nl, k) in enumerate(mats[c]):
                Kn.linear_sharded(fmt, xs[k], p, s16, nl, peers[j].ptrs[0], rank, peers[j].N,
                                  static_weights=(M <= 16))
                Kn.rank_barrier(peers[j].ptrs[2], rank, 0, dev)

        with torch.cuda.stream(stream):
            for c in range(copies):
                compute(c)
                if world > 1:
                    gather()
                    fused(c)
            if world > 1:
                single()
        torch.cuda.synchronize(dev)
        graph = fgraph = sgraph = None
        if M <= 16:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for c in range(copies):
                    compute(c)
            if world > 1:
                fgraph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(fgraph, stream=stream):
                    for c in range(copies):
                        fused(c)
                sgraph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(sgraph, stream=stream):
                    single()
            torch.cuda.synchronize(dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(10)]
        if world > 1:
            dist.barrier()
        with torch.cuda.stream(stream):
            ev[0].record(stream)
            for _ in range(reps):
                if graph is not None:
                    graph.replay()
                else:
                    for c in range(copies):
                        compute(c)
            ev[1].record(stream)
            if world > 1:
                ev[2].record(stream)
                for _ in range(reps * copies):
                    gather()
                ev[3].record(stream)
                ev[4].record(stream)
                for _ in range(reps):
                    for c in range(copies):
                        compute(c)
                        gather()
                ev[5].record(stream)
                ev[6].record(stream)
                for _ in range(reps):
                    if fgraph is not None:
                        fgraph.replay()
                    else:
                        for c in range(copies):
                            fused(c)
                ev[7].record(stream)
                ev[8].record(stream)
                for _ in range(reps * copies):
                    if sgraph is not None:
                        sgraph.replay()
                    else:
                        single()
                ev[9].record(stream)
        torch.cuda.synchronize(dev)
        n_mlp = reps * copies
        comp_s = maxed(ev[0].elapsed_time(ev[1]) * 1e-3 / n_mlp)
        r = {"compute_us_per_mlp": round(comp_s * 1e6, 2)}
        if M == 1:
            gbs = total_w / comp_s / 1e9
            r["weight_GB_per_s"] = round(gbs, 1)
            r["hbm_frac"] = round(gbs / (hbm_peak * world), 4)
        else:
            tf = flops_per_token * M / comp_s / 1e12
            r["TFLOP_per_s"] = round(tf, 1)
            r["tensor_frac"] = round(tf / (tf_peak * world), 4)
        if world > 1:
            ag_s = maxed(ev[2].elapsed_time(ev[3]) * 1e-3 / n_mlp)
            e2e_s = maxed(ev[4].elapsed_time(ev[5]) * 1e-3 / n_mlp)
            recv = sum(M * (n // world) * 2 * (world - 1) for _, n, _ in shapes)
            r["allgather_us_per_mlp"] = round(ag_s * 1e6, 2)
            r["allgather_bytes_received_per_rank"] = recv
            r["allgather_GB_per_s_per_rank"] = round(recv / ag_s / 1e9, 1)
            r["compute_plus_gather_us_per_mlp"] = round(e2e_s * 1e6, 2)
            fu_s = maxed(ev[6].elapsed_time(ev[7]) * 1e-3 / n_mlp)
            r["fused_gather_us_per_mlp"] = round(fu_s * 1e6, 2)
            if M == 1:
                r["fused_weight_GB_per_s"] = round(total_w / fu_s / 1e9, 1)
            else:
                r["fused_TFLOP_per_s"] = round(flops_per_token * M / fu_s / 1e12, 1)
            one_s = maxed(ev[8].elapsed_time(ev[9]) * 1e-3 / n_mlp)
            r["single_gpu_us_per_mlp"] = round(one_s * 1e6, 2)
            r["compute_efficiency"] = round(one_s / (world * comp_s), 4)
            r["fused_efficiency"] = round(one_s / (world * fu_s), 4)
        if world > 1:
            r["gather_bitexact"] = gather_check(torch, Kn, fmt, dev, rank, world, mats[0], xs, ys, gath,
                                                [(q.ptrs[0], q.ptrs[2], q.N, q.view0(M)) for q in peers], M)
        res[f"M={M}"] = r
        del graph, fgraph, sgraph
    res["peaks"] = f"{peak_kind} hbm_gbs {hbm_peak} and bf16_tflops {tf_peak}, times world size"
    if peers is not None:
        for q in peers:
            q.close()
    return res


def gather_check(torch, Kn, fmt, dev, rank, world, mats, xs, ys, gath, outs, M):
    """Correctness of the fused gather at this world size, checked by the bench itself: every rank runs each
    product once more with the gather fused in (peer stores + flag barrier), then computes its own shard alone,
    collects all ranks' shards with an NCCL all-gather + interleave, and compares that [M, N] with the fused
    output bit for bit.  True only if every matrix matches on every rank."""
    import torch.distributed as dist
    ok = True
    for j, (p, s16, nl, k) in enumerate(mats):
        yptrs, fptrs, ldy, view = outs[j]
        Kn.linear_sharded(fmt, xs[k], p, s16, nl, yptrs, rank, ldy, static_weights=(M <= 16))
        Kn.rank_barrier(fptrs, rank, 0, dev)
        Kn.linear(fmt, xs[k], p, s16, nl, out=ys[j])
        dist.all_gather_into_tensor(gath[j].view(-1), ys[j].view(-1))
        ref = Kn.interleave_cols(gath[j], world, M, nl)
        torch.cuda.synchronize(dev)
        ok = ok and bool(torch.equal(view, ref))
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(int(t) == 1) and Kn.device_errors(dev) == 0


def decoder_measure(torch, dev, hbm_peak, batch=8, prompt=512, steps=128):
    """the 7B-class decoder (32 layers, d=4096, 32 heads, 8 KV heads, SwiGLU 11008, vocab 32000,
    RMSNorm, RoPE), random init, every projection int4-g128 on the library's kernels (apsi_b200.decoder);
    batch 8 x 512 prompt tokens (uniform ids, seeded), then 128 greedy decode steps, each one CUDA-graph
    replay.  Tokens per second of the prefill and of the decode; the decode's weight stream (every packed
    weight once per step) as GB/s against the HBM peak."""
    from apsi_b200.decoder import QuantDecoder, DecoderConfig
    cfg = DecoderConfig()
    t0 = time.perf_counter()
    model = QuantDecoder(cfg, device=dev, fmt="int4", seed=0)
    torch.cuda.synchronize(dev)
    build_s = time.perf_counter() - t0
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    ids = torch.randint(0, cfg.V, (batch, prompt), device=dev, generator=g)
    model.generate(ids, 2)                                 # first use of every kernel shape outside the timing
    toks, t = model.generate(ids, steps)
    wb = model.weight_bytes()
    step_s = t["decode_s"] / steps
    res = {"workload": f"configs[3]: 7B-class decoder, {cfg.L} layers, d={cfg.H}, {cfg.nh}/{cfg.kvh} heads, "
                       f"ffn {cfg.I}, vocab {cfg.V}, int4-g128 projections; batch {batch} x {prompt} prompt, "
                       f"{steps} greedy decode steps (CUDA graph per step)",
           "data": "random init (seeded), uniform token ids",
           "prefill_tokens_per_s": round(t["prefill_tokens"] / t["prefill_s"], 1),
           "prefill_ms": round(t["prefill_s"] * 1e3, 2),
           "decode_tokens_per_s": round(t["decode_tokens"] / t["decode_s"], 1),
           "decode_ms_per_step": round(step_s * 1e3, 4),
           "decode_weight_GB_per_s": round(wb / step_s / 1e9, 1),
           "decode_weight_hbm_frac": round(wb / step_s / 1e9 / hbm_peak, 4),
           "weight_bytes": wb, "model_build_s": round(build_s, 2),
           "note": "embedding lookup and attention are torch ops; every projection, RMSNorm, the QKV split with "
                   "RoPE and cache write, and SwiGLU are this library's kernels"}
    del model, toks
    torch.cuda.empty_cache()
    return res


def run_case(case):
    """A short fixed workload for profiler captures (no JSON): a few launches of one kernel on one GPU.

    gemv      int4-g128 GEMV, M=1, [11008, 4096], 8 rotating weight copies (186 MB > L2), 12 launches
    gemv_down int4-g128 GEMV, M=1, [4096, 11008] (K split over a 2-CTA cluster), 12 launches
    gemv_m16  int4-g128 GEMV, M=16, [11008, 4096], 12 launches
    gemm      int4-g128 GEMM, M=2048, [12288, 4096], 4 launches (each also runs prep_x_kernel)
    gemm_m64  int4-g128 GEMM, M=64, [28672, 8192] (configs[4]'s gate / up at M = 64), 4 launches
    quant     int4-g128 quantisation of a float32 [11008, 4096] weight, 4 launches
    decode_step  one eager decode step of the configs[3] decoder (batch 8 after a 512-token prefill), inside
              the NVTX range "decode_step" (capture it with ncu --nvtx --nvtx-include "decode_step/")"""
    import torch
    from apsi_b200 import kernels as Kn
    from apsi_b200._lib import FMT_INT4_G128
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    if case in ("gemv", "gemv_down", "gemv_m16"):
        M, N, K = {"gemv": (1, 11008, 4096), "gemv_down": (1, 4096, 11008), "gemv_m16": (16, 11008, 4096)}[case]
        ws = []
        for _ in range(8):
            W = torch.randn((N, K), generator=gen, device=dev) * 0.02
            p, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
            ws.append((p, s16))
        x = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        for i in range(12):
            p, s16 = ws[i % 8]
            Kn.linear(FMT_INT4_G128, x, p, s16, N, out=y)
    elif case == "gemm":
        W = torch.randn((GN, GK), generator=gen, device=dev) * 0.02
        p, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
        x = torch.randn((GM, GK), generator=gen, device=dev).to(torch.bfloat16)
        y = torch.empty((GM, GN), dtype=torch.bfloat16, device=dev)
        for _ in range(4):
            Kn.linear(FMT_INT4_G128, x, p, s16, GN, out=y)
    elif case == "gemm_m64":
        W = torch.randn((MLP_N, MLP_K), generator=gen, device=dev) * 0.015
        p, s16, _ = Kn.quant_int4_g128(W, want_scale32=False)
        del W
        x = torch.randn((64, MLP_K), generator=gen, device=dev).to(torch.bfloat16)
        y = torch.empty((64, MLP_N), dtype=torch.bfloat16, device=dev)
        for _ in range(4):
            Kn.linear(FMT_INT4_G128, x, p, s16, MLP_N, out=y)
    elif case == "quant":
        W = torch.randn((N1, K1), generator=gen, device=dev) * 0.02
        for _ in range(4):
            Kn.quant_int4_g128(W, want_scale32=True)
    elif case == "decode_step":
        from apsi_b200.decoder import QuantDecoder, DecoderConfig
        cfg = DecoderConfig()
        model = QuantDecoder(cfg, device=dev, fmt="int4", seed=0)
        ids = torch.randint(0, cfg.V, (8, 512), device=dev, generator=gen)
        cache = model.new_cache(8, 520)
        tok = model.prefill(ids, cache).float().argmax(-1)
        pos = torch.full((1,), 512, dtype=torch.int64, device=dev)
        model.decode_step(tok, cache, pos)                   # first use of every kernel shape
        torch.cuda.synchronize(dev)
        torch.cuda.nvtx.range_push("decode_step")
        model.decode_step(tok, cache, pos)
        torch.cuda.nvtx.range_pop()
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize(dev)
    errs = Kn.device_errors(dev)
    print(f"case {case} done, device error bits {errs}")
    return 1 if errs else 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="profiling workload (see run_case); no JSON output")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.case:
        return run_case(args.case)
    if args.impl == "reference":
        return run_reference(args, rank)
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
