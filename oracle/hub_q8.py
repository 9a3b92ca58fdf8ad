"""ctypes binding of ``oracle/libhub_q8.so`` (``hub_q8.c``): the reference's fastest CPU product for a quantized
layer, restated (TEST INFRASTRUCTURE: the timed CPU baseline of bench.py and a checker in tests/).

* ``q8_from_weights(W)`` -- the reference's ``Q8.from_bf16`` (apsi/hub_cpu.py:180-194) on a float32 [O, I]
  weight already rounded to bfloat16: per 32-value block ``sc = float32(amax / 127)``, ``inv = 1 / sc`` (0 for an
  all-zero block), codes ``clip(rint(w * inv), -127, 127)`` in int8.
* ``matmul(x, codes, scales, threads)`` -- ``hub_cpu.matmul`` on a ``Q8`` for fewer than its prompt threshold of
  rows (apsi/hub_cpu.py:474-534): the row kernel on all cores, float32 [T, O].
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libhub_q8.so")
_lib = None


def build(force=False):
    src = os.path.join(HERE, "hub_q8.c")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s"] + (["-B"] if force else []) + ["-C", HERE, "libhub_q8.so"], check=True)
    return LIB


def load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        lib = ctypes.CDLL(LIB)
        P, I64 = ctypes.c_void_p, ctypes.c_int64
        lib.hub_q8_matmul.argtypes = [P, P, P, P, I64, I64, I64, ctypes.c_int]
        lib.hub_q8_matmul.restype = ctypes.c_int
        lib.hub_q8_isa.argtypes = []
        lib.hub_q8_isa.restype = ctypes.c_int
        _lib = lib
    return _lib


def q8_from_weights(W):
    """int8 codes [O, I] and float32 scales [O, I / 32] of the reference's Q8_0 layout."""
    W = np.asarray(W, np.float32)
    O, I = W.shape
    blk = W.reshape(O, I // 32, 32)
    amax = np.abs(blk).max(axis=2)
    sc = (amax / 127.0).astype(np.float32)
    inv = np.where(sc > 0, 1.0 / np.where(sc > 0, sc, 1), 0).astype(np.float32)
    codes = np.clip(np.rint(blk * inv[:, :, None]), -127, 127).astype(np.int8).reshape(O, I)
    return codes, sc


def matmul(x, codes, scales, threads=0):
    """float32 [T, O] = x [T, I] . deq(W)^T on `threads` host threads (0: all)."""
    lib = load()
    x = np.ascontiguousarray(x, np.float32)
    codes = np.ascontiguousarray(codes, np.int8)
    scales = np.ascontiguousarray(scales, np.float32)
    T, I = x.shape
    O = codes.shape[0]
    y = np.empty((T, O), np.float32)
    lib.hub_q8_matmul(codes.ctypes.data, scales.ctypes.data, x.ctypes.data, y.ctypes.data, I, T, O, int(threads))
    return y


def host_threads():
    """The thread count the reference's team uses (apsi/native/engine.py:47-54): the CPUs this process may run on."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or 1)
