"""Builds the in-tree shared library ``apsi_b200/liblowbit_b200.so`` (sm_100a) with nvcc.

The library is one CUDA translation unit (``csrc/lb_lib.cu``) with the C ABI of ``include/apsi_lowbit.h``.
It links the CUDA runtime statically and needs nothing else at run time (tensor maps are encoded through
the driver entry point), so the built file travels with the source tree.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC_DIR = os.path.join(HERE, "csrc")
LIB_PATH = os.path.join(HERE, "liblowbit_b200.so")
INCLUDE = os.path.join(ROOT, "include")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return cand


def _sources():
    out = [os.path.join(INCLUDE, "apsi_lowbit.h")]
    for f in sorted(os.listdir(SRC_DIR)):
        if f.endswith((".cu", ".cuh", ".h")):
            out.append(os.path.join(SRC_DIR, f))
    return out


def stale():
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in _sources())


def build(force=False, verbose=False):
    """Compile the library if any source is newer than it (or ``force``).  Returns the library path."""
    if not force and not stale():
        return LIB_PATH
    tmp = LIB_PATH + f".{os.getpid()}.tmp"
    cmd = [_nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
           "-I" + INCLUDE, "-o", tmp, os.path.join(SRC_DIR, "lb_lib.cu")]
    if verbose:
        cmd.insert(-3, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose:
        print(r.stderr, file=sys.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
