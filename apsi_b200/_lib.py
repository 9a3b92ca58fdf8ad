"""ctypes binding of ``liblowbit_b200.so`` (the C ABI in ``include/apsi_lowbit.h``).

The library is the only compute path: if it is missing, or the device is not an sm_100 GPU, every call
raises ``LowbitError``.  There is no CPU fallback.
"""
import ctypes
import os
import threading

from .build import LIB_PATH

LB_OK = 0
LB_E_ARG, LB_E_ALIGN, LB_E_DEVICE, LB_E_LAUNCH, LB_E_WORKSPACE, LB_E_UNSUPPORTED = -1, -2, -3, -4, -5, -6
FMT_INT8_ROW, FMT_INT4_G128, FMT_Q8_0_G32, FMT_Q4_0_G32 = 1, 2, 3, 4
FMT_FP8_E4M3, FMT_FP8_E5M2, FMT_FP6_E3M2, FMT_FP6_E2M3, FMT_FP4_E2M1 = 5, 6, 7, 8, 9
MINIFLOAT_FMT = {"fp8_e4m3": FMT_FP8_E4M3, "fp8_e5m2": FMT_FP8_E5M2, "fp6_e3m2": FMT_FP6_E3M2,
                 "fp6_e2m3": FMT_FP6_E2M3, "fp4_e2m1": FMT_FP4_E2M1}
DT_F32, DT_BF16, DT_F16 = 0, 1, 2
DEVERR_WAIT_TIMEOUT = 1
DEVERR_PEER_TIMEOUT = 2
IPC_HANDLE_BYTES = 64
MAX_RANKS = 8
LINEAR_STATIC_WEIGHTS = 1
NOALLOC_SCRATCH_BYTES = 16842752

_CODES = {LB_E_ARG: "bad argument", LB_E_ALIGN: "misaligned", LB_E_DEVICE: "device", LB_E_LAUNCH: "launch",
          LB_E_WORKSPACE: "workspace", LB_E_UNSUPPORTED: "unsupported"}

# (name, restype, argtypes) of every exported entry point
_P, _I, _I64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t
SIGNATURES = [
    ("lb_version", _I, []),
    ("lb_last_error", ctypes.c_char_p, []),
    ("lb_init", _I, [_I]),
    ("lb_device_errors", _I, [_P, ctypes.POINTER(ctypes.c_int)]),
    ("lb_quant_int8_rows", _I, [_P, _I, _I64, _I64, _P, _P, _P, _P]),
    ("lb_quant_int4_g128", _I, [_P, _I, _I64, _I64, _P, _P, _P, _P]),
    ("lb_quant_q8_0_g32", _I, [_P, _I, _I64, _I64, _P, _P, _P]),
    ("lb_quant_q4_0_g32", _I, [_P, _I, _I64, _I64, _P, _P, _P]),
    ("lb_round_g32", _I, [_I, _P, _I, _I64, _I64, _P, _P]),
    ("lb_dequant", _I, [_I, _P, _P, _I, _I64, _I64, _P, _I, _P]),
    ("lb_minifloat_bytes", _I64, [_I, _I64]),
    ("lb_quant_minifloat", _I, [_I, _P, _I, _I64, _I64, _I, _P, _P, _P, _P]),
    ("lb_dequant_minifloat", _I, [_I, _P, _I64, _I64, _I, _P, ctypes.c_float, _P, _I, _P]),
    ("lb_gguf_encode", _I, [_I, _P, _I64, _P, _P]),
    ("lb_gguf_decode", _I, [_I, _P, _I64, _P, _P]),
    ("lb_linear_workspace_size", _I, [_I, _I64, _I64, _I64, ctypes.POINTER(_SZ)]),
    ("lb_linear", _I, [_I, _P, _I64, _I64, _P, _P, _I64, _P, _I, _P, _I64, _P, _SZ, _P]),
    ("lb_linear_ex", _I, [_I, _P, _I64, _I64, _P, _P, _I64, _P, _I, _P, _I64, _P, _SZ, ctypes.c_uint, _P]),
    ("lb_weight_create", _I, [_I, _P, _P, _I64, _I64, ctypes.POINTER(_P)]),
    ("lb_weight_linear", _I, [_P, _P, _I64, _P, _I64, ctypes.c_uint, _P]),
    ("lb_weight_destroy", _I, [_P]),
    ("lb_interleave_cols", _I, [_P, _I, _I64, _I64, _P, _P]),
    ("lb_linear_noalloc", _I, [_I, _P, _I64, _I64, _P, _P, _I64, _P, _I, _P, _I64, _P]),
    ("lb_peer_alloc", _I, [_SZ, ctypes.POINTER(_P), _P]),
    ("lb_peer_open", _I, [_P, ctypes.POINTER(_P)]),
    ("lb_peer_close", _I, [_P]),
    ("lb_peer_free", _I, [_P]),
    ("lb_linear_sharded", _I, [_I, _P, _I64, _I64, _P, _P, _I64, _P, ctypes.POINTER(_P), _I, _I, _I64, _P, _SZ,
                               ctypes.c_uint, _P]),
    ("lb_rank_barrier", _I, [ctypes.POINTER(_P), _I, _I, ctypes.c_uint32, ctypes.c_uint32, _P]),
    ("lb_rmsnorm", _I, [_P, _I64, _I64, _P, _I, ctypes.c_float, ctypes.c_float, _P, _P]),
    ("lb_linear_rms_workspace_size", _I, [_I, _I64, _I64, _I64, ctypes.POINTER(_SZ)]),
    ("lb_linear_rms", _I, [_I, _P, _I64, _I64, _P, _I, ctypes.c_float, ctypes.c_float, _P, _P, _I64, _P, _I, _P, _I64,
                           _P, _SZ, ctypes.c_uint, _P]),
    ("lb_qkv_prep", _I, [_P, _I, _I, _I, _I, _I, _I, _P, _P, _P, _P, ctypes.c_float, _P, _I64, _P, _I64, _I64, _I64,
                         _P, _P, _I64, _I64, _P]),
    ("lb_act_mul", _I, [_P, _I64, _I64, _I, _P, _P]),
]


class LowbitError(RuntimeError):
    """A call into the B200 library failed (the message is the library's own)."""

    def __init__(self, code, message):
        super().__init__(f"{message} [{_CODES.get(code, code)}]")
        self.code = code


_lock = threading.Lock()
_lib = None


def load(path=None):
    """The loaded library (loads it once).  Raises LowbitError if the file is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or os.environ.get("APSI_B200_LIB", LIB_PATH)
        if not os.path.exists(p):
            raise LowbitError(LB_E_DEVICE, f"{p} is not built (run apsi_b200.build.build() or __graft_entry__.build())")
        lib = ctypes.CDLL(p)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path is None:
            _lib = lib
        return lib


def check(rc):
    """Raise LowbitError for a non-zero status, with the library's message."""
    if rc != LB_OK:
        msg = load().lb_last_error()
        raise LowbitError(rc, msg.decode() if msg else f"status {rc}")
    return rc


def call(name, *args):
    return check(getattr(load(), name)(*args))
