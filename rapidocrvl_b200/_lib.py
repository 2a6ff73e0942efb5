"""ctypes binding of libocrvl_cuda.so (include/ocrvl_cuda.h).

The library is built in-tree by rapidocrvl_b200/build.py.  There is no CPU
fallback: if the library cannot be built or loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

_lock = threading.Lock()
_lib = None

OK = 0
E_INVALID = -1
E_CUDA = -2
E_NOMEM = -3
E_TIMEOUT = -4


class OcrvlError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ocrvl error {code}: {msg}")
        self.code = code


class ModelDesc(C.Structure):
    _fields_ = [
        ("vocab_size", C.c_int32),
        ("hidden_size", C.c_int32),
        ("intermediate_size", C.c_int32),
        ("num_layers", C.c_int32),
        ("num_heads", C.c_int32),
        ("num_kv_heads", C.c_int32),
        ("head_dim", C.c_int32),
        ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_double),
        ("mrope_section", C.c_int32 * 3),
        ("max_position", C.c_int32),
        ("kv_pool_bytes", C.c_int64),
    ]


# name -> (restype, argtypes); the exported symbol set of include/ocrvl_cuda.h
P, I, I64, F = C.c_void_p, C.c_int, C.c_int64, C.c_float
SIGNATURES = {
    "ocrvl_last_error": (C.c_char_p, []),
    "ocrvl_device_count": (I, []),
    "ocrvl_init": (I, [I, C.POINTER(ModelDesc), C.POINTER(P)]),
    "ocrvl_load_tensor": (I, [P, C.c_char_p, I, I64, I64, P, P]),
    "ocrvl_load_gguf": (I, [P, C.c_char_p]),
    "ocrvl_finalize": (I, [P]),
    "ocrvl_quant_type": (I, [P]),
    "ocrvl_trace_read": (I, [P, P, I]),
    "ocrvl_set_wait_limit": (I, [P, I64]),
    "ocrvl_debug_read": (I, [P, I, P, I64]),
    "ocrvl_free": (None, [P]),
    "ocrvl_seq_create": (I, [P, I, C.POINTER(P)]),
    "ocrvl_seq_reset": (I, [P]),
    "ocrvl_seq_free": (None, [P]),
    "ocrvl_seq_len": (I, [P]),
    "ocrvl_seq_read_kv": (I, [P, I, P, P]),
    "ocrvl_seq_import_kv": (I, [P, I, P, P]),
    "ocrvl_seq_fill_synthetic": (I, [P, I, C.c_uint64]),
    "ocrvl_step": (I, [P, P, I, P, P, P, I, P, P]),
    "ocrvl_step_sample": (I, [P, P, I, P, P, P, C.c_double, I, P, P]),
    "ocrvl_generate": (I, [P, P, I, I, P, I, C.c_double, I, C.c_int64, P, I, C.POINTER(I)]),
    "ocrvl_generate_greedy": (I, [P, P, I, I, P, I, P, I, C.POINTER(I)]),
    "ocrvl_decode_greedy_device": (I, [P, P, I, P, I, P]),
    "ocrvl_model_stream": (P, [P]),
    "ocrvl_step_io_bytes": (I, [P, I, C.POINTER(I64), C.POINTER(I64)]),
    "ocrvl_op_rowsum": (I, [I, I, I, P, P, P]),
    "ocrvl_op_matvec": (I, [I, I, I, P, P, P, I, P, P, F, P, P]),
    "ocrvl_op_matvec_add_rmsnorm": (I, [I, I, I, P, P, P, I, P, P, I, P, F, P, P, P]),
    "ocrvl_op_swiglu": (I, [I, I, I, P, P, P, P, P, P, I, P, P, P]),
    "ocrvl_op_argmax": (I, [I, I, I, P, P, P, I, P, P, P]),
    "ocrvl_op_argmax_noalloc": (I, [I, I, I, P, P, P, I, P, P, P]),
    "ocrvl_op_sample": (I, [I, I, P, C.c_double, I, P, P, P, P, P, P]),
    "ocrvl_op_rmsnorm": (I, [I, I, P, P, F, P, P]),
}


def lib_path() -> str:
    return _build.LIB


def load():
    """Load (building first if needed) the CUDA library."""
    global _lib
    with _lock:
        if _lib is None:
            path = _build.build()
            L = C.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    return (load().ocrvl_last_error() or b"").decode(errors="replace")


def check(rc: int) -> int:
    if rc is not None and rc < 0:
        raise OcrvlError(rc, last_error())
    return rc
