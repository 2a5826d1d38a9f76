"""ctypes binding of ``libpi05_b200.so`` (the C ABI in ``include/pi05_b200.h``).

The library is built in-tree by ``pi05-infer_b200/build.py``.  There is no CPU
or eager fallback: if the library is missing, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libpi05_b200.so")

PI05_OK = 0
ERR_NAMES = {
    1: "INVALID_ARG",
    2: "SHAPE",
    3: "ALIGN",
    4: "WORKSPACE",
    5: "LAUNCH",
    6: "TMAP",
    7: "DEVICE",
    8: "DRIVER",
}

_P = ctypes.c_void_p
_I = ctypes.c_int
_Z = ctypes.c_size_t
_F = ctypes.c_float

# name -> (restype, argtypes); mirrors include/pi05_b200.h
SIGNATURES = {
    "pi05_abi_version": (_I, []),
    "pi05_last_error": (ctypes.c_char_p, []),
    "pi05_workspace_bytes": (_Z, [_I, _I]),
    "pi05_read_device_status": (_I, [_P, ctypes.POINTER(_I), _P]),
    "pi05_debug_set_splits": (None, [_I]),
    "pi05_debug_set_trace": (None, [_P]),
    "pi05_debug_set_fault": (None, [_I, ctypes.c_ulonglong]),
    "pi05_launch_count": (ctypes.c_longlong, []),
    "pi05_gate_up_geglu": (_I, [_P, _P, _P, _P, _I, _I, _I, _P, _Z, _P]),
    "pi05_gate_up_geglu_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _P]),
    "pi05_gate_up_geglu_noalloc_status": (_I, [ctypes.POINTER(_I), _P]),
    "pi05_qkv_rope_kv": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _Z, _P]),
    "pi05_linear_gated_residual": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _P, _Z, _P]),
    "pi05_linear": (_I, [_P, _P, _P, _I, _I, _I, _P, _Z, _P]),
}


class Pi05Error(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed: PI05_ERR_{ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def lib():
    """Load the shared library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python pi05-infer_b200/build.py` "
                "(pi05_infer has no CPU fallback)"
            )
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    s = lib().pi05_last_error()
    return s.decode() if s else ""


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != PI05_OK:
        raise Pi05Error(name, rc, last_error())
