"""ctypes binding of libb2c.so (the C ABI declared in include/b2c.h).

The library is built in-tree by ``python -m mlx_addons_b200._build``. There is
no CPU fallback: if the library is missing or no CUDA device is present, every
call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
# B2C_LIBRARY points the binding at another build of the same ABI.
LIB_PATH = os.environ.get("B2C_LIBRARY") or os.path.join(HERE, "libb2c.so")

B2C_OK = 0
B2C_ERR_INVALID_ARGUMENT = 1
B2C_ERR_UNSUPPORTED = 2
B2C_ERR_WORKSPACE = 3
B2C_ERR_CUDA = 4

OP_POSV, OP_POTRF, OP_TRSM, OP_SLOGDET, OP_GESV, OP_QR = 0, 1, 2, 3, 4, 5

# Every symbol include/b2c.h declares, with its ctypes signature.
_vp, _i64, _ci, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
SIGNATURES = {
    "b2c_version": (_ci, []),
    "b2c_last_error": (ctypes.c_char_p, []),
    "b2c_workspace_size": (_sz, [_ci, _i64, _ci, _ci]),
    "b2c_posv": (_ci, [_vp, _vp, _vp, _vp, _vp, _i64, _ci, _ci, _vp, _sz, _vp]),
    "b2c_potrf": (_ci, [_vp, _vp, _vp, _i64, _ci, _vp, _sz, _vp]),
    "b2c_trsm": (_ci, [_vp, _vp, _vp, _i64, _ci, _ci, _ci, _vp]),
    "b2c_slogdet": (_ci, [_vp, _vp, _vp, _i64, _ci, _vp, _sz, _vp]),
    "b2c_gesv": (_ci, [_vp, _vp, _vp, _i64, _ci, _ci, _vp, _sz, _vp]),
    "b2c_qr": (_ci, [_vp, _vp, _vp, _i64, _ci, _vp, _sz, _vp]),
    "b2c_posv_static_scratch": (_ci, [_vp, _vp, _vp, _vp, _i64, _ci, _ci, _vp]),
    "b2c_host_device_pointer": (_ci, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "b2c_take_device_fault": (_ci, [ctypes.POINTER(ctypes.c_uint)]),
}

_lib = None
_lock = threading.Lock()


class B2CError(RuntimeError):
    """A libb2c call failed; ``code`` is the B2C_ERR_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is not built; run `python -m mlx_addons_b200._build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc == B2C_OK:
        return
    msg = load().b2c_last_error().decode(errors="replace") or what
    if rc == B2C_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == B2C_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise B2CError(rc, msg)


def version() -> tuple:
    v = load().b2c_version()
    return (v >> 16, (v >> 8) & 0xFF, v & 0xFF)
