"""The C ABI library loads, exports every symbol include/b2c.h declares, and
validates arguments before touching the GPU. No compute call happens here."""

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from mlx_addons_b200 import _lib
import mlx_addons_b200.linalg as la

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "b2c.h")


def _declared():
    with open(HEADER) as f:
        src = f.read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(b2c_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from mlx_addons_b200 import _build
    _build.build()
    return _lib.load()


def test_header_declares_the_binding(lib):
    declared = _declared()
    assert declared == sorted(_lib.SIGNATURES), declared


def test_library_exports_every_declared_symbol(lib):
    for name in _declared():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_version(lib):
    assert _lib.version() == (0, 1, 0)


def test_argument_validation_without_gpu(lib):
    # rejected before any CUDA call
    rc = lib.b2c_posv(None, None, None, None, None, -1, 4, 1, None, 0, None)
    assert rc == _lib.B2C_ERR_INVALID_ARGUMENT
    assert b"batch" in lib.b2c_last_error()
    assert lib.b2c_posv(None, None, None, None, None, 3, 0, 1, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_posv(None, None, None, None, None, 3, 4, -2, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_posv(None, None, None, None, None, 3, 4, 1, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_posv(None, None, None, None, None, 3, 1 << 20, 1, None, 0, None) == _lib.B2C_ERR_UNSUPPORTED
    assert lib.b2c_potrf(None, None, None, 3, 4, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_trsm(None, None, None, 3, 4, 1, 2, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_trsm(None, None, None, 3, 4, 1, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_slogdet(None, None, None, 3, 0, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_slogdet(None, None, None, 3, 4, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_gesv(None, None, None, 3, 0, 1, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_gesv(None, None, None, 3, 4, 1, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_gesv(None, None, None, 3, 1 << 20, 1, None, 0, None) == _lib.B2C_ERR_UNSUPPORTED
    buf = ctypes.c_float(0)
    assert lib.b2c_gesv(ctypes.byref(buf), ctypes.byref(buf), ctypes.byref(buf), 1, 1, 1, None, 0,
                        None) == _lib.B2C_ERR_INVALID_ARGUMENT  # x aliases b
    assert b"alias" in lib.b2c_last_error()
    assert lib.b2c_qr(None, None, None, 3, 0, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_qr(None, None, None, 3, 4, None, 0, None) == _lib.B2C_ERR_INVALID_ARGUMENT
    assert lib.b2c_qr(None, None, None, 3, 1 << 20, None, 0, None) == _lib.B2C_ERR_UNSUPPORTED
    assert lib.b2c_qr(None, None, None, 0, 4, None, 0, None) == _lib.B2C_OK
    # empty batches are valid no-ops
    assert lib.b2c_posv(None, None, None, None, None, 0, 4, 1, None, 0, None) == _lib.B2C_OK
    assert lib.b2c_last_error() == b""
    assert lib.b2c_trsm(None, None, None, 0, 4, 1, 1, None) == _lib.B2C_OK


def test_check_maps_codes(lib):
    lib.b2c_posv(None, None, None, None, None, -1, 4, 1, None, 0, None)
    with pytest.raises(ValueError):
        _lib.check(_lib.B2C_ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.B2C_ERR_UNSUPPORTED, "x")
    with pytest.raises(_lib.B2CError):
        _lib.check(_lib.B2C_ERR_CUDA, "x")


def test_python_shape_validation():
    A = np.zeros((2, 3, 3), np.float32)
    with pytest.raises(ValueError):
        la.solve(np.zeros((3, 3), np.float32), np.zeros((3, 1), np.float32))
    with pytest.raises(ValueError):
        la.solve(np.zeros((2, 3, 4), np.float32), np.zeros((2, 3, 1), np.float32))
    with pytest.raises(ValueError):
        la.solve(A, np.zeros((2, 4, 1), np.float32))
    with pytest.raises(ValueError):
        la.solve(A, np.zeros((3, 3), np.float32))
    with pytest.raises(ValueError):
        la.cholesky(np.zeros((2, 2, 3, 3), np.float32))
    with pytest.raises(ValueError):
        la.slogdet(np.zeros((2, 3, 4), np.float32))
    with pytest.raises(TypeError):
        la.solve([[1.0]], [[1.0]])


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    A = np.eye(4, dtype=np.float32)[None].repeat(2, 0)
    b = np.ones((2, 4), np.float32)
    for fn, args in ((la.solve, (A, b)), (la.cholesky, (A,)), (la.logdet_spd, (A,)), (la.slogdet, (A,)),
                     (la.tril_solve, (A, b)), (la.triu_solve, (A, b))):
        with pytest.raises(RuntimeError, match="CUDA"):
            fn(*args)
