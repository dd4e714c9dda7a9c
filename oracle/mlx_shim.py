"""Run the reference's own ``mlx_addons.linalg`` Python on the host CPU.

TEST INFRASTRUCTURE ONLY: used in the development container to pin the
oracle and to write the golden fixtures under ``tests/golden/``. Needs the
reference tree (it is not on GPU machines) and ``oracle/_ref/libmlxref.so``
(built by ``oracle/build_ref.py``).

MLX (the reference's only runtime dependency, ``pyproject.toml:25-28``,
unpinned ``mlx>=0.20.0``) is not installable here, so this module installs a
numpy stand-in for ``mlx.core`` into ``sys.modules`` before importing the
reference package:

* arrays are numpy arrays; the ops the linalg path calls map one-to-one onto
  numpy (``reshape``, ``expand_dims``, ``squeeze``, ``concatenate``,
  ``zeros``/``zeros_like``, ``diagonal``, ``sum``, ``log``, ``abs``, ``sign``,
  ``prod``, ``exp``, ``arange``, ``@``);
* ``mx.fast.metal_kernel`` returns a callable that runs the SAME kernel
  source, compiled for the host by ``oracle/build_ref.py``, over the launch
  grid the reference computes (one call per batch element);
* ``mx.linalg.lu_factor(stream=mx.cpu)`` is LAPACK ``sgetrf`` through scipy,
  which is what MLX's CPU stream calls.

So the reference's Python control flow (tier choice, blocking, reshapes,
squeezes, the slogdet sign logic) and its kernel arithmetic run unmodified;
only the MLX matmul (blocked trailing update and block substitution) is
numpy/OpenBLAS float32 instead of Metal, which changes rounding only.
"""

from __future__ import annotations

import contextlib
import ctypes
import importlib
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_LIB = os.path.join(HERE, "_ref", "libmlxref.so")
DEFAULT_REFERENCE = "/root/reference"

_lib = None
_kernel_ids: dict = {}


def _load_lib():
    global _lib
    if _lib is None:
        if not os.path.exists(REF_LIB):
            raise RuntimeError("oracle/_ref/libmlxref.so missing: run python oracle/build_ref.py")
        _lib = ctypes.CDLL(REF_LIB)
        _lib.mlxref_run.restype = ctypes.c_int
        _lib.mlxref_run.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_int]
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


class _MetalKernel:
    """Callable with the ``mx.fast.metal_kernel`` call signature."""

    def __init__(self, name, input_names, output_names, source, **_):
        self.name = name
        self.input_names = list(input_names)
        self.output_names = list(output_names)
        self.source = source

    def _kernel_id(self):
        # Identify which reference constant this source is (by value).
        from oracle.build_ref import KERNEL_IDS
        mk = sys.modules.get("mlx_addons.linalg._metal_kernels")
        for const, kid in KERNEL_IDS.items():
            if getattr(mk, const, None) == self.source:
                return kid
        raise NotImplementedError(f"kernel {self.name!r} is not compiled for the host")

    def __call__(self, inputs, template, grid, threadgroup, output_shapes, output_dtypes, **_):
        t = dict(template)
        K, M, BATCH = int(t["K"]), int(t.get("M", 0)), int(t["BATCH"])
        ins = [np.ascontiguousarray(np.asarray(x), dtype=np.float32) for x in inputs]
        outs = [np.zeros(s, dtype=d) for s, d in zip(output_shapes, output_dtypes)]
        lib = _load_lib()
        optrs = (ctypes.c_void_p * 4)(*[o.ctypes.data for o in outs] + [None] * (4 - len(outs)))
        rc = lib.mlxref_run(self._kernel_id(), _ptr(ins[0]), _ptr(ins[1]) if len(ins) > 1 else None,
                            optrs, K, M, BATCH, int(os.environ.get("ORACLE_THREADS", os.cpu_count() or 1)))
        if rc != 0:
            raise RuntimeError(f"mlxref_run failed for {self.name}")
        return outs


def _lu_factor(a, stream=None):
    import scipy.linalg
    a = np.asarray(a, dtype=np.float32)
    flat = a.reshape((-1,) + a.shape[-2:])
    lus = np.empty_like(flat)
    pivs = np.empty(flat.shape[:2], dtype=np.uint32)
    for i in range(flat.shape[0]):
        lu, piv = scipy.linalg.lu_factor(flat[i], check_finite=False)
        lus[i] = lu
        pivs[i] = piv
    return lus.reshape(a.shape), pivs.reshape(a.shape[:-1])


def _make_mlx_module():
    core = types.ModuleType("mlx.core")
    core.array = lambda x, dtype=None: np.array(x, dtype=dtype)
    core.float32, core.float64, core.uint32, core.int32 = np.float32, np.float64, np.uint32, np.int32
    core.cpu, core.gpu = "cpu", "gpu"
    core.eval = lambda *a, **k: None
    core.reshape = lambda x, shape: np.reshape(x, shape)
    core.expand_dims = lambda x, axis: np.expand_dims(x, axis)
    core.squeeze = lambda x, axis=None: np.squeeze(x, axis=axis)
    core.concatenate = lambda xs, axis=0: np.concatenate(xs, axis=axis)
    core.zeros = lambda shape, dtype=np.float32: np.zeros(shape, dtype=dtype)
    core.zeros_like = lambda x: np.zeros_like(x)
    core.diagonal = lambda x, offset=0, axis1=0, axis2=1: np.diagonal(x, offset, axis1, axis2)
    core.sum = lambda x, axis=None: np.sum(x, axis=axis)
    core.prod = lambda x, axis=None: np.prod(x, axis=axis)
    core.log = np.log
    core.exp = np.exp
    core.abs = np.abs
    core.sign = np.sign
    core.arange = lambda n, dtype=None: np.arange(n, dtype=dtype)
    fast = types.ModuleType("mlx.core.fast")
    fast.metal_kernel = _MetalKernel
    core.fast = fast
    linalg = types.ModuleType("mlx.core.linalg")
    linalg.lu_factor = _lu_factor
    # qr above the GPU kernels' k <= 63 runs on the CPU stream there
    # (_metal_kernels.py:685-688): LAPACK geqrf / orgqr through numpy here
    linalg.qr = lambda a, stream=None: tuple(np.asarray(t, np.float32) for t in np.linalg.qr(np.asarray(a)))
    linalg.svd = lambda a, stream=None: tuple(np.asarray(t, np.float32) for t in np.linalg.svd(np.asarray(a)))
    core.stream = lambda s: contextlib.nullcontext()
    core.swapaxes = np.swapaxes
    core.linalg = linalg
    mlx = types.ModuleType("mlx")
    mlx.core = core
    return mlx, core


def load_reference_linalg(reference: str = DEFAULT_REFERENCE):
    """Import the reference's ``mlx_addons.linalg`` over the numpy stand-in and
    return the module. The package ``__init__`` (which would also import the
    knn/nndescent modules) is bypassed by pre-registering a bare package."""
    if "mlx_addons.linalg" in sys.modules:
        return sys.modules["mlx_addons.linalg"]
    src = os.path.join(reference, "src", "mlx_addons")
    if not os.path.isdir(src):
        raise RuntimeError(f"reference tree not found at {reference}")
    mlx, core = _make_mlx_module()
    sys.modules.setdefault("mlx", mlx)
    sys.modules.setdefault("mlx.core", core)
    pkg = types.ModuleType("mlx_addons")
    pkg.__path__ = [src]
    sys.modules["mlx_addons"] = pkg
    return importlib.import_module("mlx_addons.linalg")
