"""CPU oracle for the batched SPD Cholesky-solve path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` import this
package, as the checker and as the timed CPU baseline. The product package
(``mlx_addons_b200``) never imports it and has no CPU fallback.

Three CPU implementations live here:

* ``liborc.so`` (``chol_oracle.c``): a plain-C restatement of the reference's
  algorithms (each routine cites the reference file:line it follows). This is
  the oracle the GPU parity tests compare against.
* ``_ref/libmlxref.so`` (``build_ref.py``): the reference's own Metal kernel
  bodies compiled for the host. It pins the restatement (bit-exact on the
  unblocked paths) and is the timed "reference" CPU arm. Built only where the
  reference tree exists; the prebuilt library travels with the repository.
* ``liblapack_cpu.so`` (``lapack_cpu.c``): LAPACK spotrf/spotrs from the
  image's OpenBLAS, the stand-in for MLX's CPU stream, reported for context.

Pinning status: the restatement matches the reference's kernel code run on
the CPU bit for bit on every unblocked path (k <= 80 for solve/cholesky,
k <= 128 for the small kernels and tril/triu_solve), and matches the
reference's blocked Python path and slogdet (run over a numpy stand-in for
MLX, ``mlx_shim.py``) within float32 tolerance. Golden fixtures made from the
reference run sit in ``tests/golden/``.
"""

from __future__ import annotations

import ctypes
import glob
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_LIB = os.path.join(HERE, "liborc.so")
LAPACK_LIB = os.path.join(HERE, "liblapack_cpu.so")
REF_LIB = os.path.join(HERE, "_ref", "libmlxref.so")

# Reference constants (src/mlx_addons/linalg/_metal_kernels.py:19-20, _blocked.py:31)
MAX_GPU_K = 128
SHARED_K_MAX = 80
BLOCK_SIZE = 80
QR_SHARED_K_MAX = 63  # _metal_kernels.py:383


def build(quiet: bool = True) -> None:
    """Compile the C restatement and the LAPACK harness in-tree, and the
    reference's kernels into _ref/ when the reference tree is present."""
    flags = ["-O3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-pthread"]
    for src, out in (("chol_oracle.c", ORC_LIB), ("lapack_cpu.c", LAPACK_LIB)):
        subprocess.run(["gcc", *flags, os.path.join(HERE, src), "-o", out, "-lm"], check=True,
                       capture_output=quiet)
    from oracle import build_ref
    build_ref.build(quiet=quiet)


_orc = None


def _lib():
    global _orc
    if _orc is None:
        if not os.path.exists(ORC_LIB):
            build()
        lib = ctypes.CDLL(ORC_LIB)
        vp, i64, ci = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        sigs = {
            "orc_cholesky": [vp, vp, vp, i64, ci, ci],
            "orc_cholesky_small": [vp, vp, i64, ci, ci],
            "orc_solve": [vp, vp, vp, vp, i64, ci, ci, ci],
            "orc_solve_small": [vp, vp, vp, vp, i64, ci, ci, ci],
            "orc_tril_solve": [vp, vp, vp, i64, ci, ci, ci],
            "orc_triu_solve": [vp, vp, vp, i64, ci, ci, ci],
            "orc_logdet_spd": [vp, vp, i64, ci, ci],
            "orc_slogdet": [vp, vp, vp, i64, ci, ci],
            "orc_lu_solve": [vp, vp, vp, i64, ci, ci, ci],
            "orc_qr": [vp, vp, vp, i64, ci, ci],
        }
        for name, args in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        _orc = lib
    return _orc


def _threads(nthreads):
    return int(nthreads or os.environ.get("ORACLE_THREADS", 0) or os.cpu_count() or 1)


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return np.ascontiguousarray(np.asarray(a), dtype=np.float32)


def _rhs(b):
    """2-D b -> (B, k, 1) like _prep_b (_metal_kernels.py:489-496)."""
    b = _f32(b)
    was_2d = b.ndim == 2
    return (np.ascontiguousarray(b[..., None]) if was_2d else b), was_2d


def _check(rc, what):
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed ({rc})")


def cholesky(A, return_logdet=False, nthreads=None):
    """blocked_cholesky (_blocked.py:34-137): (B, n, n) -> L with zero upper."""
    A = _f32(A)
    B, n, _ = A.shape
    L = np.empty_like(A)
    ld = np.empty(B, np.float32) if return_logdet else None
    _check(_lib().orc_cholesky(_p(A), _p(L), _p(ld), B, n, _threads(nthreads)), "cholesky")
    return (L, ld) if return_logdet else L


def cholesky_small(A, nthreads=None):
    """_metal_kernels.cholesky (:562-590), unblocked for every k."""
    A = _f32(A)
    B, n, _ = A.shape
    L = np.empty_like(A)
    _check(_lib().orc_cholesky_small(_p(A), _p(L), B, n, _threads(nthreads)), "cholesky_small")
    return L


def solve(A, b, return_logdet=False, nthreads=None):
    """blocked_solve (_blocked.py:140-217); x has b's shape."""
    A = _f32(A)
    b3, was_2d = _rhs(b)
    B, n, _ = A.shape
    m = b3.shape[-1]
    x = np.empty_like(b3)
    ld = np.empty(B, np.float32) if return_logdet else None
    _check(_lib().orc_solve(_p(A), _p(b3), _p(x), _p(ld), B, n, m, _threads(nthreads)), "solve")
    x = x[..., 0] if was_2d else x
    return (x, ld) if return_logdet else x


def solve_small(A, b, return_logdet=False, nthreads=None):
    """_metal_kernels.solve (= solve_cholesky, :536-559 / :972), unblocked."""
    A = _f32(A)
    b3, was_2d = _rhs(b)
    B, n, _ = A.shape
    m = b3.shape[-1]
    x = np.empty_like(b3)
    ld = np.empty(B, np.float32) if return_logdet else None
    _check(_lib().orc_solve_small(_p(A), _p(b3), _p(x), _p(ld), B, n, m, _threads(nthreads)), "solve_small")
    x = x[..., 0] if was_2d else x
    return (x, ld) if return_logdet else x


def _tri(fn, L, b, nthreads):
    L = _f32(L)
    b3, was_2d = _rhs(b)
    B, k, _ = L.shape
    m = b3.shape[-1]
    x = np.empty_like(b3)
    _check(fn(_p(L), _p(b3), _p(x), B, k, m, _threads(nthreads)), "triangular solve")
    return x[..., 0] if was_2d else x


def tril_solve(L, b, nthreads=None):
    """L x = b (_metal_kernels.py:593-614)."""
    return _tri(_lib().orc_tril_solve, L, b, nthreads)


def triu_solve(L, b, nthreads=None):
    """L^T x = b with the LOWER factor L (_metal_kernels.py:617-638)."""
    return _tri(_lib().orc_triu_solve, L, b, nthreads)


def logdet_spd(A, nthreads=None):
    """2 sum log diag(cholesky(A)) (_det.py:51-67, :100-113)."""
    A = _f32(A)
    B, n, _ = A.shape
    out = np.empty(B, np.float32)
    _check(_lib().orc_logdet_spd(_p(A), _p(out), B, n, _threads(nthreads)), "logdet_spd")
    return out


def slogdet(A, nthreads=None):
    """(sign, logabsdet) via partial-pivot LU (_det.py:17-48); any leading dims."""
    A = _f32(A)
    lead, n = A.shape[:-2], A.shape[-1]
    flat = np.ascontiguousarray(A.reshape((-1, n, n)))
    s = np.empty(flat.shape[0], np.float32)
    l = np.empty(flat.shape[0], np.float32)
    _check(_lib().orc_slogdet(_p(flat), _p(s), _p(l), flat.shape[0], n, _threads(nthreads)), "slogdet")
    return s.reshape(lead), l.reshape(lead)


def det(A, nthreads=None):
    """sign * exp(logabsdet) (_det.py:70-81)."""
    s, l = slogdet(A, nthreads)
    return s * np.exp(l)


def lu_solve(A, b, nthreads=None):
    """solve_lu (_metal_kernels.py:917-969): partial-pivot LU, any square A."""
    A = _f32(A)
    b3, was_2d = _rhs(b)
    B, n, _ = A.shape
    m = b3.shape[-1]
    x = np.empty_like(b3)
    _check(_lib().orc_lu_solve(_p(A), _p(b3), _p(x), B, n, m, _threads(nthreads)), "lu_solve")
    return x[..., 0] if was_2d else x


def qr(A, nthreads=None):
    """Householder qr (_metal_kernels.py:641-694) -> (Q, R), A (B, k, k)."""
    A = _f32(A)
    B, n, _ = A.shape
    Q, R = np.empty_like(A), np.empty_like(A)
    _check(_lib().orc_qr(_p(A), _p(Q), _p(R), B, n, _threads(nthreads)), "qr")
    return Q, R


def randomized_svd(X, n_components, n_oversamples=10, n_iter=4, random_state=42, flip_signs=True):
    """numpy restatement of the reference's randomized_svd (_svd.py:48-175):
    the same Omega draw (:124-126), power iteration with a re-orthogonalising
    Householder thin QR (LAPACK through numpy, the stand-in for MLX's CPU QR,
    :28-45, :133-139), projection, small SVD (:141-145), top-k and the
    Vt-based sign flip (:155-172). Returns numpy (U, S, Vt)."""
    X = np.ascontiguousarray(np.asarray(X, dtype=np.float32))
    batched = X.ndim == 3
    if not batched:
        X = X[None]
    B, n, m = X.shape
    k = min(n_components, min(n, m))
    kp = k + n_oversamples
    omega = np.random.default_rng(random_state).standard_normal((B, m, kp)).astype(np.float32)
    qr = lambda Y: np.linalg.qr(Y)[0].astype(np.float32)  # noqa: E731
    Xt = np.swapaxes(X, -1, -2)
    Y = X @ omega
    for _ in range(n_iter):
        Y = X @ qr(Xt @ qr(Y))
    Q = qr(Y)
    Uh, S, Vt = np.linalg.svd(np.swapaxes(Q, -1, -2) @ X)
    U = (Q @ Uh.astype(np.float32))[..., :k].astype(np.float32)
    S = S[..., :k].astype(np.float32)
    Vt = Vt[..., :k, :].astype(np.float32)
    if flip_signs:
        col = np.argmax(np.abs(Vt), axis=-1)
        sg = np.sign(np.take_along_axis(Vt, col[..., None], axis=-1))[..., 0]
        sg = np.where(sg == 0, 1.0, sg).astype(np.float32)
        Vt = Vt * sg[..., :, None]
        U = U * sg[..., None, :]
    if not batched:
        return U[0], S[0], Vt[0]
    return U, S, Vt


# --------------------------------------------------------------------------
# The reference's kernels compiled for the host (oracle/_ref, see build_ref.py)
# --------------------------------------------------------------------------

_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def _reflib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise RuntimeError("oracle/_ref/libmlxref.so is not built (needs the reference tree)")
        lib = ctypes.CDLL(REF_LIB)
        lib.mlxref_run.restype = ctypes.c_int
        lib.mlxref_run.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_uint, ctypes.c_uint, ctypes.c_uint, ctypes.c_int]
        _ref = lib
    return _ref


def _run_ref(name, in0, in1, outs, K, M, B, nthreads):
    """mlxref_run with up to four output arrays."""
    arr = (ctypes.c_void_p * 4)(*[(o.ctypes.data if o is not None else None) for o in
                                  (list(outs) + [None] * (4 - len(outs)))])
    return _reflib().mlxref_run(_REF_IDS[name], _p(in0), _p(in1), arr, K, M, B, _threads(nthreads))


# ids follow the order of oracle.build_ref.KERNELS
_REF_IDS = {"cholesky_solve": 0, "cholesky": 1, "tril_solve": 2, "triu_solve": 3,
            "cholesky_solve_tg": 4, "cholesky_tg": 5, "tril_solve_tg": 6, "triu_solve_tg": 7,
            "cholesky_solve_lg": 8, "tril_solve_lg": 9, "triu_solve_lg": 10,
            "lu_solve": 11, "lu_solve_lg": 12, "qr": 13, "qr_tg": 14}


def _tier_tag(k):
    """_metal_kernels.py:523-528."""
    return "" if k <= 32 else ("_tg" if k <= SHARED_K_MAX else "_lg")


def ref_solve_small(A, b, nthreads=None, return_L=False):
    """The reference's fused cholesky_solve kernel (tier by k, _metal_kernels.py:536-559)
    run on host threads. k <= 128."""
    A = _f32(A)
    b3, was_2d = _rhs(b)
    B, k, _ = A.shape
    m = b3.shape[-1]
    if k > MAX_GPU_K:
        raise ValueError("the reference's small kernels stop at k = 128")
    L = np.empty_like(A)
    x = np.empty_like(b3)
    rc = _run_ref("cholesky_solve" + _tier_tag(k), A, b3, (L, x), k, m, B, nthreads)
    _check(rc, "mlxref cholesky_solve")
    x = x[..., 0] if was_2d else x
    return (x, L) if return_L else x


def ref_cholesky_small(A, nthreads=None):
    """The reference's cholesky kernel (ST for k <= 32 or k > 80, else TG; :562-590)."""
    A = _f32(A)
    B, k, _ = A.shape
    name = "cholesky" if (k <= 32 or k > SHARED_K_MAX) else "cholesky_tg"
    L = np.empty_like(A)
    _check(_run_ref(name, A, None, (L,), k, 0, B, nthreads), "mlxref cholesky")
    return L


def ref_tri_solve(L, b, upper=False, nthreads=None):
    """The reference's tril_solve / triu_solve kernels (tier by k)."""
    L = _f32(L)
    b3, was_2d = _rhs(b)
    B, k, _ = L.shape
    m = b3.shape[-1]
    x = np.empty_like(b3)
    name = ("triu_solve" if upper else "tril_solve") + _tier_tag(k)
    _check(_run_ref(name, L, b3, (x,), k, m, B, nthreads), "mlxref tri solve")
    return x[..., 0] if was_2d else x


def ref_lu_solve(A, b, nthreads=None):
    """The reference's solve_lu kernels (_metal_kernels.py:917-969): the
    single-thread LU for k <= 32, the large single-thread LU above."""
    A = _f32(A)
    b3, was_2d = _rhs(b)
    B, k, _ = A.shape
    m = b3.shape[-1]
    LU = np.empty_like(A)
    piv = np.empty((B, k), np.uint32)
    x = np.empty_like(b3)
    if k <= 32:
        rc = _run_ref("lu_solve", A, b3, (LU, piv, x), k, m, B, nthreads)
    else:
        scratch = np.empty((B, k), np.float32)
        rc = _run_ref("lu_solve_lg", A, b3, (LU, piv, scratch, x), k, m, B, nthreads)
    _check(rc, "mlxref lu_solve")
    return x[..., 0] if was_2d else x


def ref_qr(A, nthreads=None):
    """The reference's Householder QR kernels (_metal_kernels.py:641-694): the
    single-thread kernel for k < 12, the threadgroup kernel for 12 <= k <= 63
    (run with one thread per group). Returns (Q, R)."""
    A = _f32(A)
    B, k, _ = A.shape
    if k > QR_SHARED_K_MAX:
        raise ValueError("the reference's QR kernels stop at k = 63 (CPU LAPACK above)")
    Q, R = np.empty_like(A), np.empty_like(A)
    tau = np.empty((B, k), np.float32)
    name = "qr" if k < 12 else "qr_tg"
    _check(_run_ref(name, A, None, (Q, R, tau), k, 0, B, nthreads), "mlxref qr")
    return Q, R


# --------------------------------------------------------------------------
# LAPACK (numpy's OpenBLAS) over host threads
# --------------------------------------------------------------------------

_lap = None


def _lapack():
    global _lap
    if _lap is None:
        if not os.path.exists(LAPACK_LIB):
            build()
        nd = os.path.join(os.path.dirname(np.__file__), "..", "numpy.libs")
        cands = sorted(glob.glob(os.path.join(nd, "libscipy_openblas64_*.so")))
        if not cands:
            raise RuntimeError("numpy's OpenBLAS (ILP64) not found")
        ob = ctypes.CDLL(cands[0], mode=ctypes.RTLD_GLOBAL)
        try:
            ob.scipy_openblas_set_num_threads64_(ctypes.c_int(1))
        except AttributeError:
            pass
        lib = ctypes.CDLL(LAPACK_LIB)
        lib.lapack_posv_batch.restype = ctypes.c_int64
        lib.lapack_posv_batch.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                                                  ctypes.c_int]
        potrf = ctypes.cast(ob.scipy_spotrf_64_, ctypes.c_void_p)
        potrs = ctypes.cast(ob.scipy_spotrs_64_, ctypes.c_void_p)
        _lap = (lib, potrf, potrs, ob)
    return _lap


def lapack_posv(A, b, nthreads=None, return_logdet=True):
    """spotrf + spotrs per matrix (+ logdet), batch split over host threads."""
    lib, potrf, potrs, _ = _lapack()
    A = _f32(A)
    b3, was_2d = _rhs(b)
    B, n, _ = A.shape
    m = b3.shape[-1]
    x = np.empty_like(b3)
    ld = np.empty(B, np.float32)
    bad = lib.lapack_posv_batch(potrf, potrs, _p(A), _p(b3), _p(x), _p(ld), B, n, m, _threads(nthreads))
    if bad:
        raise np.linalg.LinAlgError(f"{bad} matrices not positive definite")
    x = x[..., 0] if was_2d else x
    return (x, ld) if return_logdet else x
