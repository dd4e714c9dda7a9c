"""Batched SPD linear algebra on NVIDIA B200 — drop-in for ``mlx_addons.linalg``.

Same names, argument meanings, batch semantics and return shapes as the
reference's public API (``src/mlx_addons/linalg/__init__.py:33-68``) for the
batched Cholesky path:

    solve(A, b)         x = A^{-1} b for SPD A (B, k, k), b (B, k, m) or (B, k)
    cholesky(A)         lower factor L, upper triangle zero
    tril_solve(L, b)    L x = b
    triu_solve(L, b)    L^T x = b (takes the LOWER factor, like the reference)
    logdet_spd(A)       2 * sum(log(diag L)), shape (B,)
    slogdet(A)          (sign, log|det|) through partial-pivot LU, A (..., n, n)
    det(A)              sign * exp(log|det|)
    solve_lu(A, b)      x = A^{-1} b for general square A, partial-pivot LU
    qr(A)               Householder (Q, R) of square A (B, k, k) or (k, k)
    randomized_svd      truncated SVD (U, S, Vt), X (n, m) or (B, n, m);
    TruncatedSVD        and its sklearn-style wrapper (_svd.py)
    solve_cholesky      alias of solve (the reference's small-kernel solve)

plus one fused extension, ``cho_solve_logdet(A, b, return_L=False)``, which
returns x and logdet (and L) from ONE pass over A — the reference needs a
separate factorisation for each of cholesky, solve and logdet_spd.

Inputs may be torch tensors, numpy arrays or any ``__dlpack__`` object; they
are cast to float32 (as the reference casts, ``_metal_kernels.py:541``).
CUDA tensors are processed on their device, on the current stream, and the
results stay there. Host (CPU) inputs are streamed through the current CUDA
device in pipelined chunks and the results come back to the host; numpy in
gives numpy out. Every computation runs in the CUDA kernels of libb2c — there
is no CPU fallback, and without a CUDA device the functions raise.

Differences from the reference, all supersets: the k <= 128 assertion of
tril_solve / triu_solve / solve_cholesky / solve_lu
(``_metal_kernels.py:539,596,620,932``) is
lifted, and mismatched shapes raise ValueError instead of reading garbage.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _lib

__all__ = [
    "solve", "cholesky", "solve_cholesky", "solve_lu", "qr", "tril_solve", "triu_solve", "det", "slogdet", "logdet_spd",
    "cho_solve_logdet", "randomized_svd", "TruncatedSVD", "MAX_GPU_K", "SHARED_K_MAX",
]

# Reference constants (src/mlx_addons/linalg/_metal_kernels.py:19-20). They
# are kept for API compatibility; neither is a limit here.
MAX_GPU_K = 128
SHARED_K_MAX = 80

# Host inputs are moved in chunks of about this many bytes of A.
_HOST_CHUNK_BYTES = 32 << 20


# ---------------------------------------------------------------------------
# argument plumbing
# ---------------------------------------------------------------------------

def _as_tensor(x, name):
    if isinstance(x, torch.Tensor):
        return x, "torch"
    if isinstance(x, np.ndarray):
        return torch.from_numpy(np.ascontiguousarray(x)), "numpy"
    if hasattr(x, "__dlpack__"):
        return torch.from_dlpack(x), "dlpack"
    raise TypeError(f"{name}: expected a torch tensor, numpy array or DLPack object, got {type(x).__name__}")


def _f32(t):
    if t.dtype != torch.float32:
        t = t.to(torch.float32)
    return t.contiguous()


def _check_square3(A, name, what="A"):
    if A.dim() != 3:
        raise ValueError(f"{name}: {what} must have shape (batch, k, k), got {tuple(A.shape)}")
    if A.shape[1] != A.shape[2]:
        raise ValueError(f"{name}: {what} must be square in its last two dims, got {tuple(A.shape)}")


def _prep_b(b, B, k, name):
    """(B, k) -> (B, k, 1) like _prep_b (_metal_kernels.py:489-496)."""
    if b.dim() == 2:
        b3, was_2d = b.unsqueeze(-1), True
    elif b.dim() == 3:
        b3, was_2d = b, False
    else:
        raise ValueError(f"{name}: b must have shape (batch, k) or (batch, k, m), got {tuple(b.shape)}")
    if b3.shape[0] != B or b3.shape[1] != k:
        raise ValueError(f"{name}: b has shape {tuple(b.shape)} but A implies batch={B}, k={k}")
    return b3, was_2d


def _ptr(t):
    """Device-accessible address of a CUDA tensor or of a pinned, mapped host
    tensor (the kernels then read / write it across PCIe)."""
    if t is None:
        return None
    if t.is_cuda:
        return t.data_ptr()
    dp = ctypes.c_void_p()
    _lib.check(_lib.load().b2c_host_device_pointer(t.data_ptr(), ctypes.byref(dp)), "b2c_host_device_pointer")
    return dp.value


def _mappable(t):
    if t.is_cuda or not t.is_pinned():
        return False
    dp = ctypes.c_void_p()
    return _lib.load().b2c_host_device_pointer(t.data_ptr(), ctypes.byref(dp)) == 0


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("mlx_addons_b200.linalg needs a CUDA device (B200); there is no CPU fallback")


def _finish(outs, kind):
    if kind == "numpy":
        return tuple(None if o is None else o.numpy() for o in outs)
    return outs


def _host_call(dev_fn, inputs):
    """Run ``dev_fn`` over host tensors: chunks of the batch alternate between
    two streams, so the copy-in of chunk i+1 overlaps chunk i's kernel and
    copy-out. Outputs land in pinned host tensors."""
    _require_cuda()
    dev = torch.device("cuda", torch.cuda.current_device())
    B = inputs[0].shape[0]
    per = max(1, inputs[0][0].numel() * 4) if B else 1
    step = max(1, min(B, _HOST_CHUNK_BYTES // per)) if B else 1
    bounds = [(lo, min(B, lo + step)) for lo in range(0, B, step)] or [(0, 0)]
    streams = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]
    outs = None
    for ci, (lo, hi) in enumerate(bounds):
        s = streams[ci % 2]
        with torch.cuda.stream(s):
            d_in = [x[lo:hi].to(dev, non_blocking=True) for x in inputs]
            d_out = dev_fn(*d_in)
            if outs is None:
                outs = [None if d is None else
                        torch.empty((B,) + tuple(d.shape[1:]), dtype=d.dtype, pin_memory=True) for d in d_out]
            for o, d in zip(outs, d_out):
                if o is not None:
                    o[lo:hi].copy_(d, non_blocking=True)
    for s in streams:
        s.synchronize()
    return outs


# ---------------------------------------------------------------------------
# device implementations (CUDA tensors in, CUDA tensors out)
# ---------------------------------------------------------------------------

def _out(shape, like):
    """Output buffer next to `like`: on its CUDA device, or pinned host memory
    for the zero-copy host path."""
    if like.is_cuda:
        return torch.empty(shape, device=like.device, dtype=torch.float32)
    return torch.empty(shape, dtype=torch.float32, pin_memory=True)


def _posv_dev(A, b3, want_x, want_L, want_logdet):
    lib = _lib.load()
    dev = A.device if A.is_cuda else torch.device("cuda", torch.cuda.current_device())
    B, k = A.shape[0], A.shape[1]
    m = b3.shape[2] if (b3 is not None and want_x) else 0
    x = _out(tuple(b3.shape), A) if want_x else None
    L = _out(tuple(A.shape), A) if want_L else None
    ld = _out((B,), A) if want_logdet else None
    with torch.cuda.device(dev):
        op = _lib.OP_POSV if m else _lib.OP_POTRF
        ws_bytes = 0 if L is not None else int(lib.b2c_workspace_size(op, B, k, m))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        if m:
            rc = lib.b2c_posv(_ptr(A), _ptr(b3), _ptr(x), _ptr(L), _ptr(ld), B, k, m, _ptr(ws), ws_bytes,
                              _stream(dev))
            _lib.check(rc, "b2c_posv")
        elif B and (L is not None or ld is not None):
            rc = lib.b2c_potrf(_ptr(A), _ptr(L), _ptr(ld), B, k, _ptr(ws), ws_bytes, _stream(dev))
            _lib.check(rc, "b2c_potrf")
        if not A.is_cuda:
            torch.cuda.current_stream(dev).synchronize()
    return x, L, ld


def _trsm_dev(L, b3, transpose):
    lib = _lib.load()
    dev = L.device
    B, k, m = b3.shape
    x = torch.empty_like(b3)
    with torch.cuda.device(dev):
        rc = lib.b2c_trsm(_ptr(L), _ptr(b3), _ptr(x), B, k, m, int(transpose), _stream(dev))
    _lib.check(rc, "b2c_trsm")
    return x


def _slogdet_dev(A3):
    lib = _lib.load()
    dev = A3.device if A3.is_cuda else torch.device("cuda", torch.cuda.current_device())
    B, n = A3.shape[0], A3.shape[1]
    sign = _out((B,), A3)
    lad = _out((B,), A3)
    with torch.cuda.device(dev):
        ws_bytes = int(lib.b2c_workspace_size(_lib.OP_SLOGDET, B, n, 0))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        rc = lib.b2c_slogdet(_ptr(A3), _ptr(sign), _ptr(lad), B, n, _ptr(ws), ws_bytes, _stream(dev))
        _lib.check(rc, "b2c_slogdet")
        if not A3.is_cuda:
            torch.cuda.current_stream(dev).synchronize()
    return sign, lad


def _gesv_dev(A, b3):
    lib = _lib.load()
    dev = A.device if A.is_cuda else torch.device("cuda", torch.cuda.current_device())
    B, k, m = b3.shape
    x = _out(tuple(b3.shape), A)
    with torch.cuda.device(dev):
        ws_bytes = int(lib.b2c_workspace_size(_lib.OP_GESV, B, k, m))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        rc = lib.b2c_gesv(_ptr(A), _ptr(b3), _ptr(x), B, k, m, _ptr(ws), ws_bytes, _stream(dev))
        _lib.check(rc, "b2c_gesv")
        if not A.is_cuda:
            torch.cuda.current_stream(dev).synchronize()
    return x


def _qr_dev(A):
    lib = _lib.load()
    dev = A.device if A.is_cuda else torch.device("cuda", torch.cuda.current_device())
    B, k = A.shape[0], A.shape[1]
    Q = _out(tuple(A.shape), A)
    R = _out(tuple(A.shape), A)
    with torch.cuda.device(dev):
        ws_bytes = int(lib.b2c_workspace_size(_lib.OP_QR, B, k, 0))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes else None
        rc = lib.b2c_qr(_ptr(A), _ptr(Q), _ptr(R), B, k, _ptr(ws), ws_bytes, _stream(dev))
        _lib.check(rc, "b2c_qr")
        if not A.is_cuda:
            torch.cuda.current_stream(dev).synchronize()
    return Q, R


def _dispatch(dev_fn, tensors, zero_copy=False):
    """Device tensors run in place on their device. Host tensors that are
    pinned and mapped are handed to the kernels directly when the kernel reads
    each input once (``zero_copy``): the data crosses PCIe inside the kernel,
    and the k <= 64 tiers fetch only the lower blocks of A. Other host
    tensors go through the pipelined staging path."""
    if tensors[0].is_cuda:
        dev = tensors[0].device
        tensors = [t if t.device == dev else t.to(dev) for t in tensors]
        return dev_fn(*tensors)
    _require_cuda()
    tensors = [t.cpu() for t in tensors]
    if zero_copy and all(_mappable(t) for t in tensors):
        return dev_fn(*tensors)
    return tuple(_host_call(dev_fn, tensors))


# ---------------------------------------------------------------------------
# public API
# ---------------------------------------------------------------------------

def cho_solve_logdet(A, b, return_L: bool = False):
    """One pass over A: x = A^{-1} b, logdet = 2 sum log diag L (and L).

    The fused form of ``cholesky`` + ``solve`` + ``logdet_spd`` on the same A."""
    At, kind = _as_tensor(A, "cho_solve_logdet")
    bt, _ = _as_tensor(b, "cho_solve_logdet")
    At = _f32(At)
    _check_square3(At, "cho_solve_logdet")
    B, k = At.shape[0], At.shape[1]
    b3, was_2d = _prep_b(_f32(bt), B, k, "cho_solve_logdet")
    x, L, ld = _dispatch(lambda a, bb: _posv_dev(a, bb, True, return_L, True), [At, b3],
                         zero_copy=not (return_L and k > 64))
    if was_2d:
        x = x.squeeze(-1)
    return _finish((x, ld, L) if return_L else (x, ld), kind)


def solve(A, b):
    """Solve A x = b for batched SPD A (any k); x has b's shape.

    Mirrors ``solve = blocked_solve`` (src/mlx_addons/linalg/__init__.py:48,
    _blocked.py:140-217): A (B, k, k), b (B, k, m) or (B, k)."""
    At, kind = _as_tensor(A, "solve")
    bt, _ = _as_tensor(b, "solve")
    At = _f32(At)
    _check_square3(At, "solve")
    B, k = At.shape[0], At.shape[1]
    b3, was_2d = _prep_b(_f32(bt), B, k, "solve")
    x, _, _ = _dispatch(lambda a, bb: _posv_dev(a, bb, True, False, False), [At, b3], zero_copy=True)
    if was_2d:
        x = x.squeeze(-1)
    return _finish((x,), kind)[0]


solve_cholesky = solve


def cholesky(A):
    """Lower Cholesky factor of batched SPD A (B, k, k), upper triangle zero.

    Mirrors ``cholesky = blocked_cholesky`` (src/mlx_addons/linalg/__init__.py:49,
    _blocked.py:34-137); non-positive pivots are clamped to sqrt(1e-12)."""
    At, kind = _as_tensor(A, "cholesky")
    At = _f32(At)
    _check_square3(At, "cholesky")
    _, L, _ = _dispatch(lambda a: _posv_dev(a, None, False, True, False), [At], zero_copy=At.shape[1] <= 64)
    return _finish((L,), kind)[0]


def logdet_spd(A):
    """2 * sum(log(diag(cholesky(A)))) for batched SPD A (B, k, k) -> (B,).

    Mirrors src/mlx_addons/linalg/_det.py:51-67, :100-113."""
    At, kind = _as_tensor(A, "logdet_spd")
    At = _f32(At)
    _check_square3(At, "logdet_spd")
    _, _, ld = _dispatch(lambda a: _posv_dev(a, None, False, False, True), [At], zero_copy=True)
    return _finish((ld,), kind)[0]


def _tri(L, b, transpose, name):
    Lt, kind = _as_tensor(L, name)
    bt, _ = _as_tensor(b, name)
    Lt = _f32(Lt)
    _check_square3(Lt, name, "L")
    B, k = Lt.shape[0], Lt.shape[1]
    b3, was_2d = _prep_b(_f32(bt), B, k, name)
    (x,) = _dispatch(lambda l, bb: (_trsm_dev(l, bb, transpose),), [Lt, b3])
    if was_2d:
        x = x.squeeze(-1)
    return _finish((x,), kind)[0]


def tril_solve(L, b):
    """Solve L x = b, L lower triangular (B, k, k) (_metal_kernels.py:593-614)."""
    return _tri(L, b, 0, "tril_solve")


def triu_solve(L, b):
    """Solve L^T x = b with the LOWER factor L (_metal_kernels.py:617-638)."""
    return _tri(L, b, 1, "triu_solve")


def slogdet(A):
    """(sign, log|det|) of square matrices A (..., n, n) via partial-pivot LU.

    Mirrors src/mlx_addons/linalg/_det.py:17-48, :84-97 (LAPACK getrf on the
    CPU stream there; batched LU kernels here)."""
    At, kind = _as_tensor(A, "slogdet")
    At = _f32(At)
    if At.dim() < 2 or At.shape[-1] != At.shape[-2]:
        raise ValueError(f"slogdet: A must have shape (..., n, n), got {tuple(At.shape)}")
    lead, n = tuple(At.shape[:-2]), At.shape[-1]
    A3 = At.reshape((-1, n, n)).contiguous()
    sign, lad = _dispatch(lambda a: _slogdet_dev(a), [A3], zero_copy=True)
    sign, lad = sign.reshape(lead), lad.reshape(lead)
    return _finish((sign, lad), kind)


def solve_lu(A, b):
    """Solve A x = b for batched general square A (B, k, k) through LU with
    partial pivoting; x has b's shape (_metal_kernels.py:917-969). Any k."""
    At, kind = _as_tensor(A, "solve_lu")
    bt, _ = _as_tensor(b, "solve_lu")
    At = _f32(At)
    _check_square3(At, "solve_lu")
    B, k = At.shape[0], At.shape[1]
    b3, was_2d = _prep_b(_f32(bt), B, k, "solve_lu")
    (x,) = _dispatch(lambda a, bb: (_gesv_dev(a, bb),), [At, b3], zero_copy=True)
    if was_2d:
        x = x.squeeze(-1)
    return _finish((x,), kind)[0]


def qr(A):
    """Householder QR of square matrices: (Q, R) with A = Q R, R upper
    triangular; A (B, k, k), or (k, k) for one matrix
    (_metal_kernels.py:641-694). Any k, all on the GPU (the reference moves
    k > 63 to CPU LAPACK, whose convention is kept above k = 63)."""
    At, kind = _as_tensor(A, "qr")
    At = _f32(At)
    squeeze = At.dim() == 2
    if squeeze:
        At = At.unsqueeze(0)
    if At.dim() != 3 or At.shape[1] != At.shape[2]:
        raise ValueError(f"qr requires square matrices, got {tuple(At.shape)}")
    Q, R = _dispatch(lambda a: _qr_dev(a), [At.contiguous()], zero_copy=True)
    if squeeze:
        Q, R = Q[0], R[0]
    return _finish((Q, R), kind)


def det(A):
    """sign * exp(log|det|) (src/mlx_addons/linalg/_det.py:70-81)."""
    sign, lad = slogdet(A)
    if isinstance(sign, np.ndarray):
        return sign * np.exp(lad)
    return sign * torch.exp(lad)


from ._svd import TruncatedSVD, randomized_svd  # noqa: E402  (uses the device helpers above)
