"""Randomized truncated SVD on the GPU: ``randomized_svd`` and the
sklearn-style ``TruncatedSVD`` of src/mlx_addons/linalg/_svd.py.

Algorithm (Halko, Martinsson and Tropp 2011, Algorithm 4.4, as in
_svd.py:48-175), batched over a leading dimension:

    Omega ~ N(0, 1) (batch, m, k + p)      numpy default_rng(random_state),
                                           the reference's draw (:124-126)
    Y = X Omega
    n_iter times: Y = X thin_qr(X^T thin_qr(Y))
    Q = thin_qr(Y);  B = Q^T X;  U_hat, S, Vt = svd(B);  U = Q U_hat
                                           (svd(B) through B^T = Qb Rb and
                                           the kp x kp svd of Rb^T)
    keep the top k, and flip each Vt row so its largest-|.| entry is positive
    (sklearn's svd_flip, :155-172).

The reference runs the thin QR and the small SVD on the CPU stream (:28-45,
:141-145). Here every step stays on the GPU. The thin QR is a shifted
Cholesky-QR (after Fukaya, Kannan, Nakatsukasa, Yamamoto and Yanagisawa
2020): three passes on the Gram matrix shifted by 1e-4 times its largest
diagonal entry, then one plain pass. Each pass is a Gram product G = Q^T Q
and Q <- Q L^{-T}, with L = cholesky(G) from libb2c's batched Cholesky
(b2c_potrf) and L^{-1} from its triangular solve (b2c_trsm against the
identity); the two products are cuBLAS GEMMs in float32. A pass multiplies Q
by a triangular matrix, so the span never changes. The shift keeps every
pivot above sqrt(1e-4) of the largest column, far above the Gram's rounding
error, so a numerically singular Gram (Y of rank below k + p, or
ill-conditioned) cannot make the factor blow up; each shifted pass maps a
direction of relative size t to t / sqrt(t^2 + 1e-4), which lifts directions
of Y that are pure rounding noise to unit length in three passes (they play
the part of the arbitrary orthonormal completion a Householder QR returns),
and the plain pass leaves Q orthonormal to working precision. Only an
exactly zero column stays zero. The small SVD of B is torch.linalg.svd on the
device.

Inputs: numpy arrays (or anything numpy converts) give numpy results, as the
reference returns; CUDA tensors give CUDA tensors on the same device.
"""

from __future__ import annotations

from typing import Optional, Tuple

import numpy as np
import torch

def _cholesky_dev(G):
    from . import _posv_dev
    _, L, _ = _posv_dev(G.contiguous(), None, False, True, False)
    return L


_EYES = {}


def _eye(B, k, dev):
    """(B, k, k) identity, cached per shape and device (never written)."""
    key = (B, k, str(dev))
    e = _EYES.get(key)
    if e is None:
        e = torch.eye(k, device=dev, dtype=torch.float32).expand(B, k, k).contiguous()
        _EYES[key] = e
    return e


def _tril_inverse_dev(L):
    from . import _trsm_dev
    B, k, _ = L.shape
    return _trsm_dev(L, _eye(B, k, L.device), 0)


_QR_SHIFT = 1e-4     # relative Gram shift of the shifted passes
_QR_SHIFTED_PASSES = 3


def thin_qr(Y: torch.Tensor) -> torch.Tensor:
    """Orthonormal basis Q (batch, n, kp) of the columns of a CUDA Y
    (batch, n, kp), n >= kp, by shifted Cholesky-QR (see the module
    docstring). Replaces _svd.py:28-45 (MLX CPU Householder QR)."""
    if Y.dim() != 3 or not Y.is_cuda:
        raise ValueError("thin_qr expects a CUDA tensor of shape (batch, n, kp)")
    B, n, kp = Y.shape
    Q = Y.float().contiguous()
    eye = _eye(B, kp, Q.device)
    for it in range(_QR_SHIFTED_PASSES + 1):
        G = torch.bmm(Q.transpose(1, 2), Q)
        if it < _QR_SHIFTED_PASSES:
            shift = _QR_SHIFT * G.diagonal(dim1=1, dim2=2).amax(-1)
            G = G + shift[:, None, None] * eye
        Linv = _tril_inverse_dev(_cholesky_dev(G))
        Q = torch.bmm(Q, Linv.transpose(1, 2))
    return Q


def _orth(Y):
    """Orthonormal basis of Y's columns: shifted Cholesky-QR for tall Y;
    the reduced QR of a wide Y (n < kp) has only n columns."""
    if Y.shape[1] >= Y.shape[2]:
        return thin_qr(Y)
    return torch.linalg.qr(Y)[0]


def _flip_signs(U, Vt):
    """svd_flip on Vt rows (_svd.py:155-172): the largest-|.| entry (first
    one on ties) of every row of Vt becomes positive."""
    idx = torch.argmax(Vt.abs(), dim=-1, keepdim=True)
    s = torch.sign(torch.gather(Vt, -1, idx))
    s = torch.where(s == 0, torch.ones_like(s), s)
    return U * s.transpose(1, 2), Vt * s


def randomized_svd(
    X,
    n_components: int,
    *,
    n_oversamples: int = 10,
    n_iter: int = 4,
    random_state: Optional[int] = 42,
    flip_signs: bool = True,
) -> Tuple:
    """Randomized truncated SVD: (U, S, Vt) of rank n_components for X of
    shape (n, m) or (batch, n, m). Same parameters, defaults, random draw and
    return shapes as src/mlx_addons/linalg/_svd.py:48-175."""
    from . import _require_cuda

    on_device = isinstance(X, torch.Tensor) and X.is_cuda
    if isinstance(X, torch.Tensor):
        Xt = X.detach().float().contiguous()
    else:
        Xt = torch.from_numpy(np.ascontiguousarray(np.asarray(X, dtype=np.float32)))
    batched = Xt.dim() == 3
    if not batched:
        if Xt.dim() != 2:
            raise ValueError(f"randomized_svd expects a 2-D or 3-D array, got shape {tuple(Xt.shape)}")
        Xt = Xt[None]
    B, n, m = Xt.shape
    k = min(int(n_components), min(n, m))
    kp = k + int(n_oversamples)
    if not on_device:
        _require_cuda()
        Xt = Xt.to(torch.device("cuda", torch.cuda.current_device()))
    dev = Xt.device

    omega = np.random.default_rng(random_state).standard_normal((B, m, kp)).astype(np.float32)
    with torch.cuda.device(dev):
        Om = torch.from_numpy(omega).to(dev)
        Y = torch.bmm(Xt, Om)
        Xtt = Xt.transpose(1, 2)
        for _ in range(int(n_iter)):
            Z = torch.bmm(Xtt, _orth(Y))
            Y = torch.bmm(Xt, _orth(Z))
        Q = _orth(Y)
        Bt = torch.bmm(Xtt, Q)  # B^T = X^T Q, (batch, m, kp)
        if m >= Bt.shape[2]:
            # B^T = Qb Rb, so B = Rb^T Qb^T and svd(B) follows from the
            # kp x kp svd(Rb^T) = Ur S Vr^T: U_hat = Ur, Vt = (Qb Vr)^T
            Qb = _orth(Bt)
            Rt = torch.bmm(Bt.transpose(1, 2), Qb)  # Rb^T = B Qb, (batch, kp, kp)
            U_hat, S, Vr_t = torch.linalg.svd(Rt)
            Vt = torch.bmm(Vr_t, Qb.transpose(1, 2))
        else:
            U_hat, S, Vt = torch.linalg.svd(Bt.transpose(1, 2), full_matrices=False)
        U = torch.bmm(Q, U_hat)
        U, S, Vt = U[:, :, :k], S[:, :k], Vt[:, :k, :]
        if flip_signs:
            U, Vt = _flip_signs(U, Vt)
    if not batched:
        U, S, Vt = U[0], S[0], Vt[0]
    if on_device:
        return U.contiguous(), S.contiguous(), Vt.contiguous()
    return U.cpu().numpy(), S.cpu().numpy(), Vt.cpu().numpy()


class TruncatedSVD:
    """sklearn-compatible wrapper around randomized_svd (_svd.py:178-250):
    fit / transform / fit_transform, ``components_`` (n_components,
    n_features) and ``singular_values_`` (n_components,)."""

    def __init__(self, n_components: int = 2, *, n_oversamples: int = 10, n_iter: int = 4,
                 random_state: Optional[int] = 42):
        self.n_components = n_components
        self.n_oversamples = n_oversamples
        self.n_iter = n_iter
        self.random_state = random_state

    def fit(self, X, y=None) -> "TruncatedSVD":
        _U, S, Vt = randomized_svd(X, n_components=self.n_components, n_oversamples=self.n_oversamples,
                                   n_iter=self.n_iter, random_state=self.random_state)
        self.components_ = Vt
        self.singular_values_ = S
        return self

    def transform(self, X):
        if isinstance(X, torch.Tensor) and X.is_cuda:
            C = self.components_
            C = C if isinstance(C, torch.Tensor) else torch.from_numpy(C).to(X.device)
            return X.float() @ C.T
        Xn = np.ascontiguousarray(np.asarray(X, dtype=np.float32))
        C = self.components_.cpu().numpy() if isinstance(self.components_, torch.Tensor) else self.components_
        return Xn @ C.T

    def fit_transform(self, X, y=None):
        return self.fit(X).transform(X)
