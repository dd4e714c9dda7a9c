"""Tolerances and error measures shared by the parity tests.

Floating-point parity bar (float32 throughout):
  * factor:   ||L - L_ref||_F / ||L_ref||_F <= 1e-5 for k <= 80, 5e-5 above
  * solve:    per-matrix backward error ||A x - b||_F / (||A||_F ||x||_F)
              <= 1e-6 for k <= 80, 5e-5 above, evaluated in float64
  * x, logdet against the oracle: relative 1e-5 (k <= 80), 5e-5 above
"""

from __future__ import annotations

import numpy as np


def factor_tol(k: int) -> float:
    return 1e-5 if k <= 80 else 5e-5


def backward_tol(k: int) -> float:
    return 1e-6 if k <= 80 else 5e-5


def rel_fro(a, ref) -> float:
    a = np.asarray(a, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref.ravel())
    return float(np.linalg.norm((a - ref).ravel()) / (den if den > 0 else 1.0))


def rel_fro_per_matrix(a, ref) -> np.ndarray:
    a = np.asarray(a, np.float64).reshape(a.shape[0], -1)
    ref = np.asarray(ref, np.float64).reshape(ref.shape[0], -1)
    den = np.linalg.norm(ref, axis=1)
    den[den == 0] = 1.0
    return np.linalg.norm(a - ref, axis=1) / den


def sym_from_lower(A):
    """The SPD matrix the reference factors: only the lower triangle of A counts."""
    A = np.asarray(A, np.float64)
    low = np.tril(A)
    return low + np.swapaxes(np.tril(A, -1), -1, -2)


def backward_error(A, x, b) -> np.ndarray:
    """Per-matrix ||A x - b||_F / (||A||_F ||x||_F), A symmetrised from its lower triangle."""
    S = sym_from_lower(A)
    x = np.asarray(x, np.float64)
    b = np.asarray(b, np.float64)
    if x.ndim == 2:
        x, b = x[..., None], b[..., None]
    r = np.matmul(S, x) - b
    num = np.linalg.norm(r.reshape(r.shape[0], -1), axis=1)
    den = np.linalg.norm(S.reshape(S.shape[0], -1), axis=1) * np.linalg.norm(x.reshape(x.shape[0], -1), axis=1)
    den[den == 0] = 1.0
    return num / den
