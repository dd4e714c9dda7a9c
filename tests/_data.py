"""Seeded synthetic inputs shared by the tests and the golden-fixture script.

The SPD generator follows the workload definition of the batched-solve
benchmark: G ~ N(0, 1) float32 of shape (B, k, k) from
``numpy.random.default_rng(seed)``, A = G G^T / k + eps I computed in float32,
and b ~ N(0, 1) of shape (B, k, m) from the same generator. ``make_spd_ref``
is the reference test-suite helper (``tests/test_linalg.py:11-21``: float64
G G^T + 2 I, seeds 42 / 43).
"""

from __future__ import annotations

import numpy as np


def spd_batch(B: int, k: int, m: int = 1, eps: float = 1.0, seed: int = 0):
    rng = np.random.default_rng(seed)
    G = rng.standard_normal((B, k, k), dtype=np.float32)
    A = np.matmul(G, G.transpose(0, 2, 1)) / np.float32(k)
    A += np.float32(eps) * np.eye(k, dtype=np.float32)
    b = rng.standard_normal((B, k, m), dtype=np.float32)
    return np.ascontiguousarray(A, dtype=np.float32), np.ascontiguousarray(b, dtype=np.float32)


def make_spd_ref(batch: int, k: int, seed: int = 42) -> np.ndarray:
    rng = np.random.default_rng(seed)
    A = rng.standard_normal((batch, k, k)).astype(np.float64)
    return A @ np.transpose(A, (0, 2, 1)) + np.eye(k, dtype=np.float64) * 2.0


def make_rhs_ref(batch: int, k: int, m: int = 1, seed: int = 43) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal((batch, k, m)).astype(np.float64)


def with_upper_garbage(A: np.ndarray, seed: int = 7) -> np.ndarray:
    """Overwrite the strict upper triangle with large random values; the
    reference never reads it, so every result must be unchanged."""
    rng = np.random.default_rng(seed)
    k = A.shape[-1]
    iu = np.triu_indices(k, 1)
    out = A.copy()
    out[:, iu[0], iu[1]] = rng.uniform(-1e3, 1e3, size=(A.shape[0], len(iu[0]))).astype(np.float32)
    return out


def general_batch(B: int, n: int, seed: int = 0) -> np.ndarray:
    """Non-symmetric, usually non-singular matrices for slogdet/det."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((B, n, n), dtype=np.float32)


# Workload shapes of the benchmark configurations: (B, k, m, eps).
CONFIGS = {
    "c1_k16": (10_000, 16, 1, 1.0),
    "c2_k64": (10_000, 64, 1, 1.0),
    "c3_k5": (1_000_000, 5, 4, 0.1),
    "c4_k256": (1_000, 256, 8, 1.0),
    "c5_k512": (8_000, 512, 1, 1.0),
}
