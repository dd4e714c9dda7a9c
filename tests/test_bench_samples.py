"""The CPU baseline and the reference arm of bench.py time the same kind of
input as the GPU arm: SPD matrices for the Cholesky workloads (every one of
them factors in float64), general matrices for LU / QR, well-conditioned
lower-triangular ones for the triangular solve."""

import numpy as np
import pytest

bench = pytest.importorskip("bench")


@pytest.mark.parametrize("name", list(bench.WORKLOADS))
@pytest.mark.parametrize("op", ["posv", "seq3"])
def test_cholesky_samples_are_spd(name, op):
    A, b = bench._cpu_sample(bench.WORKLOADS[name], 6, op)
    assert A.dtype == np.float32 and A.shape[0] == 6 and b.shape[:2] == A.shape[:2]
    np.testing.assert_array_equal(A, np.swapaxes(A, 1, 2))
    np.linalg.cholesky(A.astype(np.float64))  # raises if any matrix is not positive definite


def test_triangular_samples_are_lower_and_nonsingular():
    L, _ = bench._cpu_sample(bench.WORKLOADS["c4_k256"], 4, "trsm")
    assert np.all(np.triu(L, 1) == 0)
    assert np.all(np.abs(np.diagonal(L, axis1=1, axis2=2)) >= 1.0)
