"""GPU parity for the general-matrix rows: solve_lu (partial-pivot LU solve)
and qr (Householder), through libb2c's C ABI, against the oracle and the
golden fixtures from the reference run."""

import numpy as np
import pytest
import torch

from tests._data import general_batch, spd_batch

pytestmark = pytest.mark.gpu

la = pytest.importorskip("mlx_addons_b200.linalg")

DEV = "cuda:0"
F32_EPS = float(np.finfo(np.float32).eps)


def _gpu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _lu_tol(A):
    """Forward-error bound for two float32 LU solves of A that differ only in
    rounding: a small multiple of cond(A) * k * eps."""
    k = A.shape[-1]
    cond = np.linalg.cond(A.astype(np.float64))
    return np.maximum(1e-6, 8.0 * k * cond * F32_EPS)


def _rel_per_matrix(x, ref):
    d = (x.astype(np.float64) - ref).reshape(x.shape[0], -1)
    r = ref.astype(np.float64).reshape(x.shape[0], -1)
    return np.linalg.norm(d, axis=1) / np.maximum(np.linalg.norm(r, axis=1), 1e-30)


def _backward(A, x, b):
    A, x, b = A.astype(np.float64), x.astype(np.float64), b.astype(np.float64)
    if x.ndim == 2:
        x, b = x[..., None], b[..., None]
    r = np.abs(A @ x - b).max(axis=(1, 2))
    s = (np.abs(A) @ np.abs(x) + np.abs(b)).max(axis=(1, 2))
    return r / s


# --------------------------------------------------------------------------
# solve_lu
# --------------------------------------------------------------------------

@pytest.mark.parametrize("k", [1, 2, 3, 5, 8, 16, 31, 32, 33, 48, 64, 100, 128, 150, 224, 225, 256, 300, 500,
                               864, 865])
@pytest.mark.parametrize("m", [1, 3, 9])
def test_solve_lu_vs_oracle(orc, k, m):
    B = 23 if k <= 128 else (5 if k <= 256 else 3)
    A = general_batch(B, k, seed=7000 + k)
    b = np.random.default_rng(7100 + k + m).standard_normal((B, k, m), dtype=np.float32)
    x = _np(la.solve_lu(_gpu(A), _gpu(b)))
    x_ref = orc.lu_solve(A, b)
    assert x.shape == b.shape
    assert np.all(np.isfinite(x))
    assert np.all(_rel_per_matrix(x, x_ref) <= _lu_tol(A))
    assert np.max(_backward(A, x, b)) < 20 * k * F32_EPS


def test_solve_lu_golden(golden):
    n = 0
    for case, g in sorted(golden.items()):
        if not case.startswith("solve_lu_k"):
            continue
        x = _np(la.solve_lu(_gpu(g["A"]), _gpu(g["b"])))
        assert np.all(_rel_per_matrix(x, g["x"]) <= _lu_tol(g["A"])), case
        n += 1
    assert n >= 9
    g = golden["solve_lu_b2d_k10"]
    x = _np(la.solve_lu(_gpu(g["A"]), _gpu(g["b"])))
    assert x.shape == g["x"].shape
    assert np.all(_rel_per_matrix(x[..., None], g["x"][..., None]) <= _lu_tol(g["A"]))


def test_solve_lu_special_cases(golden, orc):
    """A permutation and a singular matrix (zero column and zero row) whose
    eliminations are exact: x bit for bit, inf and NaN where the reference
    has them; and an upper-triangular matrix, to rounding."""
    g = golden["solve_lu_special_k4"]
    x = _np(la.solve_lu(_gpu(g["A"]), _gpu(g["b"])))
    for want in (g["x"], orc.lu_solve(g["A"], g["b"])):
        for i in (0, 1):
            assert np.array_equal(np.isnan(x[i]), np.isnan(want[i]))
            assert np.array_equal(np.nan_to_num(x[i]), np.nan_to_num(want[i]))
        np.testing.assert_allclose(x[2], want[2], rtol=1e-5, atol=1e-6)
    assert not np.all(np.isfinite(g["x"][1]))


@pytest.mark.parametrize("k", [5, 32, 64, 200, 300])
def test_solve_lu_permutations_exact(orc, k):
    rng = np.random.default_rng(k)
    A = np.stack([np.eye(k, dtype=np.float32)[rng.permutation(k)] for _ in range(6)])
    b = rng.integers(-50, 50, size=(6, k, 2)).astype(np.float32)
    x = _np(la.solve_lu(_gpu(A), _gpu(b)))
    assert np.array_equal(x, orc.lu_solve(A, b))
    assert np.array_equal(x, np.swapaxes(A, 1, 2) @ b)


@pytest.mark.parametrize("k", [4, 20, 40, 100, 256, 300])
def test_solve_lu_nonfinite_patterns(orc, k):
    """Zero columns and NaN entries: the pivot search skips NaN and keeps the
    diagonal row of an all-zero column; x is non-finite where the
    reference's is."""
    A = general_batch(4, k, seed=k)
    A[0, :, 1] = 0.0
    A[1] = 0.0
    A[2, k // 2, 0] = np.nan
    b = np.ones((4, k, 1), np.float32)
    x = _np(la.solve_lu(_gpu(A), _gpu(b)))
    x_ref = orc.lu_solve(A, b)
    assert np.array_equal(np.isfinite(x), np.isfinite(x_ref))
    # all-zero A, b = 1: x_last = 1/0 = inf, then 0 * inf = NaN above it
    assert np.isposinf(x[1, -1, 0]) and np.all(np.isnan(x[1, :-1]))
    assert np.all(_rel_per_matrix(x[3:], x_ref[3:]) <= _lu_tol(A[3:]))


@pytest.mark.parametrize("k", [256, 300])
def test_solve_lu_blocked_walks_several_matrices(orc, k):
    """More matrices than resident CTAs of the blocked LU: each CTA reuses
    its scratch slot and row map for several matrices; a sample is checked."""
    B = 2 * 148 * 2 + 5
    A = general_batch(B, k, seed=7800 + k)
    b = np.random.default_rng(7801 + k).standard_normal((B, k, 2), dtype=np.float32)
    x = _np(la.solve_lu(_gpu(A), _gpu(b)))
    idx = np.random.default_rng(k).choice(B, 12, replace=False)
    idx[-1] = B - 1
    x_ref = orc.lu_solve(A[idx], b[idx])
    assert np.all(np.isfinite(x))
    assert np.all(_rel_per_matrix(x[idx], x_ref) <= _lu_tol(A[idx]))


def test_solve_lu_many_matrices_per_warp(orc):
    B, k = 9_001, 16
    A = general_batch(B, k, seed=11)
    b = np.random.default_rng(12).standard_normal((B, k), dtype=np.float32)
    x = _np(la.solve_lu(_gpu(A), _gpu(b)))
    assert x.shape == (B, k)
    assert np.all(_rel_per_matrix(x[..., None], orc.lu_solve(A, b)[..., None]) <= _lu_tol(A))


def test_solve_lu_spd_matches_solve(orc):
    A, b = spd_batch(10, 40, m=2, seed=5)
    np.testing.assert_allclose(_np(la.solve_lu(_gpu(A), _gpu(b))), _np(la.solve(_gpu(A), _gpu(b))),
                               rtol=2e-4, atol=2e-5)


def test_solve_lu_host_inputs(orc):
    A = general_batch(7, 12, seed=3)
    b = np.random.default_rng(4).standard_normal((7, 12, 2), dtype=np.float32)
    x = la.solve_lu(A, b)
    assert isinstance(x, np.ndarray)
    pin_A, pin_b = torch.from_numpy(A).pin_memory(), torch.from_numpy(b).pin_memory()
    xp = la.solve_lu(pin_A, pin_b)
    assert not xp.is_cuda
    assert np.array_equal(xp.numpy(), x)
    assert np.array_equal(x, _np(la.solve_lu(_gpu(A), _gpu(b))))


# --------------------------------------------------------------------------
# qr
# --------------------------------------------------------------------------

def _qr_checks(A, Q, R, Q_ref, R_ref):
    k = A.shape[-1]
    A64, Q64, R64 = A.astype(np.float64), Q.astype(np.float64), R.astype(np.float64)
    assert np.all(np.tril(R, -1) == 0)
    recon = np.abs(Q64 @ R64 - A64).max(axis=(1, 2)) / np.maximum(np.abs(A64).max(axis=(1, 2)), 1e-30)
    assert np.max(recon) < 10 * k * F32_EPS
    orth = np.abs(np.swapaxes(Q64, 1, 2) @ Q64 - np.eye(k)).max(axis=(1, 2))
    assert np.max(orth) < 10 * k * F32_EPS
    tol = _lu_tol(A)
    assert np.all(_rel_per_matrix(Q, Q_ref) <= tol)
    assert np.all(_rel_per_matrix(R, R_ref) <= tol)


@pytest.mark.parametrize("k", [1, 2, 3, 5, 8, 11, 12, 16, 31, 32, 33, 48, 63, 64, 65, 96, 128, 160, 161, 200])
def test_qr_vs_oracle(orc, k):
    B = 13 if k <= 64 else 4
    A = general_batch(B, k, seed=7300 + k)
    Q, R = la.qr(_gpu(A))
    Q, R = _np(Q), _np(R)
    Q_ref, R_ref = orc.qr(A)
    _qr_checks(A, Q, R, Q_ref, R_ref)


def test_qr_golden(golden):
    n = 0
    for case, g in sorted(golden.items()):
        if not case.startswith("qr_k"):
            continue
        Q, R = la.qr(_gpu(g["A"]))
        _qr_checks(g["A"], _np(Q), _np(R), g["Q"], g["R"])
        n += 1
    assert n >= 12
    g = golden["qr_2d_k10"]
    Q, R = la.qr(_gpu(g["A"]))
    assert tuple(Q.shape) == (10, 10) and tuple(R.shape) == (10, 10)
    _qr_checks(g["A"][None], _np(Q)[None], _np(R)[None], g["Q"][None], g["R"][None])


@pytest.mark.parametrize("k", [64, 70, 200])
def test_qr_lapack_convention_keeps_triangular_input(orc, k):
    """Above k = 63 a column with nothing below its diagonal is left alone,
    so an upper-triangular A comes back as Q = I, R = A, bit for bit."""
    A = np.triu(general_batch(3, k, seed=k))
    Q, R = la.qr(_gpu(A))
    assert np.array_equal(_np(R), A) and np.array_equal(_np(Q), np.broadcast_to(np.eye(k, dtype=np.float32), A.shape))
    Q_ref, R_ref = orc.qr(A)
    assert np.array_equal(_np(R), R_ref) and np.array_equal(_np(Q), Q_ref)


@pytest.mark.parametrize("k", [6, 40])
def test_qr_zero_column(orc, k):
    """A zero column takes the reference's 1e-30 clamp: r_jj = -1e-15 and no
    reflection (tau = 0)."""
    A = general_batch(2, k, seed=k)
    A[:, :, 0] = 0.0
    Q, R = la.qr(_gpu(A))
    Q_ref, R_ref = orc.qr(A)
    assert np.all(_np(R)[:, 0, 0] == R_ref[:, 0, 0])
    assert np.allclose(_np(Q) @ _np(R), A, atol=1e-4)


@pytest.mark.parametrize("k", [40, 56, 64])
def test_qr_warp_kernel_walks_several_matrices(orc, k):
    """More matrices than resident warps (12 or 8 per SM x 148 SMs): every
    warp factors several matrices, its reflector buffer reused; a sample is
    checked against the oracle."""
    B = 148 * 12 * 2 + 7
    A = general_batch(B, k, seed=7700 + k)
    Q, R = la.qr(_gpu(A))
    idx = np.random.default_rng(k).choice(B, 24, replace=False)
    idx[-1] = B - 1
    Q_ref, R_ref = orc.qr(A[idx])
    _qr_checks(A[idx], _np(Q)[idx], _np(R)[idx], Q_ref, R_ref)


def test_qr_many_matrices_and_host_inputs(orc):
    A = general_batch(5_003, 9, seed=3)
    Q, R = la.qr(A)
    assert isinstance(Q, np.ndarray)
    Q_ref, R_ref = orc.qr(A)
    _qr_checks(A, Q, R, Q_ref, R_ref)
    Qd, Rd = la.qr(_gpu(A))
    assert np.array_equal(_np(Qd), Q) and np.array_equal(_np(Rd), R)
