"""GPU parity of the 2-D tile tier (one matrix per warp on a 2-D cyclic
register layout; 33 <= k <= 64, at most one right-hand side, no L output)
through libb2c's C ABI: against the oracle, the golden fixtures and the
two-rows-per-lane kernel that keeps m >= 2 and L outputs (B2C_TILE_TIER=0
routes a call to it). Tolerances: tests/_tol.py."""

import numpy as np
import pytest
import torch

from tests._data import spd_batch, with_upper_garbage
from tests._tol import backward_error, backward_tol, factor_tol, rel_fro_per_matrix

pytestmark = pytest.mark.gpu

la = pytest.importorskip("mlx_addons_b200.linalg")

DEV = "cuda:0"
TILE_KS = [33, 34, 37, 39, 40, 41, 45, 47, 48, 49, 53, 55, 56, 57, 60, 63, 64]


def _gpu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("k", TILE_KS)
@pytest.mark.parametrize("B", [1, 2, 37])
def test_tile_solve_logdet_vs_oracle(orc, k, B):
    """x and logdet of one fused call; B = 1, 2 and 37 leave most warps of the
    grid without a matrix."""
    A, b = spd_batch(B, k, m=1, eps=1.0, seed=9000 + 3 * k + B)
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    x = _np(x)
    assert np.max(rel_fro_per_matrix(x, x_ref)) < factor_tol(k)
    assert np.max(backward_error(A, x, b)) < backward_tol(k)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))
    # logdet alone (no right-hand side) runs the same tier without the solve
    np.testing.assert_allclose(_np(la.logdet_spd(_gpu(A))), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("k", [33, 40, 47, 56, 64])
def test_tile_many_rounds(orc, k):
    """A batch large enough that every warp walks several matrices (the
    staging of the next matrix overlaps the current one), odd so the last
    round is partial; sampled matrices against the oracle."""
    B = 20_001
    A, b = spd_batch(B, k, m=1, eps=0.5, seed=9500 + k)
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    x, ld = _np(x), _np(ld)
    idx = np.r_[0:40, B // 2 - 20:B // 2 + 20, B - 41:B]
    x_ref, ld_ref = orc.solve(A[idx], b[idx], return_logdet=True)
    assert np.max(rel_fro_per_matrix(x[idx], x_ref)) < factor_tol(k)
    np.testing.assert_allclose(ld[idx], ld_ref, rtol=factor_tol(k), atol=factor_tol(k))
    assert np.max(backward_error(A[:2000], x[:2000], b[:2000])) < backward_tol(k)


@pytest.mark.parametrize("k", [33, 48, 64])
def test_tile_matches_two_rows_per_lane_kernel(k, monkeypatch):
    """Same inputs through both k <= 64 kernels: equal within the factor
    tolerance (their FMA orders differ)."""
    A, b = spd_batch(501, k, m=1, seed=9700 + k)
    x1, ld1 = la.cho_solve_logdet(_gpu(A), _gpu(b))
    monkeypatch.setenv("B2C_TILE_TIER", "0")
    x0, ld0 = la.cho_solve_logdet(_gpu(A), _gpu(b))
    monkeypatch.delenv("B2C_TILE_TIER")
    assert np.max(rel_fro_per_matrix(_np(x1), _np(x0))) < factor_tol(k)
    np.testing.assert_allclose(_np(ld1), _np(ld0), rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("k", [33, 40, 52, 64])
def test_tile_upper_triangle_ignored_and_vector_b(k):
    A, b = spd_batch(9, k, m=1, seed=9800 + k)
    Ag = with_upper_garbage(A, seed=k)
    x = la.solve(_gpu(A), _gpu(b))
    assert torch.equal(la.solve(_gpu(Ag), _gpu(b)), x)
    assert torch.equal(la.logdet_spd(_gpu(Ag)), la.logdet_spd(_gpu(A)))
    # a (B, k) right-hand side gives a (B, k) solution, the same numbers
    x2 = la.solve(_gpu(A), _gpu(b[..., 0]))
    assert tuple(x2.shape) == (9, k) and torch.equal(x2, x[..., 0])


@pytest.mark.parametrize("k", [36, 64])
def test_tile_misaligned_inputs(orc, k):
    """A and b 4-byte aligned only: the element-wise staging path."""
    A, b = spd_batch(7, k, m=1, seed=9900 + k)
    bigA = torch.zeros(7 * k * k + 1, device=DEV)
    bigA[1:] = _gpu(A).reshape(-1)
    bigb = torch.zeros(7 * k + 1, device=DEV)
    bigb[1:] = _gpu(b).reshape(-1)
    Am, bm = bigA[1:].view(7, k, k), bigb[1:].view(7, k, 1)
    assert Am.data_ptr() % 16 != 0 and bm.data_ptr() % 16 != 0
    x = _np(la.solve(Am, bm))
    assert np.max(rel_fro_per_matrix(x, orc.solve(A, b))) < factor_tol(k)
    assert torch.allclose(la.solve(Am, bm), la.solve(_gpu(A), _gpu(b)), rtol=1e-6, atol=1e-6)


def test_tile_x_aliases_b():
    from mlx_addons_b200 import _lib
    lib = _lib.load()
    for k in (40, 64):
        A, b = spd_batch(5, k, m=1, seed=9950 + k)
        Ag, bg = _gpu(A), _gpu(b)
        ref = la.solve(Ag, bg)
        rc = lib.b2c_posv(Ag.data_ptr(), bg.data_ptr(), bg.data_ptr(), None, None, 5, k, 1, None, 0,
                          torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "posv")
        assert torch.equal(bg, ref)


def test_tile_clamp_non_spd():
    """Non-positive pivots are clamped, L_jj = sqrt(1e-12), as in the reference."""
    for k in (40, 64):
        A = -np.eye(k, dtype=np.float32)[None].repeat(3, 0)
        b = np.ones((3, k, 1), np.float32)
        x = _np(la.solve(_gpu(A), _gpu(b)))
        np.testing.assert_allclose(x, 1e12, rtol=1e-4)
        np.testing.assert_allclose(_np(la.logdet_spd(_gpu(A))), k * np.log(1e-12), rtol=1e-5)


def test_tile_golden(golden):
    n = 0
    for case, g in sorted(golden.items()):
        if not case.startswith(("solve_k", "config_", "upper_garbage")):
            continue
        k = g["A"].shape[-1]
        if not 33 <= k <= 64 or g["b"].ndim == 3 and g["b"].shape[-1] != 1:
            continue
        x = _np(la.solve(_gpu(g["A"]), _gpu(g["b"])))
        assert np.max(rel_fro_per_matrix(x.reshape(x.shape[0], -1), g["x"].reshape(x.shape[0], -1))) < factor_tol(k)
        if "logdet" in g:
            np.testing.assert_allclose(_np(la.logdet_spd(_gpu(g["A"]))), g["logdet"], rtol=5e-5, atol=5e-5)
        n += 1
    assert n >= 1
