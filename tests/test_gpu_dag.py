"""GPU parity of the task-graph form of the shared-memory tier (k % 4 == 0,
m <= 8, A in device memory; blocks loaded by TMA tiles, warps scheduled over
a dependency graph, trailing updates as 3xTF32 tensor-core products) against
the oracle and against the barrier-phased kernel of the same tier. By default
the library routes 193 <= k <= 256 (m <= 8) and 65 <= k <= 160 with
2 <= m <= 8 to it; every test here sets
B2C_SMEM_DAG=all so that it takes every k >= 65 (=0 routes a call to the
barrier-phased kernel). Tolerances: tests/_tol.py."""

import ctypes

import numpy as np
import pytest
import torch

from tests._data import spd_batch, with_upper_garbage
from tests._tol import backward_error, backward_tol, factor_tol, rel_fro_per_matrix

pytestmark = pytest.mark.gpu

la = pytest.importorskip("mlx_addons_b200.linalg")

DEV = "cuda:0"
# every block count 3..8, full and ragged last blocks (k % 32 = 4 .. 28)
DAG_KS = [68, 72, 80, 96, 100, 116, 124, 128, 132, 160, 164, 192, 200, 220, 228, 252, 256]


def _gpu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(autouse=True)
def _need_cuda(monkeypatch):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    monkeypatch.setenv("B2C_SMEM_DAG", "all")


def _fault():
    from mlx_addons_b200 import _lib
    f = ctypes.c_uint(7)
    assert _lib.load().b2c_take_device_fault(ctypes.byref(f)) == 0
    return f.value


@pytest.mark.parametrize("k", DAG_KS)
@pytest.mark.parametrize("m", [1, 2, 5, 8])
def test_dag_solve_logdet_vs_oracle(orc, k, m):
    B = 13
    A, b = spd_batch(B, k, m=m, eps=1.0, seed=12000 + 5 * k + m)
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    x = _np(x)
    assert np.all(np.isfinite(x))
    assert np.max(rel_fro_per_matrix(x, x_ref)) < factor_tol(k)
    assert np.max(backward_error(A, x, b)) < backward_tol(k)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("k", DAG_KS)
def test_dag_cholesky_and_logdet_vs_oracle(orc, k):
    """m = 0: the factor (upper triangle zeroed) and logdet, no substitution tasks."""
    B = 11
    A, _ = spd_batch(B, k, m=1, eps=1.0, seed=12500 + k)
    L = _np(la.cholesky(_gpu(A)))
    L_ref, ld_ref = orc.cholesky(A, return_logdet=True)
    assert np.all(np.triu(L, 1) == 0)
    assert np.max(rel_fro_per_matrix(L, L_ref)) < factor_tol(k)
    np.testing.assert_allclose(_np(la.logdet_spd(_gpu(A))), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("k,m", [(100, 1), (128, 8), (200, 3), (256, 8)])
def test_dag_many_matrices_per_cta(orc, k, m):
    """Several matrices per CTA (each reuses every mbarrier with the next
    phase and resets the task counter), last round partial; sampled
    matrices against the oracle, all finite, fault flag clear."""
    B = 3 * 148 * (4 if k <= 128 else 1) + 29
    A, b = spd_batch(B, k, m=m, eps=0.5, seed=13000 + k)
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    torch.cuda.synchronize()
    x, ld = _np(x), _np(ld)
    assert np.all(np.isfinite(x)) and np.all(np.isfinite(ld))
    idx = np.r_[0:8, B // 2 - 4:B // 2 + 4, B - 9:B]
    x_ref, ld_ref = orc.solve(A[idx], b[idx], return_logdet=True)
    assert np.max(rel_fro_per_matrix(x[idx], x_ref)) < factor_tol(k)
    np.testing.assert_allclose(ld[idx], ld_ref, rtol=factor_tol(k), atol=factor_tol(k))
    assert np.max(backward_error(A[:64], x[:64], b[:64])) < backward_tol(k)
    assert _fault() == 0


@pytest.mark.parametrize("k", [96, 164, 256])
def test_dag_matches_barrier_phased_kernel(k, monkeypatch):
    """Same inputs through both forms of the tier: equal within the factor
    tolerance (their summation orders differ)."""
    A, b = spd_batch(77, k, m=4, seed=13500 + k)
    x1, ld1 = la.cho_solve_logdet(_gpu(A), _gpu(b))
    monkeypatch.setenv("B2C_SMEM_DAG", "0")
    x0, ld0 = la.cho_solve_logdet(_gpu(A), _gpu(b))
    monkeypatch.setenv("B2C_SMEM_DAG", "all")
    assert np.max(rel_fro_per_matrix(_np(x1), _np(x0))) < factor_tol(k)
    np.testing.assert_allclose(_np(ld1), _np(ld0), rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("warps", ["4", "8", "12", "16"])
def test_dag_every_warp_count(orc, warps, monkeypatch):
    """The schedule does not depend on the number of warps taking tasks."""
    monkeypatch.setenv("B2C_DAG_WARPS", warps)
    for k in (72, 160, 256):
        A, b = spd_batch(9, k, m=8, seed=14000 + k)
        x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
        x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
        assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
        np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


def test_dag_ignores_the_upper_triangle(orc):
    """The tile loads bring whole 32 x 32 blocks, upper halves of the
    diagonal blocks included: NaN and huge values there change nothing."""
    for k in (100, 256):
        A, b = spd_batch(7, k, m=2, seed=14500 + k)
        x_clean = _np(la.solve(_gpu(A), _gpu(b)))
        Ag = with_upper_garbage(A)
        iu = np.triu_indices(k, 1)
        Ag[:, iu[0][::3], iu[1][::3]] = np.nan
        x = _np(la.solve(_gpu(Ag), _gpu(b)))
        np.testing.assert_array_equal(x, x_clean)


def test_dag_in_a_cuda_graph(orc):
    """The tensor map is a kernel parameter, so a captured launch replays on
    the captured buffers."""
    k, B = 256, 40
    A, b = spd_batch(B, k, m=8, seed=15000)
    Ag, bg = _gpu(A), _gpu(b)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        la.cho_solve_logdet(Ag, bg)  # warm-up outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        x, ld = la.cho_solve_logdet(Ag, bg)
    x.fill_(float("nan"))
    ld.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    del g
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("k", [100, 200, 256])
def test_dag_outputs_agree_across_calls(k):
    """The same factorisation whatever else is asked: logdet with right-hand
    sides equals logdet alone, x with L written equals x without it, bit for
    bit."""
    A, b = spd_batch(21, k, m=5, seed=15500 + k)
    x, ld, L = la.cho_solve_logdet(_gpu(A), _gpu(b), return_L=True)
    x2, ld2 = la.cho_solve_logdet(_gpu(A), _gpu(b))
    ld3 = la.logdet_spd(_gpu(A))
    assert torch.equal(x, x2)
    assert torch.equal(ld, ld2) and torch.equal(ld, ld3)
    assert torch.equal(L, la.cholesky(_gpu(A)))


def test_dag_wait_timeout_is_reported_and_contained(orc, monkeypatch):
    """With the test-only switch B2C_DAG_INJECT_TIMEOUT=1 (read per call),
    CTA 0 waits for an mbarrier phase that nothing completes, every wait
    limited to 1 ms: the CTA gives up, lets its tile loads land, writes NaN
    to x and logdet of each matrix it owned and sets the device flag; the
    other CTAs' matrices are right, and the next call runs normally. No
    fault and no hang are involved."""
    k, B = 256, 300
    A, b = spd_batch(B, k, m=8, seed=16000)
    _fault()
    monkeypatch.setenv("B2C_DAG_INJECT_TIMEOUT", "1")
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    torch.cuda.synchronize()
    monkeypatch.delenv("B2C_DAG_INJECT_TIMEOUT")
    assert _fault() != 0
    x, ld = _np(x), _np(ld)
    bad = np.flatnonzero(~np.isfinite(ld))
    assert bad.size >= 1 and bad[0] == 0
    if bad.size > 1:  # CTA 0's matrices: 0, grid, 2 grid, ...
        np.testing.assert_array_equal(bad, np.arange(0, B, bad[1]))
    assert np.all(np.isnan(x[bad]))
    good = np.setdiff1d(np.arange(B), bad)[:24]
    x_ref, ld_ref = orc.solve(A[good], b[good], return_logdet=True)
    assert np.max(rel_fro_per_matrix(x[good], x_ref)) < factor_tol(k)
    x2, ld2 = la.cho_solve_logdet(_gpu(A[:40]), _gpu(b[:40]))
    torch.cuda.synchronize()
    assert _fault() == 0
    assert np.all(np.isfinite(_np(x2))) and np.all(np.isfinite(_np(ld2)))
