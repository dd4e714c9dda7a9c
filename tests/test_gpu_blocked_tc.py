"""The tiers above k = 64: the shared-memory tier (the default to k = 256),
the blocked tier with its panel products on FP32 FFMA
(B2C_SMEM_TIER=0, and the default above) and on the tensor cores (3xTF32
tcgen05, B2C_BLOCKED_GEMM=tc). All are checked against the oracle at the same
tolerances, across ragged k (k % 4 != 0 takes the scalar-load path, k % 32 !=
0 a ragged last panel), fused and unfused forward substitutions (m <= 8 and
m > 8) and the factor-only call; the library's device fault flag must stay
clear."""

# "smem": the barrier-phased shared-memory kernel (the task-graph form of the
# tier, which takes m <= 8 only, has its own file: tests/test_gpu_dag.py)
# "legacy": the earlier blocked kernel (posv_blocked.cu), which serves k > 9,216
# only by default, forced here at every k
FORM_ENV = {"smem": {"B2C_SMEM_DAG": "0"}, "ffma": {"B2C_SMEM_TIER": "0"}, "tc": {"B2C_BLOCKED_GEMM": "tc"},
            "legacy": {"B2C_SMEM_TIER": "0", "B2C_BLOCKED_LEGACY": "1"}}

import ctypes

import numpy as np
import pytest
import torch

from tests._data import spd_batch
from tests._tol import backward_error, backward_tol, factor_tol, rel_fro_per_matrix

pytestmark = pytest.mark.gpu

la = pytest.importorskip("mlx_addons_b200.linalg")
from mlx_addons_b200 import _lib  # noqa: E402

DEV = "cuda:0"
KS = [65, 80, 96, 100, 127, 128, 130, 160, 200, 256, 300, 384, 512, 600]


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _gpu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _np(t):
    return t.detach().cpu().numpy()


def _fault():
    f = ctypes.c_uint(7)
    assert _lib.load().b2c_take_device_fault(ctypes.byref(f)) == 0
    return f.value


@pytest.mark.parametrize("form", ["smem", "ffma", "tc", "legacy"])
@pytest.mark.parametrize("k", KS)
@pytest.mark.parametrize("m", [1, 3, 8, 9, 20])
def test_blocked_forms_vs_oracle(orc, k, m, form, monkeypatch):
    for name, value in FORM_ENV[form].items():
        monkeypatch.setenv(name, value)
    B = 7 if k <= 256 else 3
    A, b = spd_batch(B, k, m=m, eps=1.0, seed=9100 + 13 * k + m)
    x, ld, L = la.cho_solve_logdet(_gpu(A), _gpu(b), return_L=True)
    x2 = la.solve(_gpu(A), _gpu(b))  # the slot in scratch instead of L
    ld2 = la.logdet_spd(_gpu(A))     # factor only
    torch.cuda.synchronize()
    assert _fault() == 0
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    L_ref = orc.cholesky(A)
    L = _np(L)
    assert np.all(np.triu(L, 1) == 0)
    assert np.max(rel_fro_per_matrix(L, L_ref)) < factor_tol(k)
    assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
    assert np.max(backward_error(A, _np(x), b)) < backward_tol(k)
    assert torch.equal(x, x2)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))
    assert torch.equal(ld, ld2)


@pytest.mark.parametrize("form", ["smem", "tc", "legacy"])
@pytest.mark.parametrize("k", [1, 5, 16, 33, 64])
def test_forms_small_k(orc, k, form, monkeypatch):
    """Forced above the register tiers, a single ragged panel (bw < 32 for k < 32)."""
    monkeypatch.setenv("B2C_TIER", "blocked")
    for name, value in FORM_ENV[form].items():
        monkeypatch.setenv(name, value)
    A, b = spd_batch(9, k, m=2, seed=9300 + k)
    x, ld, L = la.cho_solve_logdet(_gpu(A), _gpu(b), return_L=True)
    torch.cuda.synchronize()
    assert _fault() == 0
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
    assert np.max(rel_fro_per_matrix(_np(L), orc.cholesky(A))) < factor_tol(k)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("form,k", [("tc", 96), ("smem", 96), ("smem", 256)])
def test_forms_many_matrices_per_cta(orc, form, k, monkeypatch):
    """More matrices than resident CTAs: each CTA walks several matrices (the
    tensor-core form carrying its tensor memory and mbarrier phases across
    them, the shared-memory tier reloading its blocks)."""
    for name, value in FORM_ENV[form].items():
        monkeypatch.setenv(name, value)
    B = 5000 if k <= 128 else 700
    A, b = spd_batch(B, k, m=1, eps=1.0, seed=9400)
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    torch.cuda.synchronize()
    assert _fault() == 0
    idx = np.random.default_rng(0).choice(B, 40, replace=False)
    x_ref, ld_ref = orc.solve(A[idx], b[idx], return_logdet=True)
    assert np.max(rel_fro_per_matrix(_np(x)[idx], x_ref)) < factor_tol(k)
    np.testing.assert_allclose(_np(ld)[idx], ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


def test_tc_wait_timeout_is_reported_and_contained(orc, monkeypatch):
    """A tensor-core completion wait that runs out (B2C_TC_INJECT_TIMEOUT=1:
    CTA 0 waits on an mbarrier phase nothing will complete, with no MMA in
    flight, every wait limited to 1 ms) is reported through the device fault
    flag, which reading clears; that CTA's matrices come back NaN, every other
    matrix is solved, and the next call runs normally. No fault, no hang."""
    monkeypatch.setenv("B2C_BLOCKED_GEMM", "tc")
    k, B = 300, 20  # one matrix per CTA: only matrix 0 belongs to CTA 0
    A, b = spd_batch(B, k, m=1, seed=11)
    _fault()
    monkeypatch.setenv("B2C_TC_INJECT_TIMEOUT", "1")
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    torch.cuda.synchronize()
    assert _fault() == 1
    assert _fault() == 0
    x, ld = _np(x), _np(ld)
    assert np.all(np.isnan(x[0])) and np.isnan(ld[0])
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert np.max(rel_fro_per_matrix(x[1:], x_ref[1:])) < factor_tol(k)
    np.testing.assert_allclose(ld[1:], ld_ref[1:], rtol=factor_tol(k), atol=factor_tol(k))
    monkeypatch.delenv("B2C_TC_INJECT_TIMEOUT")
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    assert _fault() == 0
    assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
