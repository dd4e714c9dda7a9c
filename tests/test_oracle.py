"""Pins the CPU oracle (oracle/chol_oracle.c) to the reference.

* against the golden fixtures written from the reference run (its own Python
  and kernel bodies, tests/golden/make_golden.py): bit-exact wherever the
  reference takes an unblocked kernel path, within float32 tolerance on the
  blocked path (whose trailing update is an MLX GEMM) and for slogdet (LAPACK);
* against the reference's kernels compiled for the host (oracle/_ref), live,
  when that library is present;
* through the reference's own test suite (tests/test_linalg.py), restated
  with the oracle in place of mlx_addons.linalg and the same tolerances;
* against LAPACK spotrf/spotrs.
"""

import os

import numpy as np
import pytest

from tests._data import general_batch, make_rhs_ref, make_spd_ref, spd_batch
from tests._tol import backward_error, factor_tol, rel_fro


def _cases(golden, prefix):
    return sorted(c for c in golden if c.startswith(prefix))


def _k_of(case):
    return int(case.split("_k")[1].split("_")[0])


# --------------------------------------------------------------------------
# golden fixtures
# --------------------------------------------------------------------------

def test_golden_solve_cholesky_logdet(golden, orc):
    checked = 0
    for case in _cases(golden, "solve_k"):
        g = golden[case]
        k = _k_of(case)
        x = orc.solve(g["A"], g["b"])
        L = orc.cholesky(g["A"])
        ld = orc.logdet_spd(g["A"])
        if k <= 80:  # the reference runs one fused kernel / one small kernel here
            assert np.array_equal(x, g["x"]), case
            assert np.array_equal(L, g["L"]), case
        else:
            assert rel_fro(x, g["x"]) < factor_tol(k), case
            assert rel_fro(L, g["L"]) < factor_tol(k), case
        np.testing.assert_allclose(ld, g["logdet"], rtol=2e-5, atol=2e-5, err_msg=case)
        checked += 1
    assert checked >= 20


def test_golden_solve_cholesky_small_kernel(golden, orc):
    for case in _cases(golden, "solve_cholesky_k"):
        g = golden[case]
        assert np.array_equal(orc.solve_small(g["A"], g["b"]), g["x"]), case


def test_golden_b2d(golden, orc):
    for case in _cases(golden, "solve_b2d"):
        g = golden[case]
        x = orc.solve(g["A"], g["b"])
        assert x.shape == g["b"].shape == g["x"].shape
        k = _k_of(case)
        if k <= 80:
            assert np.array_equal(x, g["x"])
        else:
            assert rel_fro(x, g["x"]) < factor_tol(k)


def test_golden_upper_garbage_and_clamp(golden, orc):
    for case in _cases(golden, "upper_garbage") + ["clamp_k4"]:
        g = golden[case]
        k = g["A"].shape[-1]
        x = orc.solve(g["A"], g["b"])
        L = orc.cholesky(g["A"])
        if k <= 80:
            assert np.array_equal(x, g["x"]), case
            assert np.array_equal(L, g["L"]), case
        else:
            assert rel_fro(x, g["x"]) < factor_tol(k), case
            assert rel_fro(L, g["L"]) < factor_tol(k), case
    g = golden["clamp_k4"]
    assert np.all(np.isfinite(g["x"])) and np.all(np.isfinite(g["L"]))
    assert g["L"][0, 1, 1] == np.float32(1e-6)  # sqrt(max(-1, 1e-12))


def test_golden_triangular(golden, orc):
    for case in _cases(golden, "tri_k"):
        g = golden[case]
        assert np.array_equal(orc.tril_solve(g["L"], g["b"]), g["x_lower"]), case
        assert np.array_equal(orc.triu_solve(g["L"], g["b"]), g["x_upper"]), case


def test_golden_slogdet(golden, orc):
    for case in _cases(golden, "slogdet"):
        g = golden[case]
        s, l = orc.slogdet(g["A"])
        assert s.shape == g["sign"].shape
        assert np.array_equal(s, g["sign"]), case
        finite = np.isfinite(g["logabsdet"])
        assert np.array_equal(np.isfinite(l), finite), case
        np.testing.assert_allclose(l[finite], g["logabsdet"][finite], rtol=1e-4, atol=1e-4, err_msg=case)
    g = golden["slogdet_lead_dims_n6"]
    np.testing.assert_allclose(orc.det(g["A"]), g["det"], rtol=1e-4, atol=1e-6)
    g = golden["slogdet_special_n4"]
    assert g["sign"][0] == 0 and np.isneginf(g["logabsdet"][0])
    assert g["sign"][1] == 1 and g["logabsdet"][1] == 0


def test_golden_configs(golden, orc):
    for case in _cases(golden, "config_"):
        g = golden[case]
        k = g["A"].shape[-1]
        x = orc.solve(g["A"], g["b"])
        if k <= 80:
            assert np.array_equal(x, g["x"]), case
        else:
            assert rel_fro(x, g["x"]) < factor_tol(k), case
        if "L" in g:
            L = orc.cholesky(g["A"])
            assert rel_fro(L, g["L"]) < factor_tol(k), case
        np.testing.assert_allclose(orc.logdet_spd(g["A"]), g["logdet"], rtol=5e-5, atol=5e-5)


def _same_nonfinite(a, b):
    return np.array_equal(np.isnan(a), np.isnan(b)) and np.array_equal(np.isposinf(a), np.isposinf(b)) and \
        np.array_equal(np.isneginf(a), np.isneginf(b))


def test_golden_solve_lu(golden, orc):
    cases = _cases(golden, "solve_lu")
    assert len(cases) >= 10
    for case in cases:
        g = golden[case]
        x = orc.lu_solve(g["A"], g["b"])
        assert x.shape == g["x"].shape, case
        assert _same_nonfinite(x, g["x"]), case
        assert np.array_equal(np.nan_to_num(x), np.nan_to_num(g["x"])), case  # bit-exact restatement
    g = golden["solve_lu_special_k4"]
    assert np.array_equal(g["x"][0], np.linalg.solve(g["A"][0], g["b"][0]))  # permutation: exact
    assert not np.all(np.isfinite(g["x"][1]))                                  # singular: inf / NaN
    assert np.isposinf(g["x"][1]).any() or np.isneginf(g["x"][1]).any() or np.isnan(g["x"][1]).any()


def test_golden_qr(golden, orc):
    cases = _cases(golden, "qr_k")
    assert len(cases) >= 12
    for case in cases:
        g = golden[case]
        Q, R = orc.qr(g["A"])
        k = g["A"].shape[-1]
        if k <= orc.QR_SHARED_K_MAX:  # the reference's GPU kernels: bit-exact restatement
            assert np.array_equal(Q, g["Q"]) and np.array_equal(R, g["R"]), case
        else:  # the reference's CPU LAPACK path: same Householder convention, to rounding
            assert rel_fro(Q, g["Q"]) < 1e-4 and rel_fro(R, g["R"]) < 1e-4, case
    g = golden["qr_2d_k10"]
    Q, R = orc.qr(g["A"][None])
    assert np.array_equal(Q[0], g["Q"]) and np.array_equal(R[0], g["R"])


# --------------------------------------------------------------------------
# live comparison with the reference's kernels compiled for the host
# --------------------------------------------------------------------------

_REF_BUILT = os.path.exists(os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref", "libmlxref.so"))


@pytest.mark.skipif(not _REF_BUILT, reason="oracle/_ref not built here")
@pytest.mark.parametrize("k", [1, 2, 5, 12, 31, 32, 33, 64, 100, 128])
def test_lu_solve_bit_exact_vs_reference_kernels(orc, k):
    A = general_batch(11, k, seed=40 + k)
    b = np.random.default_rng(k).standard_normal((11, k, 3), dtype=np.float32)
    A[0, :, 0] = 0.0  # a zero column: no pivot, no scaling, inf / NaN in x
    assert np.array_equal(np.nan_to_num(orc.lu_solve(A, b)), np.nan_to_num(orc.ref_lu_solve(A, b)))


@pytest.mark.skipif(not _REF_BUILT, reason="oracle/_ref not built here")
@pytest.mark.parametrize("k", [1, 2, 3, 8, 11, 12, 13, 32, 40, 63])
def test_qr_bit_exact_vs_reference_kernels(orc, k):
    A = general_batch(9, k, seed=70 + k)
    A[0, :, -1] = 0.0
    Q, R = orc.qr(A)
    Qr, Rr = orc.ref_qr(A)
    assert np.array_equal(Q, Qr) and np.array_equal(R, Rr)

@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref",
                                                    "libmlxref.so")), reason="oracle/_ref not built here")
@pytest.mark.parametrize("k", [1, 2, 7, 16, 32, 33, 57, 64, 80, 81, 100, 128])
def test_oracle_bit_exact_vs_reference_kernels(orc, k):
    A, b = spd_batch(9, k, m=2, eps=0.5, seed=k)
    x_ref, L_ref = orc.ref_solve_small(A, b, return_L=True)
    assert np.array_equal(orc.solve_small(A, b), x_ref)
    Lc = orc.ref_cholesky_small(A)
    assert np.array_equal(orc.cholesky_small(A), Lc)
    assert np.array_equal(orc.tril_solve(Lc, b), orc.ref_tri_solve(Lc, b, upper=False))
    assert np.array_equal(orc.triu_solve(Lc, b), orc.ref_tri_solve(Lc, b, upper=True))


# --------------------------------------------------------------------------
# the reference's test suite (tests/test_linalg.py), oracle in place of MLX
# --------------------------------------------------------------------------

@pytest.mark.parametrize("k", [3, 5, 8, 10, 15, 20, 30])
def test_ref_suite_solve_small_accuracy(orc, k):  # test_linalg.py:30-39
    A, b = make_spd_ref(100, k), make_rhs_ref(100, k)
    x = orc.solve(A.astype(np.float32), b.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(A @ x - b)) / np.max(np.abs(b)) < 1e-3


@pytest.mark.parametrize("k", [48, 64, 96, 128])
def test_ref_suite_solve_large_accuracy(orc, k):  # :41-50
    A, b = make_spd_ref(20, k), make_rhs_ref(20, k)
    x = orc.solve(A.astype(np.float32), b.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(A @ x - b)) / np.max(np.abs(b)) < 1e-2


def test_ref_suite_multi_rhs(orc):  # :52-60
    A, b = make_spd_ref(50, 8), make_rhs_ref(50, 8, m=4)
    x = orc.solve(A.astype(np.float32), b.astype(np.float32))
    assert x.shape == (50, 8, 4)
    assert np.max(np.abs(A @ x.astype(np.float64) - b)) / np.max(np.abs(b)) < 1e-3


@pytest.mark.parametrize("k,tol", [(3, 1e-4), (5, 1e-4), (10, 1e-4), (20, 1e-4), (30, 1e-4),
                                   (48, 1e-3), (64, 1e-3), (128, 1e-3)])
def test_ref_suite_cholesky_reconstruction(orc, k, tol):  # :69-87
    A = make_spd_ref(50 if k <= 30 else 10, k)
    L = orc.cholesky(A.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(A - L @ np.transpose(L, (0, 2, 1)))) / np.max(np.abs(A)) < tol


def test_ref_suite_lower_triangular(orc):  # :89-96
    L = orc.cholesky(make_spd_ref(10, 6).astype(np.float32))
    assert np.all(np.abs(L[:, np.triu_indices(6, 1)[0], np.triu_indices(6, 1)[1]]) < 1e-6)


@pytest.mark.parametrize("k", [6, 20, 48, 64, 80, 96])
def test_ref_suite_triangular(orc, k):  # :105-127
    A = make_spd_ref(30, k).astype(np.float32)
    L = orc.cholesky(A)
    b = make_rhs_ref(30, k).astype(np.float32)
    assert np.max(np.abs(L @ orc.tril_solve(L, b) - b)) < 5e-3
    assert np.max(np.abs(np.swapaxes(L, -1, -2) @ orc.triu_solve(L, b) - b)) < 5e-3


@pytest.mark.parametrize("n", [3, 5, 10, 20])
def test_ref_suite_det(orc, n):  # :136-145
    A = make_spd_ref(10, n)
    d = orc.det(A.astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(np.log(np.abs(d)) - np.log(np.abs(np.linalg.det(A))))) < 0.01


@pytest.mark.parametrize("n", [3, 5, 10, 20, 50])
def test_ref_suite_slogdet(orc, n):  # :147-157
    A = make_spd_ref(10, n)
    s_ref, l_ref = np.linalg.slogdet(A)
    s, l = orc.slogdet(A.astype(np.float32))
    assert np.all(s == s_ref)
    assert np.max(np.abs(l - l_ref)) < 0.1


@pytest.mark.parametrize("n", [3, 5, 10, 20, 64, 128])
def test_ref_suite_logdet_spd(orc, n):  # :159-167
    A = make_spd_ref(10, n)
    _, l_ref = np.linalg.slogdet(A)
    assert np.max(np.abs(orc.logdet_spd(A.astype(np.float32)) - l_ref)) < 0.1


@pytest.mark.parametrize("k", [3, 5, 8, 10, 16, 20, 32, 48, 63, 64, 96, 128])
def test_ref_suite_qr_accuracy(orc, k):  # :176-191
    A = np.random.default_rng(42).standard_normal((50 if k <= 64 else 10, k, k)).astype(np.float32)
    Q, R = orc.qr(A)
    assert np.max(np.abs(Q @ R - A)) < (1e-3 if k <= 63 else 5e-3)


@pytest.mark.parametrize("k", [3, 8, 16])
def test_ref_suite_qr_orthogonality_and_upper(orc, k):  # :193-217
    A = np.random.default_rng(123).standard_normal((100, k, k)).astype(np.float32)
    Q, R = orc.qr(A)
    assert np.max(np.abs(np.swapaxes(Q, -1, -2) @ Q - np.eye(k, dtype=np.float32))) < 1e-3
    assert np.all(np.abs(np.tril(R, -1)) < 1e-4)


@pytest.mark.parametrize("k", [2, 7, 32, 90])
def test_lu_solve_accuracy(orc, k):
    A = general_batch(20, k, seed=k) + np.float32(0.0)
    b = np.random.default_rng(k + 1).standard_normal((20, k, 2), dtype=np.float32)
    x = orc.lu_solve(A, b).astype(np.float64)
    r = np.abs(A.astype(np.float64) @ x - b)
    scale = np.abs(A.astype(np.float64)) @ np.abs(x) + np.abs(b)
    assert np.max(r / scale) < 1e-4


def test_golden_randomized_svd(golden, orc):
    cases = _cases(golden, "rsvd_")
    assert len(cases) >= 4
    for case in cases:
        g = golden[case]
        U, S, Vt = orc.randomized_svd(g["X"], int(g["k"]), n_iter=int(g["n_iter"]), random_state=0)
        np.testing.assert_allclose(S, g["S"], rtol=1e-5, err_msg=case)
        np.testing.assert_allclose(U, g["U"], atol=1e-4, err_msg=case)
        np.testing.assert_allclose(Vt, g["Vt"], atol=1e-4, err_msg=case)


def test_ref_suite_randomized_svd(orc):  # tests/test_svd.py:15-50, :66-85
    rng = np.random.default_rng(0)
    n, m, r, k = 500, 128, 32, 16
    U_, _ = np.linalg.qr(rng.standard_normal((n, r)).astype(np.float32))
    V_, _ = np.linalg.qr(rng.standard_normal((m, r)).astype(np.float32))
    X = (U_ * (10.0 * np.exp(-0.3 * np.arange(r))).astype(np.float32)) @ V_.T
    Ue, Se, Vte = np.linalg.svd(X, full_matrices=False)
    tail = np.linalg.norm(X - (Ue[:, :k] * Se[:k]) @ Vte[:k]) / np.linalg.norm(X)
    U, S, Vt = orc.randomized_svd(X, k, n_iter=6, random_state=0)
    assert np.linalg.norm(X - (U * S) @ Vt) / np.linalg.norm(X) < max(1.5 * tail, 1e-3)
    U, S, Vt = orc.randomized_svd(rng.standard_normal((5, 300, 60)).astype(np.float32), 8, random_state=0)
    assert U.shape == (5, 300, 8) and S.shape == (5, 8) and Vt.shape == (5, 8, 60)


# --------------------------------------------------------------------------
# LAPACK stand-in for MLX's CPU stream
# --------------------------------------------------------------------------

@pytest.mark.parametrize("k,m", [(5, 4), (16, 1), (64, 1), (130, 2)])
def test_oracle_vs_lapack(orc, k, m):
    A, b = spd_batch(16, k, m=m, seed=3)
    x_l, ld_l = orc.lapack_posv(A, b)
    x_o, ld_o = orc.solve(A, b, return_logdet=True)
    assert rel_fro(x_o, x_l) < factor_tol(k)
    np.testing.assert_allclose(ld_o, ld_l, rtol=1e-5, atol=1e-5)
    assert np.max(backward_error(A, x_o, b)) < 1e-6
