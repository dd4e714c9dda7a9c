"""GPU randomized SVD (mlx_addons_b200.linalg.randomized_svd / TruncatedSVD)
against the golden fixtures from the reference run, the oracle, and the
reference's own test suite (tests/test_svd.py), plus the shifted Cholesky-QR
thin QR on full-rank, ill-conditioned and rank-deficient inputs."""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

la = pytest.importorskip("mlx_addons_b200.linalg")
from mlx_addons_b200.linalg import _svd  # noqa: E402

DEV = "cuda:0"


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _low_rank(rng, n, m, r, decay):
    U_, _ = np.linalg.qr(rng.standard_normal((n, r)).astype(np.float32))
    V_, _ = np.linalg.qr(rng.standard_normal((m, r)).astype(np.float32))
    return ((U_ * (10.0 * np.exp(-decay * np.arange(r))).astype(np.float32)) @ V_.T).astype(np.float32)


def _relerr(X, U, S, Vt):
    return np.linalg.norm(X - (U * S[..., None, :]) @ Vt) / np.linalg.norm(X)


# --------------------------------------------------------------------------
# thin QR
# --------------------------------------------------------------------------

@pytest.mark.parametrize("n,kp,rank,cond", [(100, 16, 16, 1), (500, 26, 26, 1), (10_000, 42, 42, 1), (100, 16, 10, 1),
                                            (300, 22, 20, 1), (64, 64, 64, 1), (500, 26, 26, 1e4),
                                            (500, 26, 26, 1e6), (2000, 42, 30, 1e3)])
def test_thin_qr_orthonormal_basis_of_the_range(n, kp, rank, cond):
    rng = np.random.default_rng(n + kp)
    U, _ = np.linalg.qr(rng.standard_normal((3, n, rank)))
    V, _ = np.linalg.qr(rng.standard_normal((3, kp, rank)))
    Y = ((U * np.logspace(0, -np.log10(cond), rank)) @ np.swapaxes(V, 1, 2)).astype(np.float32)
    Yd = torch.from_numpy(Y).to(DEV)
    Q = _svd.thin_qr(Yd).double()
    eye = torch.eye(kp, dtype=torch.float64, device=DEV)
    assert float((Q.transpose(1, 2) @ Q - eye).abs().max()) < 1e-4
    Y64 = Yd.double()
    resid = torch.linalg.norm(Y64 - Q @ (Q.transpose(1, 2) @ Y64)) / torch.linalg.norm(Y64)
    assert float(resid) < 1e-5


# --------------------------------------------------------------------------
# randomized_svd
# --------------------------------------------------------------------------

def test_randomized_svd_golden(golden, orc):
    n = 0
    for case, g in sorted(golden.items()):
        if not case.startswith("rsvd_"):
            continue
        k, it = int(g["k"]), int(g["n_iter"])
        U, S, Vt = la.randomized_svd(g["X"], n_components=k, n_iter=it, random_state=0)
        assert isinstance(U, np.ndarray) and U.shape == g["U"].shape and Vt.shape == g["Vt"].shape
        np.testing.assert_allclose(S, g["S"], rtol=2e-4, err_msg=case)
        if "lowrank" in case or "batched" in case:  # separated spectrum: vectors are well defined
            np.testing.assert_allclose(U, g["U"], atol=2e-3, err_msg=case)
            np.testing.assert_allclose(Vt, g["Vt"], atol=2e-3, err_msg=case)
        assert abs(_relerr(g["X"], U, S, Vt) - _relerr(g["X"], g["U"], g["S"], g["Vt"])) < 1e-4
        n += 1
    assert n >= 4


@pytest.mark.parametrize("shape,k,true_rank", [((100, 30), 6, 10), ((500, 128), 16, 32), ((1000, 64), 8, 16),
                                               ((2000, 256), 24, 48)])
def test_ref_suite_low_rank_recovery(shape, k, true_rank):  # test_svd.py:15-50
    n, m = shape
    rng = np.random.default_rng(0)
    U_t, _ = np.linalg.qr(rng.standard_normal((n, true_rank)).astype(np.float32))
    V_t, _ = np.linalg.qr(rng.standard_normal((m, true_rank)).astype(np.float32))
    X = (U_t * (10.0 * np.exp(-0.3 * np.arange(true_rank))).astype(np.float32)) @ V_t.T
    Ue, Se, Vte = np.linalg.svd(X, full_matrices=False)
    tail = np.linalg.norm(X - (Ue[:, :k] * Se[:k]) @ Vte[:k], "fro") / np.linalg.norm(X, "fro")
    U, S, Vt = la.randomized_svd(X, n_components=k, n_iter=6, random_state=0)
    assert _relerr(X, U, S, Vt) < max(tail * 1.5, 1e-3)


@pytest.mark.parametrize("shape,k", [((500, 64), 8), ((1000, 128), 24)])
def test_ref_suite_matches_full_svd(shape, k):  # :52-63
    X = np.random.default_rng(1).standard_normal(shape).astype(np.float32)
    S_true = np.linalg.svd(X, compute_uv=False)[:k]
    _, S, _ = la.randomized_svd(X, n_components=k, n_iter=6, random_state=0)
    assert (np.abs(S - S_true) / S_true).max() < 5e-2


def test_ref_suite_sign_canonicalization_and_orthonormal_U():  # :65-79
    rng = np.random.default_rng(2)
    X = rng.standard_normal((200, 50)).astype(np.float32)
    _, _, Va = la.randomized_svd(X, n_components=12, random_state=42)
    _, _, Vb = la.randomized_svd(X, n_components=12, random_state=42)
    np.testing.assert_allclose(Va, Vb, atol=1e-6)
    X = np.random.default_rng(3).standard_normal((300, 80)).astype(np.float32)
    U, _, _ = la.randomized_svd(X, n_components=20, random_state=0)
    assert np.abs(U.T @ U - np.eye(20)).max() < 1e-3


def test_ref_suite_batched():  # :81-120
    rng = np.random.default_rng(31)
    U, S, Vt = la.randomized_svd(rng.standard_normal((5, 300, 60)).astype(np.float32), n_components=8,
                                 random_state=0)
    assert U.shape == (5, 300, 8) and S.shape == (5, 8) and Vt.shape == (5, 8, 60)
    rng = np.random.default_rng(33)
    X = np.stack([_low_rank(rng, 400, 80, 24, 0.3) for _ in range(6)])
    U, S, Vt = la.randomized_svd(X, n_components=10, n_iter=6, random_state=0)
    for i in range(6):
        assert np.linalg.norm(X[i] - (U[i] * S[i]) @ Vt[i]) / np.linalg.norm(X[i]) < 0.1


def test_truncated_svd_class():  # :123-160
    rng = np.random.default_rng(7)
    X = rng.standard_normal((400, 100)).astype(np.float32)
    svd = la.TruncatedSVD(n_components=16, random_state=0)
    Z = svd.fit_transform(X)
    assert Z.shape == (400, 16) and svd.components_.shape == (16, 100) and svd.singular_values_.shape == (16,)
    Xn = rng.standard_normal((50, 100)).astype(np.float32)
    np.testing.assert_allclose(svd.transform(Xn), Xn @ svd.components_.T, atol=1e-5)


def test_device_inputs_stay_on_device(orc):
    rng = np.random.default_rng(9)
    X = _low_rank(rng, 300, 70, 20, 0.3)
    U, S, Vt = la.randomized_svd(torch.from_numpy(X).to(DEV), n_components=8, random_state=5)
    assert U.is_cuda and S.is_cuda and Vt.is_cuda
    Uo, So, Vto = orc.randomized_svd(X, 8, random_state=5)
    np.testing.assert_allclose(S.cpu().numpy(), So, rtol=2e-4)
    np.testing.assert_allclose(Vt.cpu().numpy(), Vto, atol=2e-3)
