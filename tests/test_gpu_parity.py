"""GPU parity: the CUDA kernels (through libb2c's C ABI) against the oracle
and the golden fixtures from the reference run. Tolerances: tests/_tol.py."""

import ctypes
import os

import numpy as np
import pytest
import torch

from tests._data import CONFIGS, general_batch, spd_batch, with_upper_garbage
from tests._tol import backward_error, backward_tol, factor_tol, rel_fro, rel_fro_per_matrix

pytestmark = pytest.mark.gpu

la = pytest.importorskip("mlx_addons_b200.linalg")

DEV = "cuda:0"

SOLVE_KS = [1, 2, 3, 4, 5, 6, 7, 8, 9, 12, 15, 16, 17, 20, 24, 31, 32, 33, 37, 40, 47, 48, 55, 56, 63, 64, 65,
            80, 81, 96, 100, 128, 130, 160, 200, 256]


def _gpu(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


# --------------------------------------------------------------------------
# solve / cholesky / logdet against the oracle
# --------------------------------------------------------------------------

@pytest.mark.parametrize("k", SOLVE_KS)
@pytest.mark.parametrize("m", [1, 3, 8])
def test_solve_vs_oracle(orc, k, m):
    B = 37 if k <= 128 else 9
    A, b = spd_batch(B, k, m=m, eps=1.0, seed=1000 + 7 * k + m)
    x = _np(la.solve(_gpu(A), _gpu(b)))
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert x.shape == b.shape
    assert np.all(np.isfinite(x))
    assert np.max(rel_fro_per_matrix(x, x_ref)) < factor_tol(k)
    assert np.max(backward_error(A, x, b)) < backward_tol(k)


@pytest.mark.parametrize("k", [2, 5, 8, 9, 12, 16])
@pytest.mark.parametrize("m", [1, 2, 3, 4])
def test_thread_tier_many_tiles_per_block(orc, k, m):
    """k <= 16, m <= 4: a ragged batch large enough that every CTA walks
    several tiles, so the double-buffered staging is exercised past its first
    tile (both register layouts of the factor: square and packed)."""
    B = 150_001
    A, b = spd_batch(B, k, m=m, eps=0.5, seed=8000 + 10 * k + m)
    x, ld, L = la.cho_solve_logdet(_gpu(A), _gpu(b), return_L=True)
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    L_ref = orc.cholesky(A)
    assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
    assert np.max(rel_fro_per_matrix(_np(L), L_ref)) < factor_tol(k)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("k", [16, 17, 23, 24, 25, 30, 32])
@pytest.mark.parametrize("m", [1, 2, 4, 5])
def test_segment_tier_many_rounds(orc, k, m):
    """8 or 16 lanes per matrix (17 <= k <= 32, and k = 16 with m >= 4): a
    ragged batch large enough that every CTA walks several rounds of staged
    matrices, with the factor, solve and logdet outputs checked together
    (padded KP = 24 and 32, 4-, 8- and 16-byte staging paths)."""
    B = 20_011
    A, b = spd_batch(B, k, m=m, eps=0.5, seed=8500 + 10 * k + m)
    x, ld, L = la.cho_solve_logdet(_gpu(A), _gpu(b), return_L=True)
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    L_ref = orc.cholesky(A)
    assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
    assert np.max(rel_fro_per_matrix(_np(L), L_ref)) < factor_tol(k)
    assert np.all(np.triu(_np(L)[:64], 1) == 0)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))
    assert np.max(backward_error(A[:500], _np(x)[:500], b[:500])) < backward_tol(k)


@pytest.mark.parametrize("k", SOLVE_KS)
def test_cholesky_logdet_vs_oracle(orc, k):
    B = 37 if k <= 128 else 9
    A, _ = spd_batch(B, k, eps=1.0, seed=2000 + k)
    L = _np(la.cholesky(_gpu(A)))
    L_ref, ld_ref = orc.cholesky(A, return_logdet=True)
    assert np.all(np.triu(L, 1) == 0)
    assert np.max(rel_fro_per_matrix(L, L_ref)) < factor_tol(k)
    ld = _np(la.logdet_spd(_gpu(A)))
    np.testing.assert_allclose(ld, ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


@pytest.mark.parametrize("k", [5, 16, 64, 96, 256])
def test_fused_cho_solve_logdet(orc, k):
    A, b = spd_batch(11, k, m=2, seed=3000 + k)
    x, ld, L = la.cho_solve_logdet(_gpu(A), _gpu(b), return_L=True)
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert np.max(rel_fro_per_matrix(_np(x), x_ref)) < factor_tol(k)
    np.testing.assert_allclose(_np(ld), ld_ref, rtol=factor_tol(k), atol=factor_tol(k))
    assert np.max(rel_fro_per_matrix(_np(L), orc.cholesky(A))) < factor_tol(k)
    # same kernel with and without the optional outputs
    assert torch.equal(x, la.solve(_gpu(A), _gpu(b)))


@pytest.mark.parametrize("k", [1, 5, 8, 16, 33, 48, 64])
def test_blocked_tier_small_k(orc, k, monkeypatch):
    """The blocked tier handles every k (ragged single panel included)."""
    monkeypatch.setenv("B2C_TIER", "blocked")
    A, b = spd_batch(13, k, m=3, seed=4000 + k)
    x = _np(la.solve(_gpu(A), _gpu(b)))
    L = _np(la.cholesky(_gpu(A)))
    ld = _np(la.logdet_spd(_gpu(A)))
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert np.max(rel_fro_per_matrix(x, x_ref)) < factor_tol(k)
    assert np.max(rel_fro_per_matrix(L, orc.cholesky(A))) < factor_tol(k)
    np.testing.assert_allclose(ld, ld_ref, rtol=1e-5, atol=1e-5)


# --------------------------------------------------------------------------
# triangular solves and slogdet
# --------------------------------------------------------------------------

@pytest.mark.parametrize("k", [1, 2, 6, 16, 20, 31, 32, 33, 48, 64, 80, 96, 128, 150, 256])
@pytest.mark.parametrize("m", [1, 4, 9])
def test_triangular_vs_oracle(orc, k, m):
    A, b = spd_batch(21, k, m=m, seed=5000 + k + m)
    L = orc.cholesky(A)
    xl = _np(la.tril_solve(_gpu(L), _gpu(b)))
    xu = _np(la.triu_solve(_gpu(L), _gpu(b)))
    assert np.max(rel_fro_per_matrix(xl, orc.tril_solve(L, b))) < factor_tol(k)
    assert np.max(rel_fro_per_matrix(xu, orc.triu_solve(L, b))) < factor_tol(k)


@pytest.mark.parametrize("n", [1, 2, 3, 5, 8, 16, 31, 32, 33, 50, 64, 100, 128, 200, 224, 225, 256, 300, 500])
def test_slogdet_vs_oracle(orc, n):
    A = general_batch(17 if n <= 128 else 5, n, seed=6000 + n)
    s, l = la.slogdet(_gpu(A))
    s_ref, l_ref = orc.slogdet(A)
    assert np.array_equal(_np(s), s_ref)
    np.testing.assert_allclose(_np(l), l_ref, rtol=1e-4, atol=1e-4)
    d = _np(la.det(_gpu(A[:, :min(n, 8), :min(n, 8)].copy())))
    np.testing.assert_allclose(d, orc.det(A[:, :min(n, 8), :min(n, 8)].copy()), rtol=1e-3, atol=1e-6)


def test_slogdet_spd_and_lead_dims(orc):
    A, _ = spd_batch(4, 40, seed=7)
    s, l = la.slogdet(_gpu(A))
    assert torch.all(s == 1)
    np.testing.assert_allclose(_np(l), orc.logdet_spd(A), rtol=1e-4, atol=1e-4)
    G = general_batch(12, 6, seed=8).reshape(2, 3, 2, 6, 6)
    s, l = la.slogdet(_gpu(G))
    assert tuple(s.shape) == (2, 3, 2)
    s_ref, l_ref = orc.slogdet(G)
    assert np.array_equal(_np(s), s_ref)
    np.testing.assert_allclose(_np(l), l_ref, rtol=1e-4, atol=1e-4)


# --------------------------------------------------------------------------
# golden fixtures from the reference run
# --------------------------------------------------------------------------

def test_golden_fixtures(golden):
    n = 0
    for case, g in sorted(golden.items()):
        if case.startswith(("solve_k", "upper_garbage", "config_", "solve_b2d", "solve_cholesky")):
            k = g["A"].shape[-1]
            x = _np(la.solve(_gpu(g["A"]), _gpu(g["b"])))
            assert x.shape == g["x"].shape, case
            assert rel_fro(x, g["x"]) < factor_tol(k), case
            if "L" in g:
                assert rel_fro(_np(la.cholesky(_gpu(g["A"]))), g["L"]) < factor_tol(k), case
            if "logdet" in g:
                np.testing.assert_allclose(_np(la.logdet_spd(_gpu(g["A"]))), g["logdet"], rtol=5e-5, atol=5e-5,
                                           err_msg=case)
            n += 1
        elif case.startswith("tri_k"):
            k = g["L"].shape[-1]
            assert rel_fro(_np(la.tril_solve(_gpu(g["L"]), _gpu(g["b"]))), g["x_lower"]) < factor_tol(k), case
            assert rel_fro(_np(la.triu_solve(_gpu(g["L"]), _gpu(g["b"]))), g["x_upper"]) < factor_tol(k), case
            n += 1
        elif case.startswith("slogdet"):
            s, l = la.slogdet(_gpu(g["A"]))
            assert np.array_equal(_np(s), g["sign"]), case
            fin = np.isfinite(g["logabsdet"])
            assert np.array_equal(np.isfinite(_np(l)), fin), case
            np.testing.assert_allclose(_np(l)[fin], g["logabsdet"][fin], rtol=1e-4, atol=1e-4, err_msg=case)
            n += 1
        elif case == "clamp_k4":
            x = _np(la.solve(_gpu(g["A"]), _gpu(g["b"])))
            L = _np(la.cholesky(_gpu(g["A"])))
            assert np.all(np.isfinite(x)) and np.all(np.isfinite(L))
            np.testing.assert_allclose(L, g["L"], rtol=1e-6)
            np.testing.assert_allclose(x, g["x"], rtol=1e-5)
            n += 1
    assert n >= 50


# --------------------------------------------------------------------------
# API semantics
# --------------------------------------------------------------------------

def test_upper_triangle_is_ignored(orc):
    for k, m in ((5, 2), (16, 2), (16, 4), (24, 2), (30, 2), (40, 2), (64, 2), (90, 2), (200, 2)):
        A, b = spd_batch(6, k, m=m, seed=k)
        Ag = with_upper_garbage(A, seed=k + 1)
        assert torch.equal(la.solve(_gpu(Ag), _gpu(b)), la.solve(_gpu(A), _gpu(b))), (k, m)
        assert torch.equal(la.cholesky(_gpu(Ag)), la.cholesky(_gpu(A))), (k, m)


def test_clamp_no_nan_on_non_spd():
    for k in (3, 20, 64, 100):
        A = -np.eye(k, dtype=np.float32)[None].repeat(3, 0)
        b = np.ones((3, k, 1), np.float32)
        L = _np(la.cholesky(_gpu(A)))
        x = _np(la.solve(_gpu(A), _gpu(b)))
        np.testing.assert_allclose(np.diagonal(L, axis1=1, axis2=2), 1e-6, rtol=1e-5)
        np.testing.assert_allclose(x, 1e12, rtol=1e-4)


@pytest.mark.parametrize("k", [3, 9, 12, 16, 24, 37, 50, 64, 100, 300])
def test_nan_input_follows_the_reference(orc, k):
    """A NaN in the lower triangle of one matrix: as in the reference, the
    pivot clamp max(s, 1e-12) absorbs the NaN that reaches the later pivots,
    so that matrix's log-determinant stays finite and equals the oracle's,
    its solution is NaN where the oracle's is, and the other matrices are
    untouched. k = 24, 37 and 50 pad the matrix with identity rows, which
    the NaN reaches and which must not count."""
    A, b = spd_batch(40 if k <= 128 else 8, k, m=1, seed=77 + k)
    A[5, k - 1, k // 2] = np.nan
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    x, ld = _np(x), _np(ld)
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    np.testing.assert_allclose(ld, ld_ref, rtol=factor_tol(k), atol=factor_tol(k))
    assert np.array_equal(np.isnan(x), np.isnan(x_ref))
    ok = np.arange(A.shape[0]) != 5
    assert np.max(rel_fro_per_matrix(x[ok], x_ref[ok])) < factor_tol(k)


@pytest.mark.parametrize("k,m", [(5, 1), (16, 2), (24, 1), (48, 1), (64, 1), (64, 2), (100, 1), (300, 1)])
def test_inf_pivot_is_contained(orc, k, m):
    """+inf on one diagonal entry of one matrix. The reference gives that
    matrix L_jj = inf, logdet = +inf and a finite x (b_j / inf = 0). Here the
    tile tier (33 <= k <= 64, one right-hand side), which sums log s_j, gives
    exactly that; the other tiers form L_jj = s (1 / sqrt s) = inf * 0 and give
    a NaN logdet (and a NaN x in the thread and blocked tiers). In every tier
    the matrix's logdet is never a wrong finite number and the other matrices
    are untouched."""
    A, b = spd_batch(6, k, m=m, seed=k + 4)
    A[2, k // 2, k // 2] = np.inf
    x, ld = la.cho_solve_logdet(_gpu(A), _gpu(b))
    x, ld = _np(x), _np(ld)
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert np.isposinf(ld_ref[2]) and np.all(np.isfinite(x_ref[2]))
    assert not np.isfinite(ld[2])
    ok = np.arange(6) != 2
    np.testing.assert_allclose(ld[ok], ld_ref[ok], rtol=factor_tol(k), atol=factor_tol(k))
    assert np.max(rel_fro_per_matrix(x[ok], x_ref[ok])) < factor_tol(k)
    if 32 < k <= 64 and m == 1:
        assert np.isposinf(ld[2])
        assert rel_fro(x[2], x_ref[2]) < factor_tol(k)


def test_b_shapes_dtypes_and_host_path(orc):
    A, b = spd_batch(50, 8, m=1, seed=11)
    x2 = la.solve(_gpu(A), _gpu(b[..., 0]))
    assert tuple(x2.shape) == (50, 8)
    x3 = la.solve(_gpu(A), _gpu(b))
    assert torch.equal(x2, x3[..., 0])
    # float64 input is cast to float32
    x64 = la.solve(_gpu(A).double(), _gpu(b).double())
    assert x64.dtype == torch.float32 and torch.equal(x64, x3)
    # numpy in -> numpy out, computed through the device
    xn = la.solve(A, b)
    assert isinstance(xn, np.ndarray) and np.array_equal(xn, _np(x3))
    # CPU torch tensors go through the pipelined host path
    xc = la.solve(torch.from_numpy(A), torch.from_numpy(b))
    assert xc.device.type == "cpu" and torch.equal(xc, x3.cpu())
    # any DLPack producer (here a minimal one wrapping a device tensor)
    class Producer:
        def __init__(self, t):
            self.t = t

        def __dlpack__(self, **kw):
            return self.t.__dlpack__(**kw)

        def __dlpack_device__(self):
            return self.t.__dlpack_device__()

    xd = la.solve(Producer(_gpu(A)), _gpu(b))
    assert torch.equal(xd, x3)


def test_host_path_large_batch_chunks(orc, monkeypatch):
    import mlx_addons_b200.linalg as lam
    monkeypatch.setattr(lam, "_HOST_CHUNK_BYTES", 64 * 64 * 4 * 100)  # force many chunks
    A, b = spd_batch(1234, 64, m=1, seed=12)
    x = la.solve(torch.from_numpy(A), torch.from_numpy(b))
    assert torch.equal(x, la.solve(_gpu(A), _gpu(b)).cpu())
    s, l = la.slogdet(torch.from_numpy(A[:300]))
    s2, l2 = la.slogdet(_gpu(A[:300]))
    assert torch.equal(s, s2.cpu()) and torch.equal(l, l2.cpu())


def test_misaligned_and_noncontiguous(orc):
    for k in (5, 16, 24, 30, 48, 64, 100):
        A, b = spd_batch(9, k, m=2, seed=20 + k)
        big = torch.zeros(9 * k * k + 1, device=DEV)
        big[1:] = _gpu(A).reshape(-1)
        Am = big[1:].view(9, k, k)  # 4-byte aligned only
        assert Am.data_ptr() % 16 != 0
        ref = la.solve(_gpu(A), _gpu(b))
        # a 4-byte aligned A may take another kernel of the tier (the tile
        # loads want 16 bytes): equal within the factor tolerance
        assert np.max(rel_fro_per_matrix(_np(la.solve(Am, _gpu(b))), _np(ref))) < factor_tol(k)
        At = _gpu(np.ascontiguousarray(np.swapaxes(A, 1, 2))).transpose(1, 2)  # non-contiguous view
        assert torch.allclose(la.solve(At, _gpu(b)), ref, rtol=1e-6, atol=1e-6)


def test_x_may_alias_b_and_empty_batch():
    from mlx_addons_b200 import _lib
    lib = _lib.load()
    for k in (6, 30, 64, 70):
        A, b = spd_batch(5, k, m=2, seed=30 + k)
        Ag, bg = _gpu(A), _gpu(b)
        ref = la.solve(Ag, bg)
        ws_bytes = lib.b2c_workspace_size(0, 5, k, 2)
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=DEV)
        rc = lib.b2c_posv(Ag.data_ptr(), bg.data_ptr(), bg.data_ptr(), None, None, 5, k, 2, ws.data_ptr(),
                          ws_bytes, torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "posv")
        assert torch.equal(bg, ref)
    E = torch.zeros((0, 7, 7), device=DEV)
    assert la.solve(E, torch.zeros((0, 7, 2), device=DEV)).shape == (0, 7, 2)
    assert la.cholesky(E).shape == (0, 7, 7)
    assert la.slogdet(E)[0].shape == (0,)


def test_workspace_errors(monkeypatch):
    """The blocked kernels keep their factor in a caller workspace and refuse
    a missing one; the shared-memory tier (k <= 256) needs none, and the size
    query says so."""
    from mlx_addons_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for k in (100, 300):
        A, b = spd_batch(4, k, m=1, seed=1)
        Ag, bg = _gpu(A), _gpu(b)
        x = torch.empty_like(bg)
        rc = lib.b2c_posv(Ag.data_ptr(), bg.data_ptr(), x.data_ptr(), None, None, 4, k, 1, None, 0, stream)
        if k <= 256:
            assert lib.b2c_workspace_size(_lib.OP_POSV, 4, k, 1) == 0
            _lib.check(rc, "posv")
            assert torch.equal(x, la.solve(Ag, bg))
            # with the shared-memory tier switched off, the blocked kernel needs scratch
            monkeypatch.setenv("B2C_SMEM_TIER", "0")
            assert lib.b2c_workspace_size(_lib.OP_POSV, 4, k, 1) > 0
            rc = lib.b2c_posv(Ag.data_ptr(), bg.data_ptr(), x.data_ptr(), None, None, 4, k, 1, None, 0, stream)
            monkeypatch.delenv("B2C_SMEM_TIER")
        assert lib.b2c_workspace_size(_lib.OP_POSV, 4, k, 1) > 0 or k <= 256
        assert rc == _lib.B2C_ERR_WORKSPACE, k
        assert b"workspace" in lib.b2c_last_error()


# --------------------------------------------------------------------------
# full benchmark sizes: size-independent properties on sampled matrices
# --------------------------------------------------------------------------

def _gpu_spd(B, k, m, eps, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    G = torch.randn((B, k, k), generator=g, device=DEV)
    A = torch.bmm(G, G.transpose(1, 2)) / k
    A.diagonal(dim1=1, dim2=2).add_(eps)
    b = torch.randn((B, k, m), generator=g, device=DEV)
    return A, b


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_size_configs(orc, name):
    B, k, m, eps = CONFIGS[name]
    A, b = _gpu_spd(B, k, m, eps, seed=31 * k + m)
    x, ld = la.cho_solve_logdet(A, b)
    torch.cuda.synchronize()
    assert torch.isfinite(x).all() and torch.isfinite(ld).all()
    idx = torch.randperm(B, device="cpu")[:24]
    As, bs, xs, lds = (_np(t[idx.to(DEV)]) for t in (A, b, x, ld))
    assert np.max(backward_error(As, xs, bs)) < backward_tol(k)
    x_ref, ld_ref = orc.solve(As, bs, return_logdet=True)
    assert np.max(rel_fro_per_matrix(xs, x_ref)) < factor_tol(k)
    np.testing.assert_allclose(lds, ld_ref, rtol=5e-5, atol=5e-5)
    # solve and the fused call agree exactly on the same input
    assert torch.equal(la.solve(A[:64], b[:64]), x[:64])
    # the factor of the whole batch, ||L - L_ref||_F / ||L_ref||_F on the samples
    L = la.cholesky(A)
    Ls = _np(L[idx.to(DEV)])
    del L
    assert np.all(np.triu(Ls, 1) == 0)
    assert np.max(rel_fro_per_matrix(Ls, orc.cholesky(As))) < factor_tol(k)


def test_solve_sharded_single_device_matches_solve():
    from mlx_addons_b200.linalg._shard import solve_sharded
    A, b = spd_batch(101, 64, m=1, seed=41)
    outs = solve_sharded(torch.from_numpy(A), torch.from_numpy(b), devices=[0])
    assert len(outs) == 1 and outs[0].device.type == "cuda"
    assert torch.equal(outs[0], la.solve(_gpu(A), _gpu(b)))


@pytest.mark.parametrize("k", [16, 64, 100])
def test_solve_sharded_over_two_devices(orc, k):
    """The batch split over two GPUs (contiguous shards, one stream each, no
    collective): every shard equals the one-device solve of the same rows, on
    the device that owns it."""
    from mlx_addons_b200.linalg._shard import shard_bounds, solve_sharded
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    A, b = spd_batch(1001, k, m=1, seed=43 + k)
    outs = solve_sharded(torch.from_numpy(A), torch.from_numpy(b), devices=[0, 1])
    assert [o.device.index for o in outs] == [0, 1]
    x_one = la.solve(_gpu(A), _gpu(b)).cpu()
    for (lo, hi), o in zip(shard_bounds(1001, 2), outs):
        assert torch.equal(o.cpu(), x_one[lo:hi])
    x_ref = orc.solve(A, b)
    assert np.max(rel_fro_per_matrix(torch.cat([o.cpu() for o in outs]).numpy(), x_ref)) < factor_tol(k)


@pytest.mark.parametrize("k", [5, 16, 64, 100])
def test_pinned_host_inputs_zero_copy(k):
    """Pinned host inputs go to the kernels directly (zero-copy); results are
    host tensors equal to the device path's: bit for bit up to k = 64; above,
    host A takes the shared-memory tier's cp.async kernel while device A may
    take its TMA task-graph kernel, so equal within the factor tolerance."""
    A, b = spd_batch(300, k, m=2, seed=60 + k)
    Ah, bh = torch.from_numpy(A).pin_memory(), torch.from_numpy(b).pin_memory()
    Ad, bd = _gpu(A), _gpu(b)

    def same(h, d):
        if k <= 64:
            return torch.equal(h, d.cpu())
        return float(np.max(rel_fro_per_matrix(_np(h.reshape(h.shape[0], -1)), _np(d.reshape(d.shape[0], -1))))) \
            < factor_tol(k)

    x, ld = la.cho_solve_logdet(Ah, bh)
    assert x.device.type == "cpu" and ld.device.type == "cpu"
    xr, ldr = la.cho_solve_logdet(Ad, bd)
    assert same(x, xr)
    np.testing.assert_allclose(_np(ld), _np(ldr), rtol=0 if k <= 64 else factor_tol(k), atol=0)
    assert same(la.solve(Ah, bh[..., 0]), la.solve(Ad, bd[..., 0]))
    assert same(la.cholesky(Ah), la.cholesky(Ad))
    np.testing.assert_allclose(_np(la.logdet_spd(Ah)), _np(la.logdet_spd(Ad)),
                               rtol=0 if k <= 64 else factor_tol(k), atol=0)
    s, l = la.slogdet(Ah)
    s2, l2 = la.slogdet(Ad)
    assert torch.equal(s, s2.cpu()) and torch.equal(l, l2.cpu())
