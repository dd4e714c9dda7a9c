"""Write the golden fixtures in tests/golden/ from the reference itself.

Runs only where the reference tree exists (the development container): it
imports the reference's ``mlx_addons.linalg`` over the numpy stand-in for MLX
(``oracle/mlx_shim.py``), whose kernels are the reference's own kernel bodies
compiled for the host (``oracle/build_ref.py``), and records inputs and
outputs of the public functions on small seeded cases, including the edge
cases the reference semantics define (ragged last block, 2-D b, garbage in
the strict upper triangle, clamped non-SPD pivots).

Usage: python tests/golden/make_golden.py
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

from tests._data import CONFIGS, general_batch, spd_batch, with_upper_garbage  # noqa: E402


def main():
    import oracle
    from oracle import build_ref, mlx_shim

    if build_ref.build(quiet=True) is None:
        raise SystemExit("reference tree not found; golden fixtures are generated where it exists")
    oracle.build()
    ref = mlx_shim.load_reference_linalg()

    out = {}

    def put(name, **arrays):
        for key, val in arrays.items():
            out[f"{name}/{key}"] = np.asarray(val)

    # solve / cholesky / logdet_spd across the tier and block boundaries
    solve_ks = [1, 2, 3, 5, 8, 16, 20, 31, 32, 33, 48, 63, 64, 65, 80, 81, 96, 128, 130, 160, 256]
    for i, k in enumerate(solve_ks):
        B = 6 if k <= 128 else 2
        m = 1 if i % 2 == 0 else 3
        A, b = spd_batch(B, k, m=m, eps=1.0, seed=100 + k)
        put(f"solve_k{k}_m{m}", A=A, b=b, x=ref.solve(A, b), L=ref.cholesky(A), logdet=ref.logdet_spd(A))
    # the small-kernel solve (solve_cholesky), LG tier range
    for k in (96, 128):
        A, b = spd_batch(4, k, m=2, seed=200 + k)
        put(f"solve_cholesky_k{k}", A=A, b=b, x=ref.solve_cholesky(A, b))
    # 2-D b round trip
    A, b = spd_batch(5, 12, m=1, seed=300)
    put("solve_b2d_k12", A=A, b=b[..., 0], x=ref.solve(A, b[..., 0]))
    A, b = spd_batch(3, 100, m=1, seed=301)
    put("solve_b2d_k100", A=A, b=b[..., 0], x=ref.solve(A, b[..., 0]))
    # upper-triangle garbage is ignored
    for k in (7, 40, 90):
        A, b = spd_batch(4, k, m=2, seed=400 + k)
        Ag = with_upper_garbage(A, seed=401 + k)
        put(f"upper_garbage_k{k}", A=Ag, b=b, x=ref.solve(Ag, b), L=ref.cholesky(Ag))
    # clamped pivots: non-SPD input yields sqrt(1e-12) pivots, no NaN
    A = np.zeros((3, 4, 4), np.float32)
    A[0] = np.diag([1.0, -1.0, 1.0, 4.0])
    A[1] = np.diag([0.0, 2.0, 0.0, 9.0])
    A[2] = np.diag([-5.0, -5.0, -5.0, -5.0])
    b = np.ones((3, 4, 1), np.float32)
    put("clamp_k4", A=A, b=b, x=ref.solve(A, b), L=ref.cholesky(A))
    # triangular solves (k <= 128, the reference's small kernels)
    for k in (1, 6, 20, 32, 33, 48, 64, 80, 96, 128):
        A, b = spd_batch(5, k, m=2, seed=500 + k)
        L = ref.cholesky(A)
        put(f"tri_k{k}", L=L, b=b, x_lower=ref.tril_solve(L, b), x_upper=ref.triu_solve(L, b))
    # slogdet / det on general and SPD matrices, with extra leading dims
    for n in (1, 2, 3, 5, 10, 20, 50, 64, 128, 200):
        G = general_batch(6 if n <= 64 else 2, n, seed=600 + n)
        s, l = ref.slogdet(G)
        put(f"slogdet_general_n{n}", A=G, sign=s.astype(np.float32), logabsdet=l)
    A, _ = spd_batch(6, 256, seed=700)[0][:2], None
    s, l = ref.slogdet(A)
    put("slogdet_spd_n256", A=A, sign=s.astype(np.float32), logabsdet=l)
    G = general_batch(12, 6, seed=701).reshape(2, 3, 2, 6, 6)
    s, l = ref.slogdet(G)
    put("slogdet_lead_dims_n6", A=G, sign=s.astype(np.float32), logabsdet=l, det=ref.det(G))
    Sg = np.zeros((2, 4, 4), np.float32)
    Sg[0] = np.arange(16, dtype=np.float32).reshape(4, 4)  # singular
    Sg[1] = np.eye(4, dtype=np.float32)[[1, 0, 3, 2]]       # permutation, det +1
    s, l = ref.slogdet(Sg)
    put("slogdet_special_n4", A=Sg, sign=s.astype(np.float32), logabsdet=l)
    # solve_lu on general matrices (both reference kernels), special cases
    for k in (1, 3, 5, 16, 32, 33, 64, 100, 128):
        G = general_batch(6 if k <= 64 else 2, k, seed=1000 + k)
        b = np.random.default_rng(1100 + k).standard_normal((G.shape[0], k, 2), dtype=np.float32)
        put(f"solve_lu_k{k}", A=G, b=b, x=ref.solve_lu(G, b))
    Sg = np.zeros((3, 4, 4), np.float32)
    Sg[0] = np.eye(4, dtype=np.float32)[[2, 0, 3, 1]]       # permutation
    # singular (zero column and zero row) with an exact elimination: every
    # multiplier is a power of two, so inf / NaN positions are rounding-free
    Sg[1] = np.array([[4, 2, 0, 1], [2, 3, 0, 1], [0, 0, 0, 0], [1, 1, 0, 2]], np.float32)
    Sg[2] = np.triu(np.arange(1, 17, dtype=np.float32).reshape(4, 4))
    bs = np.arange(12, dtype=np.float32).reshape(3, 4, 1) - 5.0
    put("solve_lu_special_k4", A=Sg, b=bs, x=ref.solve_lu(Sg, bs))
    G = general_batch(3, 10, seed=1200)
    put("solve_lu_b2d_k10", A=G, b=G[:, :, 0].copy(), x=ref.solve_lu(G, G[:, :, 0].copy()))
    # Householder qr: single-thread kernel (k < 12), threadgroup kernel
    # (12..63), CPU LAPACK above (_metal_kernels.py:641-694)
    for k in (1, 3, 5, 8, 11, 12, 16, 20, 32, 48, 63, 64, 96):
        G = general_batch(5 if k <= 63 else 2, k, seed=1300 + k)
        Q, R = ref.qr(G)
        put(f"qr_k{k}", A=G, Q=Q, R=R)
    G = general_batch(1, 10, seed=1400)[0]
    Q, R = ref.qr(G)
    put("qr_2d_k10", A=G, Q=Q, R=R)
    # randomized_svd (_svd.py:48-175): low-rank with a decaying spectrum
    # (vectors well defined) and Gaussian (singular values only), 2-D and
    # batched, true rank below k + p included
    def low_rank(rng, n, m, r, decay):
        U_, _ = np.linalg.qr(rng.standard_normal((n, r)).astype(np.float32))
        V_, _ = np.linalg.qr(rng.standard_normal((m, r)).astype(np.float32))
        return ((U_ * (10.0 * np.exp(-decay * np.arange(r))).astype(np.float32)) @ V_.T).astype(np.float32)

    rng = np.random.default_rng(1500)
    for name, X, k, it in (("rsvd_lowrank_100x30_k6", low_rank(rng, 100, 30, 10, 0.3), 6, 6),
                           ("rsvd_lowrank_500x128_k16", low_rank(rng, 500, 128, 32, 0.3), 16, 6),
                           ("rsvd_gauss_300x80_k20", rng.standard_normal((300, 80)).astype(np.float32), 20, 4),
                           ("rsvd_batched_4x300x60_k12",
                            np.stack([low_rank(rng, 300, 60, 20, 0.2) for _ in range(4)]), 12, 6)):
        U, S, Vt = ref.randomized_svd(X, n_components=k, n_iter=it, random_state=0)
        put(name, X=X, U=U, S=S, Vt=Vt, k=np.int64(k), n_iter=np.int64(it))
    # small samples of every benchmark configuration's distribution
    for name, (_, k, m, eps) in CONFIGS.items():
        Bs = 8 if k <= 64 else (2 if k <= 256 else 1)
        A, b = spd_batch(Bs, k, m=m, eps=eps, seed=900 + k)
        arrays = dict(A=A, b=b, x=ref.solve(A, b), logdet=ref.logdet_spd(A))
        if k <= 256:
            arrays["L"] = ref.cholesky(A)
        put(f"config_{name}", **arrays)

    path = os.path.join(HERE, "reference_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path) / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
