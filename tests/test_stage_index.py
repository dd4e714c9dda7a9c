"""CPU checks of the index arithmetic of the chunked staging loops of the
k <= 64 tiers, for every k they serve with 16-byte copies (k % 4 == 0):
which 16-byte chunks of A each warp copies into shared memory, from where and
to where. The loops are restated here lane by lane from tile_stage
(mlx_addons_b200/csrc/posv_tile.cu) and w64_stage
(mlx_addons_b200/csrc/posv_warp64.cu); a change to either loop needs the same
change here.

Checked: every chunk holding a lower-triangle entry of rows < k is copied
exactly once and only those; every read stays inside its row of the k x k
matrix; the tile layout writes identity chunks for the padding rows k..KP-1
that cover their lower triangle; destinations are 16-byte aligned, distinct
and inside the staged matrix."""

import pytest


def _tile_layout(KP):
    rowbase = lambda r: 32 * r if r < 32 else 1024 + 64 * (r - 32)  # noqa: E731
    chunkpos = lambda r, q: (q & 8) | ((q & 7) ^ (r & 7))  # noqa: E731
    return rowbase, chunkpos, rowbase(KP)


def _tile_stage(K, KP):
    """(copies, identity) of one warp: copies = [(dst, src_float, r, q)],
    identity = [(dst, r, q)], dst in floats."""
    rowbase, chunkpos, _ = _tile_layout(KP)
    dst = lambda r, q: rowbase(r) + 4 * chunkpos(r, q)  # noqa: E731
    copies, ident = [], []
    for t in range(8):
        for lane in range(32):
            r, q = (lane >> 3) + 4 * t, lane & 7
            if q <= t:
                copies.append((dst(r, q), r * K + 4 * q, r, q))
    Q, TOTAL = KP // 4, (KP - 32) * (KP // 4)
    for f0 in range(0, TOTAL, 32):
        for lane in range(32):
            f = f0 + lane
            r, q = 32 + f // Q, f % Q
            if f < TOTAL and q <= (r >> 2):
                if r < K:
                    copies.append((dst(r, q), r * K + 4 * q, r, q))
                else:
                    ident.append((dst(r, q), r, q))
    return copies, ident


def _tile_kp(k):
    return 48 if k <= 48 else 64


@pytest.mark.parametrize("K", list(range(36, 65, 4)))
def test_tile_stage_chunks(K):
    KP = _tile_kp(K)
    _, _, MAT = _tile_layout(KP)
    copies, ident = _tile_stage(K, KP)
    want = {(r, q) for r in range(K) for q in range(KP // 4) if 4 * q <= r}
    got = [(r, q) for _, _, r, q in copies]
    assert sorted(got) == sorted(want)  # each lower-triangle chunk once
    for _, src, r, q in copies:
        assert r * K <= src and src + 3 < (r + 1) * K  # inside row r of A
        assert src % 4 == 0  # 16-byte aligned when A and k % 4 == 0 are
    want_id = {(r, q) for r in range(K, KP) for q in range(KP // 4) if 4 * q <= r}
    assert sorted((r, q) for _, r, q in ident) == sorted(want_id)
    assert all(r >= 32 for _, r, _ in ident)  # the padding rows lie in the second loop
    dsts = [d for d, *_ in copies] + [d for d, *_ in ident]
    assert len(set(dsts)) == len(dsts)
    assert all(d % 4 == 0 and 0 <= d and d + 4 <= MAT for d in dsts)


def _w64_layout(KP):
    NB = KP - 32
    SW1 = KP % 32 == 0
    S1 = KP if SW1 else KP + 4
    off0 = lambda r, q: r * 32 + 4 * (q ^ (r & 7))  # noqa: E731
    off1 = (lambda r, q: 1024 + r * KP + 4 * (q ^ (r & 7))) if SW1 else (lambda r, q: 1024 + r * S1 + 4 * q)
    return NB, off0, off1, 1024 + NB * S1


def _w64_stage(K, KP):
    NB, off0, off1, _ = _w64_layout(KP)
    copies = []
    for t in range(8):
        for lane in range(32):
            r, q = (lane >> 3) + 4 * t, lane & 7
            if q <= t:
                copies.append((off0(r, q), r * K + 4 * q, r, q))
    Q, TOTAL = KP // 4, NB * (KP // 4)
    for f0 in range(0, TOTAL, 32):
        for lane in range(32):
            f = f0 + lane
            if f < TOTAL:
                r, q = f // Q, f - (f // Q) * Q
                if 32 + r < K and q <= 8 + (r >> 2):
                    copies.append((off1(r, q), (32 + r) * K + 4 * q, 32 + r, q))
    return copies


def _w64_kp(k):
    return 40 if k <= 40 else 48 if k <= 48 else 56 if k <= 56 else 64


@pytest.mark.parametrize("K", list(range(36, 65, 4)))
def test_warp64_stage_chunks(K):
    KP = _w64_kp(K)
    *_, STAGE = _w64_layout(KP)
    copies = _w64_stage(K, KP)
    want = {(r, q) for r in range(K) for q in range(KP // 4) if 4 * q <= r}
    assert sorted((r, q) for *_, r, q in copies) == sorted(want)
    for _, src, r, q in copies:
        assert r * K <= src and src + 3 < (r + 1) * K
    dsts = [d for d, *_ in copies]
    assert len(set(dsts)) == len(dsts)
    assert all(d % 4 == 0 and 0 <= d and d + 4 <= STAGE for d in dsts)
