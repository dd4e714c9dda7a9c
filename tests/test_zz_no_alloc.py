"""b2c_posv_static_scratch, the entry point that allocates nothing.

It serves callers that cannot allocate GPU memory while they solve (an
allocator that forbids cudaMalloc in steady state, memory partitioned up
front, a plugin host that hands over only inputs and outputs): its scratch is
a fixed array inside the library. This file is collected last so that a run
stopping at the first failure has already run every other test; it passes on
its own in a fresh process too, since the entry point sets itself up on its
first call.
"""

import numpy as np
import pytest
import torch

from mlx_addons_b200 import _lib
from tests._data import spd_batch
from tests._tol import factor_tol, rel_fro_per_matrix

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("k,m,B", [(100, 2, 40), (512, 1, 20)])
def test_static_scratch_matches_posv(k, m, B):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    A, b = spd_batch(B, k, m=m, seed=77 + k)
    Ag, bg = torch.from_numpy(A).cuda(), torch.from_numpy(b).cuda()
    # reference result: the existing entry point with a caller workspace
    ws_bytes = int(lib.b2c_workspace_size(_lib.OP_POSV, B, k, m))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    x_ref = torch.empty_like(bg)
    ld_ref = torch.empty(B, device="cuda")
    _lib.check(lib.b2c_posv(Ag.data_ptr(), bg.data_ptr(), x_ref.data_ptr(), None, ld_ref.data_ptr(), B, k, m,
                            ws.data_ptr(), ws_bytes, _stream()), "b2c_posv")
    for _ in range(2):  # two calls in a row share the library's scratch
        x = torch.full_like(bg, float("nan"))
        ld = torch.full((B,), float("nan"), device="cuda")
        _lib.check(lib.b2c_posv_static_scratch(Ag.data_ptr(), bg.data_ptr(), x.data_ptr(), ld.data_ptr(), B, k, m,
                                               _stream()), "b2c_posv_static_scratch")
        torch.cuda.synchronize()
        assert torch.isfinite(x).all()
        assert np.max(rel_fro_per_matrix(x.cpu().numpy(), x_ref.cpu().numpy())) < factor_tol(k)
        np.testing.assert_allclose(ld.cpu().numpy(), ld_ref.cpu().numpy(), rtol=factor_tol(k), atol=factor_tol(k))


def test_static_scratch_rejects_k_beyond_its_array():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = _lib.load()
    dummy = torch.empty(16, device="cuda")
    rc = lib.b2c_posv_static_scratch(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None, 1, 4096, 1,
                                     _stream())
    assert rc == _lib.B2C_ERR_UNSUPPORTED
    assert b"2048" in lib.b2c_last_error()
