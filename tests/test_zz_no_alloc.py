"""b2c_posv_static_scratch, the entry point that allocates nothing.

It serves callers that cannot allocate GPU memory while they solve (an
allocator that forbids cudaMalloc in steady state, memory partitioned up
front, a plugin host that hands over only inputs and outputs): its scratch is
a fixed 16 MiB array inside the library, so k <= 2048 and at most
16 MiB / (4 k^2) matrices are factored at a time. Results are checked against
the oracle at the tolerances of the other tests, on two calls in a row (the
second finds the first one's data in the shared array). This file is
collected last so that a run stopping at the first failure has already run
every other test; it passes on its own in a fresh process too, since every
call outside stream capture looks the array's address up itself.
"""

import ctypes

import numpy as np
import pytest
import torch

from mlx_addons_b200 import _lib
from tests._data import spd_batch
from tests._tol import backward_error, backward_tol, factor_tol, rel_fro_per_matrix

pytestmark = pytest.mark.gpu

FORM_ENV = {"smem": {}, "ffma": {"B2C_SMEM_TIER": "0"}, "tc": {"B2C_BLOCKED_GEMM": "tc"}}


@pytest.fixture(autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _fault():
    f = ctypes.c_uint(7)
    assert _lib.load().b2c_take_device_fault(ctypes.byref(f)) == 0
    return f.value


def _call(lib, Ag, bg, x, ld, B, k, m):
    _lib.check(lib.b2c_posv_static_scratch(Ag.data_ptr(), bg.data_ptr(), x.data_ptr(), ld.data_ptr(), B, k, m,
                                           _stream()), "b2c_posv_static_scratch")


def _check(orc, A, b, x, ld, k):
    x_ref, ld_ref = orc.solve(A, b, return_logdet=True)
    assert np.all(np.isfinite(x))
    assert np.max(rel_fro_per_matrix(x, x_ref)) < factor_tol(k)
    assert np.max(backward_error(A, x, b)) < backward_tol(k)
    np.testing.assert_allclose(ld, ld_ref, rtol=factor_tol(k), atol=factor_tol(k))


# (k, m, B): k = 5 and 64 take the launcher above k = 64 too; k = 1024 holds 4
# matrices in the array (B = 9 walks them several times), k = 2048 holds one
@pytest.mark.parametrize("k,m,B", [(5, 1, 40), (64, 1, 40), (100, 2, 40), (512, 1, 20), (1024, 1, 9),
                                   (2048, 1, 3)])
def test_static_scratch_vs_oracle(orc, k, m, B):
    lib = _lib.load()
    A, b = spd_batch(B, k, m=m, seed=77 + k)
    Ag, bg = torch.from_numpy(A).cuda(), torch.from_numpy(b).cuda()
    for _ in range(2):  # two calls in a row share the library's array
        x = torch.full_like(bg, float("nan"))
        ld = torch.full((B,), float("nan"), device="cuda")
        _call(lib, Ag, bg, x, ld, B, k, m)
        torch.cuda.synchronize()
        _check(orc, A, b, x.cpu().numpy(), ld.cpu().numpy(), k)
    assert _fault() == 0


@pytest.mark.parametrize("form", ["smem", "ffma", "tc"])
@pytest.mark.parametrize("k", [100, 300])
def test_static_scratch_forms(orc, monkeypatch, form, k):
    """The shared-memory tier, the FFMA blocked tier and the tensor-core blocked
    tier all run from the library's array."""
    for key, val in FORM_ENV[form].items():
        monkeypatch.setenv(key, val)
    lib = _lib.load()
    B = 21
    A, b = spd_batch(B, k, m=1, seed=300 + k)
    Ag, bg = torch.from_numpy(A).cuda(), torch.from_numpy(b).cuda()
    for _ in range(2):
        x = torch.full_like(bg, float("nan"))
        ld = torch.full((B,), float("nan"), device="cuda")
        _call(lib, Ag, bg, x, ld, B, k, 1)
        torch.cuda.synchronize()
        _check(orc, A, b, x.cpu().numpy(), ld.cpu().numpy(), k)
    assert _fault() == 0


def test_static_scratch_in_a_cuda_graph(orc):
    """A call captured in a CUDA graph uses the address the last call outside
    capture recorded for this context."""
    lib = _lib.load()
    k, B = 512, 12
    A, b = spd_batch(B, k, m=1, seed=5)
    Ag, bg = torch.from_numpy(A).cuda(), torch.from_numpy(b).cuda()
    x = torch.empty_like(bg)
    ld = torch.empty((B,), device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        _call(lib, Ag, bg, x, ld, B, k, 1)  # outside capture: looks the address up
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        _call(lib, Ag, bg, x, ld, B, k, 1)
    x.fill_(float("nan"))
    ld.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    del g
    _check(orc, A, b, x.cpu().numpy(), ld.cpu().numpy(), k)


def test_static_scratch_on_two_devices(orc):
    """Each device has its own copy of the array (a device address is valid
    only in its own context); alternate between two GPUs."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    lib = _lib.load()
    k, B = 300, 8
    A, b = spd_batch(B, k, m=1, seed=6)
    for dev in (1, 0, 1):
        with torch.cuda.device(dev):
            Ag, bg = torch.from_numpy(A).cuda(), torch.from_numpy(b).cuda()
            x = torch.full_like(bg, float("nan"))
            ld = torch.full((B,), float("nan"), device="cuda")
            _call(lib, Ag, bg, x, ld, B, k, 1)
            torch.cuda.synchronize()
            _check(orc, A, b, x.cpu().numpy(), ld.cpu().numpy(), k)


def test_static_scratch_rejects_k_beyond_its_array():
    lib = _lib.load()
    dummy = torch.empty(16, device="cuda")
    rc = lib.b2c_posv_static_scratch(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), None, 1, 4096, 1,
                                     _stream())
    assert rc == _lib.B2C_ERR_UNSUPPORTED
    assert b"2048" in lib.b2c_last_error()
