"""mlx_addons_b200 — the batched SPD Cholesky-solve path of
guillaume-osmo/mlx-addons (``mlx_addons.linalg``), rebuilt for NVIDIA B200.

The Python layer (``mlx_addons_b200.linalg``) mirrors the reference API; the
work happens in hand-written sm_100a CUDA kernels behind the C ABI of
``libb2c.so`` (declared in ``include/b2c.h``).
"""

__version__ = "0.1.0"

from . import linalg  # noqa: E402,F401
