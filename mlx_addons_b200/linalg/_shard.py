"""Batch sharding across GPUs.

Every matrix of a batched solve is independent (the reference's launch grid
runs over the batch only, src/mlx_addons/linalg/_metal_kernels.py:504-512), so
the path scales by splitting the batch into contiguous shards, one per GPU,
with no collective on the data path: each GPU reads its shard from its own
HBM and its results stay there.

Two ways to use it:

* one process per GPU (torchrun): ``local_shard(batch, rank, world)`` gives
  the rank's [lo, hi) slice and ``run_local_shard`` applies a solver to it;
* one process driving several GPUs: ``solve_sharded`` copies each shard to its
  device and launches there, one stream per device; the per-device results
  are returned without gathering.
"""

from __future__ import annotations

from typing import Callable, List, Sequence, Tuple


def shard_bounds(batch: int, world: int) -> List[Tuple[int, int]]:
    """Contiguous [lo, hi) slices covering range(batch); sizes differ by at
    most one and the first ``batch % world`` shards are the larger ones."""
    if world < 1:
        raise ValueError("world must be >= 1")
    if batch < 0:
        raise ValueError("batch must be >= 0")
    base, extra = divmod(batch, world)
    out, lo = [], 0
    for r in range(world):
        hi = lo + base + (1 if r < extra else 0)
        out.append((lo, hi))
        lo = hi
    return out


def local_shard(batch: int, rank: int, world: int) -> Tuple[int, int]:
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    return shard_bounds(batch, world)[rank]


def run_local_shard(solver: Callable, arrays: Sequence, rank: int, world: int):
    """Apply ``solver`` to this rank's slice of every array (batch first)."""
    batch = arrays[0].shape[0]
    for a in arrays:
        if a.shape[0] != batch:
            raise ValueError("all arrays must share the batch dimension")
    lo, hi = local_shard(batch, rank, world)
    return solver(*[a[lo:hi] for a in arrays])


def max_over_ranks(seconds: float, device=None) -> float:
    """Slowest rank's time (the bench reports throughput against it)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(seconds)
    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def solve_sharded(A, b, devices: Sequence[int] = None, solver: Callable = None):
    """Split (A, b) over ``devices`` (default: all visible GPUs), solve each
    shard on its own device and stream, return the list of per-device x."""
    import torch

    if solver is None:
        from . import solve as solver
    if devices is None:
        devices = list(range(torch.cuda.device_count()))
    if not devices:
        raise RuntimeError("solve_sharded needs at least one CUDA device")
    outs = []
    for (lo, hi), dev in zip(shard_bounds(A.shape[0], len(devices)), devices):
        d = torch.device("cuda", dev)
        with torch.cuda.device(d), torch.cuda.stream(torch.cuda.Stream(d)):
            outs.append(solver(A[lo:hi].to(d, non_blocking=True), b[lo:hi].to(d, non_blocking=True)))
    for dev in devices:
        torch.cuda.synchronize(dev)
    return outs
