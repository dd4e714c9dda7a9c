"""Batch sharding host logic, including world-size-2 runs over gloo on CPU.

The compute inside the gloo ranks is the oracle (the CPU checker), standing in
for the per-GPU kernels; what is tested is the partition, the per-rank
slicing, reassembly order and the max-over-ranks timing reduction.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlx_addons_b200.linalg._shard import local_shard, max_over_ranks, run_local_shard, shard_bounds
from tests._data import spd_batch


@pytest.mark.parametrize("batch,world", [(0, 1), (1, 2), (7, 2), (10_000, 8), (10_001, 8), (3, 4)])
def test_shard_bounds_partition(batch, world):
    b = shard_bounds(batch, world)
    assert len(b) == world
    assert b[0][0] == 0 and b[-1][1] == batch
    for (lo, hi), (lo2, _) in zip(b, b[1:]):
        assert hi == lo2
    sizes = [hi - lo for lo, hi in b]
    assert max(sizes) - min(sizes) <= 1
    assert sizes == sorted(sizes, reverse=True)


def test_shard_bounds_errors():
    with pytest.raises(ValueError):
        shard_bounds(5, 0)
    with pytest.raises(ValueError):
        local_shard(5, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        import oracle
        A, b = spd_batch(37, 12, m=2, seed=5)
        x = run_local_shard(lambda a, bb: oracle.solve(a, bb, nthreads=1), [A, b], rank, world)
        xt = torch.from_numpy(np.ascontiguousarray(x))
        sizes = [hi - lo for lo, hi in shard_bounds(37, world)]
        parts = [torch.empty((n, 12, 2)) for n in sizes]
        # gloo all_gather needs equal shapes: pad to the largest shard
        pad = max(sizes)
        buf = torch.zeros((pad, 12, 2))
        buf[: xt.shape[0]] = xt
        gathered = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(gathered, buf)
        full = torch.cat([g[:n] for g, n in zip(gathered, sizes)]).numpy()
        slowest = max_over_ranks(0.5 + rank)
        q.put((rank, full, slowest))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_shards_reassemble(orc):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    A, b = spd_batch(37, 12, m=2, seed=5)
    ref = orc.solve(A, b)
    for rank, full, slowest in res:
        assert np.array_equal(full, ref), rank
        assert slowest == 1.5
