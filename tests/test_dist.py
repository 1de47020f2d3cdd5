"""Multi-rank host logic on CPU with the gloo backend (world size 2).

The device kernels are not involved: each rank forms its f64 partial with
numpy over its shard, the partials go through the same all-reduce the GPU
path uses, and the finalised sum/mean must equal the oracle.  A rank that
leaves before the collective makes its peer fail with a timeout error.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from lazy_compiler_b200.dist import shard
from oracle import expressions as O


@pytest.mark.parametrize("n", [0, 1, 7, 100, 1 << 20, 1000003])
@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_cover_range_exactly(n, world):
    covered = []
    for r in range(world):
        start, count = shard(n, world, r)
        covered.extend(range(start, start + count))
    assert covered == list(range(n))
    counts = [shard(n, world, r)[1] for r in range(world)]
    assert max(counts) - min(counts) <= 1


def test_shard_rejects_bad_requests():
    for args in ((10, 0, 0), (10, 2, 2), (-1, 2, 0)):
        with pytest.raises(ValueError):
            shard(*args)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _sum_worker(rank, world, port, n, results):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    x = O.uniform(n, seed=0)
    start, count = shard(n, world, rank)
    partial = torch.tensor([x[start:start + count].astype(np.float64).sum()], dtype=torch.float64)
    dist.all_reduce(partial)
    results[rank] = (float(np.float32(partial.item())), float(np.float32(partial.item() / n)))
    dist.destroy_process_group()


def test_partial_allreduce_matches_oracle_gloo():
    n = 1_000_003
    port = _port()
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_sum_worker, args=(2, port, n, results), nprocs=2, join=True)
        got = dict(results)
    x = O.uniform(n, seed=0)
    for rank in range(2):
        assert got[rank][0] == float(O.sum_(x)[0])
        assert got[rank][1] == float(O.mean(x)[0])


def _failing_worker(rank, world, port, results):
    import datetime

    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        return  # leaves without joining the collective
    t = torch.ones(1)
    try:
        dist.all_reduce(t)
        results[rank] = "completed"
    except Exception as exc:  # the survivor learns of the failure through the timeout
        results[rank] = type(exc).__name__


def test_survivor_times_out_when_a_rank_leaves_gloo():
    port = _port()
    with mp.Manager() as manager:
        results = manager.dict()
        ctx = mp.start_processes(_failing_worker, args=(2, port, results), nprocs=2, join=False,
                                 start_method="spawn")
        for p in ctx.processes:
            p.join(timeout=60)
        for p in ctx.processes:
            if p.is_alive():
                p.kill()
        got = dict(results)
    assert got.get(0) not in (None, "completed")
