"""Multi-GPU parity: the range-sharded sum/mean over NCCL equals the oracle.

Runs one process per GPU on the first two GPUs (skipped with fewer than two).
Each rank takes its contiguous shard of the same seeded array, reduces it to
an f64 partial on its GPU, the partials are all-reduced over NCCL and every
rank finalises; the result must equal the float64 oracle within 1e-5.
NVLS is off and the process group has a short timeout.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import expressions as O

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, results):
    import datetime

    import torch
    import torch.distributed as dist

    from lazy_compiler_b200.dist import shard, sharded_sum
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    x = O.uniform(n, seed=5)
    start, count = shard(n, world, rank)
    xs = torch.from_numpy(x[start:start + count].copy()).cuda()
    out = torch.empty(2, device="cuda")
    total = torch.tensor([float(n)], device="cuda")
    sharded_sum(xs, count, out[:1])
    sharded_sum(xs, count, out[1:], total)
    results[rank] = out.cpu().numpy().tolist()
    dist.destroy_process_group()


def test_sharded_sum_two_gpus_matches_oracle(cuda_device):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    n = (1 << 24) + 13
    with mp.Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(2, _port(), n, results), nprocs=2, join=True)
        got = dict(results)
    x = O.uniform(n, seed=5)
    for rank in range(2):
        assert np.isclose(got[rank][0], O.sum_(x)[0], rtol=1e-5, atol=1e-30)
        assert np.isclose(got[rank][1], O.mean(x)[0], rtol=1e-5, atol=1e-30)
