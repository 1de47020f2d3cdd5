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
    with mp.get_context("spawn").Manager() as manager:
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
    with mp.get_context("spawn").Manager() as manager:
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


def _rows_worker(rank, world, port, results):
    import datetime

    import torch
    import torch.distributed as dist

    from lazy_compiler_b200.dist import gather
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    rows, cols = 1001, 37
    x = O.normal((rows, cols), 3)
    start, count = shard(rows, world, rank)
    local = torch.from_numpy(O.rowsum(x[start:start + count])[0])
    whole = gather(local, rows)
    results[rank] = np.array_equal(whole.numpy(), O.rowsum(x)[0])
    blocks = torch.from_numpy(x[start:start + count].copy())
    results[rank] = results[rank] and np.array_equal(gather(blocks, rows).numpy(), x)
    dist.destroy_process_group()


def test_row_blocks_gather_to_the_whole_gloo():
    """Row-block shards computed per rank and all-gathered equal the whole-array oracle (uneven split)."""
    port = _port()
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        mp.spawn(_rows_worker, args=(2, port, results), nprocs=2, join=True)
        got = dict(results)
    assert got == {0: True, 1: True}


def test_partition_helpers_reject_a_wrong_local_shape():
    import torch

    from lazy_compiler_b200 import dist as D
    x = torch.zeros(9, 4)
    out = torch.zeros(9, 4)
    with pytest.raises(ValueError, match="this rank owns"):
        D.sharded_rows("softmax", 10, 4, x, out)
    with pytest.raises(ValueError, match="this rank owns"):
        D.sharded_gemm("f16", 10, 8, 4, torch.zeros(10, 4), torch.zeros(4, 9), torch.zeros(10, 8))
    with pytest.raises(ValueError, match="this rank owns"):
        D.sharded_sdpa(3, 16, 16, 8, *(torch.zeros(2, 16, 8) for _ in range(4)), scale=1.0)
    with pytest.raises(ValueError, match="this rank owns"):
        D.sharded_pointwise("add", 100, torch.zeros(99), torch.zeros(100), y=torch.zeros(100))


def _mailbox_model(world: int, calls: int, seed: int) -> int:
    """Random interleavings of the peer-sum exchange protocol (lc_sum_peer_f32).

    Each rank runs its calls in order (one stream).  A call with epoch e:
    store (value, e) into slot e & 1 of every rank's mailbox, one peer at a
    time (value first, then the flag, as the release store orders them), then
    wait until all flags of slot e & 1 in its own mailbox equal e and read the
    values.  Every read must return the value the writer produced for that
    same epoch; a write of epoch e+2 landing before a peer's read of epoch e
    would break it.  Returns the number of scheduler steps.
    """
    import random
    rnd = random.Random(seed)
    value = [[[None] * world for _ in range(2)] for _ in range(world)]  # box[p].partial[slot][writer]
    flag = [[[0] * world for _ in range(2)] for _ in range(world)]
    state = [{"call": 1, "phase": "write", "peer": 0, "sub": 0} for _ in range(world)]
    steps = 0
    while any(s["call"] <= calls for s in state):
        r = rnd.choice([i for i in range(world) if state[i]["call"] <= calls])
        s = state[r]
        e = s["call"]
        slot = e & 1
        steps += 1
        if s["phase"] == "write":
            p = s["peer"]
            if s["sub"] == 0:
                value[p][slot][r] = (r, e)
                s["sub"] = 1
            else:
                flag[p][slot][r] = e
                s["sub"] = 0
                s["peer"] += 1
                if s["peer"] == world:
                    s["phase"] = "wait"
        else:
            if all(flag[r][slot][q] == e for q in range(world)):
                for q in range(world):
                    assert value[r][slot][q] == (q, e), (r, q, e, value[r][slot][q])
                s.update(call=e + 1, phase="write", peer=0, sub=0)
    return steps


@pytest.mark.parametrize("world", [2, 3, 8])
def test_peer_exchange_protocol_under_random_interleavings(world):
    for seed in range(40):
        assert _mailbox_model(world, calls=12, seed=seed) > 0
