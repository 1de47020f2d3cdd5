"""Multi-GPU partitioning of the operation classes (one process per GPU).

The reference is single-GPU (one kernel per problem, submit.py:80-159).  Here
the work that shards naturally is partitioned across the ranks of a
``torch.distributed`` process group:

* whole-array sum / mean: contiguous ranges; each rank reduces its range to
  an f64 partial (``lc_sum_partial_f32``), the partials are all-reduced over
  NCCL (8 bytes), and ``lc_sum_finalize`` casts (sum) or divides by the global
  count (mean);
* row operations: blocks of rows; GEMM: blocks of rows of A with B replicated;
  attention: ranges of (batch, head).  None of these needs a collective.
"""
from __future__ import annotations

import ctypes

from . import runtime


def shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced range ``(start, count)`` of ``n`` items for ``rank``."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def sharded_sum(x, n_local: int, out, count=None, group=None, stream=None) -> None:
    """Sum (or mean when ``count`` is a one-element device tensor) over all ranks.

    ``x`` is this rank's shard (a CUDA tensor), ``out`` a one-element f32
    CUDA tensor that receives the global result on every rank.
    """
    import torch
    import torch.distributed as dist

    partial = torch.zeros(1, dtype=torch.float64, device=x.device)
    s = ctypes.c_void_p(stream if stream is not None else torch.cuda.current_stream(x.device).cuda_stream)
    runtime.call("lc_sum_partial_f32", ctypes.c_void_p(x.data_ptr()), n_local,
                 ctypes.c_void_p(partial.data_ptr()), s)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(partial, group=group)
    runtime.call("lc_sum_finalize", ctypes.c_void_p(partial.data_ptr()),
                 ctypes.c_void_p(count.data_ptr()) if count is not None else ctypes.c_void_p(0),
                 ctypes.c_void_p(out.data_ptr()), s)
