"""Multi-GPU partitioning of the operation classes (one process per GPU).

The reference is single-GPU (one kernel per problem, submit.py:80-159).  Here
each operation class is partitioned across the ranks of a ``torch.distributed``
process group (NCCL), every rank holding only its own shard:

* whole-array sum / mean: contiguous element ranges.  Each rank reduces its
  range to an f64 shard sum; the shard sums are exchanged either inside the
  reduction kernel over NVLink peer memory (:class:`PeerSum`, the default:
  one kernel, no collective call) or by an NCCL all-reduce of the 8-byte
  partials followed by a finalising kernel (:func:`sharded_sum`).  Both give
  the same value on every rank;
* pointwise operations: contiguous element ranges (:func:`sharded_pointwise`);
* row operations (row sum, RMSNorm, softmax, L2 norm): blocks of whole rows
  (:func:`sharded_rows`);
* GEMM: blocks of rows of A and C, B replicated (:func:`sharded_gemm`);
* attention: ranges of (batch, head) pairs (:func:`sharded_sdpa`).

Only the sum / mean has an exchange step; every other partition is
independent and its output stays sharded (:func:`gather` collects the shards
where a caller needs the whole result).  Each helper takes the full logical
problem size and this rank's local tensors, checks that their shapes are
exactly this rank's shard, and launches the library's kernel on it.
"""
from __future__ import annotations

import ctypes

from . import runtime

P = ctypes.c_void_p


def shard(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous balanced range ``(start, count)`` of ``n`` items for ``rank``."""
    if world < 1 or not 0 <= rank < world or n < 0:
        raise ValueError(f"bad shard request n={n} world={world} rank={rank}")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def _world_rank(group=None) -> tuple[int, int]:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0


def _stream(stream, device) -> P:
    import torch
    return P(stream if stream is not None else torch.cuda.current_stream(device).cuda_stream)


def _expect(t, shape: tuple, what: str) -> None:
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{what}: local shard has shape {tuple(t.shape)}, this rank owns {tuple(shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{what}: local shard must be contiguous")


def sharded_sum(x, n_local: int, out, count=None, group=None, stream=None) -> None:
    """Sum (or mean when ``count`` is a one-element device tensor) over all ranks, via NCCL.

    ``x`` is this rank's shard (a CUDA tensor), ``out`` a one-element f32
    CUDA tensor that receives the global result on every rank.
    """
    import torch
    import torch.distributed as dist

    partial = torch.zeros(1, dtype=torch.float64, device=x.device)
    s = _stream(stream, x.device)
    runtime.call("lc_sum_partial_f32", P(x.data_ptr()), n_local, P(partial.data_ptr()), s)
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(partial, group=group)
    runtime.call("lc_sum_finalize", P(partial.data_ptr()),
                 P(count.data_ptr()) if count is not None else P(0), P(out.data_ptr()), s)


class PeerSum:
    """Range-sharded sum / mean with the shard-sum exchange fused into the kernel.

    Construction is collective: every rank creates its mailbox
    (``lc_peer_mailbox``), the CUDA IPC handles are all-gathered over the
    process group, and each rank maps its peers' mailboxes
    (``lc_peer_open``).  A call then launches one kernel
    (``lc_sum_peer_f32``) that reduces the local shard and exchanges the
    f64 shard sums with plain NVLink stores and flag waits.  All ranks must
    make the same sequence of calls (each call is one exchange epoch,
    counted on the device, so the call may be captured in a CUDA graph).
    A process maps each peer's mailbox once: use :meth:`shared` for the
    object of the current device and group.
    """

    _instances: dict = {}

    @classmethod
    def shared(cls, group=None) -> "PeerSum":
        """The process's PeerSum for the current device and ``group`` (created collectively once)."""
        import torch
        key = (torch.cuda.current_device(), id(group))
        if key not in cls._instances:
            cls._instances[key] = cls(group)
        return cls._instances[key]

    def __init__(self, group=None):
        import torch
        import torch.distributed as dist

        self.world, self.rank = _world_rank(group)
        if self.world > 8:
            raise ValueError("PeerSum supports at most 8 ranks (one node)")
        box = P()
        handle = ctypes.create_string_buffer(64)
        runtime.call("lc_peer_mailbox", ctypes.byref(box), handle)
        handles = [handle.raw]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        pointers = []
        for r, raw in enumerate(handles):
            if r == self.rank:
                pointers.append(box.value)
                continue
            peer = P()
            runtime.call("lc_peer_open", ctypes.create_string_buffer(raw, 64), ctypes.byref(peer))
            self._opened.append(peer.value)
            pointers.append(peer.value)
        self._boxes = (P * self.world)(*pointers)
        self._group = group
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=group)

    def __call__(self, x, n_local: int, out, count=None, stream=None) -> None:
        """``out[0]`` = sum of every rank's shard (or that sum / ``count[0]``)."""
        runtime.call("lc_sum_peer_f32", P(x.data_ptr()), n_local,
                     P(count.data_ptr()) if count is not None else P(0), P(out.data_ptr()),
                     self._boxes, self.world, self.rank, _stream(stream, x.device))

    def reset(self, stream=None) -> None:
        """Zero this rank's mailbox; call on every rank between barriers, nothing in flight."""
        import torch
        runtime.call("lc_peer_reset", _stream(stream, torch.cuda.current_device()))

    def close(self) -> None:
        """Unmap the peers' mailboxes (collective use of this object ends here)."""
        for ptr in self._opened:
            runtime.call("lc_peer_close", P(ptr))
        self._opened = []
        for key, obj in list(PeerSum._instances.items()):
            if obj is self:
                del PeerSum._instances[key]


POINTWISE = {"add": "lc_add_f32", "relumul": "lc_relumul_f32"}


def sharded_pointwise(op: str, n: int, x, out, y=None, a=None, b=None, group=None, stream=None) -> None:
    """One pointwise operation on this rank's contiguous range of ``n`` elements.

    ``op`` is ``add`` / ``relumul`` (x, y), ``axpb`` (a, b one-element
    tensors) or ``gelu_erf`` / ``gelu_tanh`` (f32).
    """
    world, rank = _world_rank(group)
    _, count = shard(n, world, rank)
    for t, name in ((x, "x"), (out, "out")) + (((y, "y"),) if y is not None else ()):
        _expect(t, (count,), f"sharded_pointwise {name}")
    s = _stream(stream, x.device)
    if op in POINTWISE:
        runtime.call(POINTWISE[op], P(x.data_ptr()), P(y.data_ptr()), P(out.data_ptr()), count, s)
    elif op == "axpb":
        runtime.call("lc_axpb_f32", P(a.data_ptr()), P(b.data_ptr()), P(x.data_ptr()), P(out.data_ptr()),
                     count, s)
    elif op in ("gelu_erf", "gelu_tanh"):
        runtime.call("lc_gelu", 0, 0 if op == "gelu_erf" else 1, P(x.data_ptr()), P(out.data_ptr()), count, s)
    else:
        raise ValueError(f"unknown pointwise op {op!r}")


def sharded_rows(op: str, rows: int, cols: int, x, out, w=None, count=None, eps=None, group=None,
                 stream=None) -> None:
    """One row operation on this rank's block of whole rows of ``X[rows, cols]``.

    ``op``: ``rowsum`` (out has this rank's rows), ``rmsnorm`` (w[cols],
    one-element count and eps), ``softmax`` or ``l2norm``.
    """
    world, rank = _world_rank(group)
    _, r = shard(rows, world, rank)
    _expect(x, (r, cols), f"sharded_rows({op}) x")
    _expect(out, (r,) if op == "rowsum" else (r, cols), f"sharded_rows({op}) out")
    s = _stream(stream, x.device)
    if op == "rowsum":
        runtime.call("lc_rowsum_f32", P(x.data_ptr()), P(out.data_ptr()), r, cols, s)
    elif op == "rmsnorm":
        runtime.call("lc_rmsnorm_f32", P(count.data_ptr()), P(eps.data_ptr()), P(x.data_ptr()),
                     P(w.data_ptr()), P(out.data_ptr()), r, cols, s)
    elif op == "softmax":
        runtime.call("lc_softmax_f32", P(x.data_ptr()), P(out.data_ptr()), r, cols, s)
    elif op == "l2norm":
        runtime.call("lc_l2norm_f32", P(x.data_ptr()), P(out.data_ptr()), r, cols, s)
    else:
        raise ValueError(f"unknown row op {op!r}")


GEMM_TYPES = {"f16": runtime.LC_F16, "bf16": runtime.LC_BF16, "f32": runtime.LC_F32}


def sharded_gemm(ab: str, m: int, n: int, k: int, a, b, c, epilogue: str = "none", group=None,
                 stream=None) -> None:
    """C[rows] = epilogue(A[rows] @ B) for this rank's block of rows of an (m, n, k) GEMM.

    ``a`` is this rank's [rows, k] block of A, ``b`` the whole [k, n] B
    (replicated on every rank), ``c`` this rank's [rows, n] f32 block of C.
    """
    world, rank = _world_rank(group)
    _, rows = shard(m, world, rank)
    _expect(a, (rows, k), "sharded_gemm a")
    _expect(b, (k, n), "sharded_gemm b")
    _expect(c, (rows, n), "sharded_gemm c")
    if rows == 0:
        return
    runtime.call("lc_gemm", GEMM_TYPES[ab], runtime.LC_F32, runtime.B_LAYOUTS["kn"], runtime.EPILOGUES[epilogue],
                 P(a.data_ptr()), P(b.data_ptr()), P(c.data_ptr()), rows, n, k, _stream(stream, a.device))


def sharded_sdpa(batch_heads: int, s_q: int, s_kv: int, d: int, q, k, v, o, scale: float, group=None,
                 stream=None) -> None:
    """Non-causal f16 attention for this rank's range of (batch, head) pairs.

    ``q``, ``o`` are [bh, s_q, d] and ``k``, ``v`` [bh, s_kv, d] for this
    rank's ``bh`` pairs; the softmax statistics are f32.
    """
    world, rank = _world_rank(group)
    _, bh = shard(batch_heads, world, rank)
    _expect(q, (bh, s_q, d), "sharded_sdpa q")
    _expect(k, (bh, s_kv, d), "sharded_sdpa k")
    _expect(v, (bh, s_kv, d), "sharded_sdpa v")
    _expect(o, (bh, s_q, d), "sharded_sdpa o")
    if bh == 0:
        return
    runtime.call("lc_sdpa_f16", P(q.data_ptr()), P(k.data_ptr()), P(v.data_ptr()), P(o.data_ptr()), bh, s_q,
                 s_kv, d, ctypes.c_float(scale), _stream(stream, q.device))


def gather(local, total: int, group=None):
    """All-gather row / element shards along dim 0 into the whole tensor (every rank)."""
    import torch
    import torch.distributed as dist

    world, _ = _world_rank(group)
    if world == 1:
        return local
    counts = [shard(total, world, r)[1] for r in range(world)]
    width = max(counts)
    padded = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[:local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
