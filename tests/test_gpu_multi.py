"""Multi-GPU parity: every partitioned operation class over two GPUs equals the oracle.

One process per GPU on the first two GPUs (skipped with fewer than two).
Each rank holds only its shard of the same seeded problem
(``lazy_compiler_b200.dist``):

* sum / mean over contiguous ranges, with the shard sums exchanged by the
  fused peer-memory kernel (``PeerSum``: several calls in a row, then the
  same calls replayed from a CUDA graph) and by the NCCL all-reduce path;
  every rank must hold the float64 oracle's value within 1e-5, and both
  paths must agree bit for bit;
* pointwise add / relu*mul / GELU over element ranges (gathered, bit-exact
  for add and relu*mul, 1e-5 for GELU);
* row sum / RMSNorm / softmax / L2 norm over row blocks (gathered, 1e-5);
* f16 GEMM over row blocks of A with B replicated (gathered, 2e-2 and a
  normwise bound);
* f16 SDPA over (batch, head) ranges (gathered, 2e-2 and normwise 5e-3).

Uneven sizes make the two shards differ.  NVLS is off, the process group has
a short timeout, and each rank leaves only after its last collective.
"""
import math
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


def _close(got, ref, rtol, atol=0.0):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return bool(got.shape == ref.shape and np.isfinite(got).all() and np.isclose(got, ref, rtol=rtol, atol=atol).all())


def _close16(got, ref, norm_bound):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    rms = float(np.sqrt(np.mean(ref ** 2))) or 1.0
    norm = np.linalg.norm(got - ref) / (np.linalg.norm(ref) or 1.0)
    return bool(np.isfinite(got).all() and np.isclose(got, ref, rtol=2e-2, atol=2e-2 * rms).all()
                and norm < norm_bound)


def _worker(rank, world, port, results):
    import datetime

    import torch
    import torch.distributed as dist

    from lazy_compiler_b200 import dist as D
    from lazy_compiler_b200 import runtime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    out = {}
    cuda = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731

    # sum / mean: NCCL path and fused peer path
    n = (1 << 24) + 13
    x = O.uniform(n, seed=5)
    start, count = D.shard(n, world, rank)
    xs = cuda(x[start:start + count])
    total = torch.tensor([float(n)], device="cuda")
    nccl = torch.empty(2, device="cuda")
    D.sharded_sum(xs, count, nccl[:1])
    D.sharded_sum(xs, count, nccl[1:], total)
    peer = D.PeerSum.shared()
    calls = torch.full((6,), float("nan"), device="cuda")
    for i in range(6):
        peer(xs, count, calls[i:i + 1], total if i % 2 else None)
    graph_out = torch.full((4,), float("nan"), device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        peer(xs, count, graph_out[:1])  # warm the library's workspace of this stream
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        peer(xs, count, graph_out[:1])
        peer(xs, count, graph_out[1:2], total)
    dist.barrier()
    graph_out[:2].fill_(float("nan"))
    graph.replay()
    graph.replay()
    torch.cuda.synchronize()
    runtime.call("lc_device_status", None)
    want_sum, want_mean = float(O.sum_(x)[0]), float(O.mean(x)[0])
    c = calls.cpu().numpy()
    gsum, gmean = graph_out[:2].cpu().numpy()
    ns, nm = nccl.cpu().numpy()
    out["sum_nccl"] = _close(ns, want_sum, 1e-5) and _close(nm, want_mean, 1e-5)
    out["sum_peer"] = _close(c[0::2], [want_sum] * 3, 1e-5) and _close(c[1::2], [want_mean] * 3, 1e-5)
    out["sum_peer_graph"] = _close(gsum, want_sum, 1e-5) and _close(gmean, want_mean, 1e-5)
    out["sum_paths_agree"] = bool(c[0] == ns and c[1] == nm and gsum == ns and gmean == nm)
    del graph

    # pointwise over element ranges
    n = 1_000_003
    px, py = O.normal((n,), 11), O.normal((n,), 12)
    start, count = D.shard(n, world, rank)
    lx, ly = cuda(px[start:start + count]), cuda(py[start:start + count])
    lo = torch.empty(count, device="cuda")
    for op, want, tol in (("add", px + py, 0.0), ("relumul", np.maximum(px, 0) * py, 0.0),
                          ("gelu_erf", O.gelu(px, "none"), 1e-5), ("gelu_tanh", O.gelu(px, "tanh"), 1e-5)):
        D.sharded_pointwise(op, n, lx, lo, y=ly)
        got = D.gather(lo, n).cpu().numpy()
        out[f"pointwise_{op}"] = bool(np.array_equal(got, want)) if tol == 0 else _close(got, want, tol, 2e-6)

    # row blocks
    rows, cols = 1001, 4096
    X = O.normal((rows, cols), 3)
    w = O.normal((cols,), 4, mean=1.0, std=0.1)
    start, r = D.shard(rows, world, rank)
    lx = cuda(X[start:start + r])
    lw = cuda(w)
    cnt, eps = torch.tensor([float(cols)], device="cuda"), torch.tensor([1e-6], device="cuda")
    for op in ("rowsum", "rmsnorm", "softmax", "l2norm"):
        lo = torch.empty((r,) if op == "rowsum" else (r, cols), device="cuda")
        D.sharded_rows(op, rows, cols, lx, lo, w=lw, count=cnt, eps=eps)
        got = D.gather(lo, rows).cpu().numpy()
        want = {"rowsum": lambda: O.rowsum(X), "rmsnorm": lambda: O.rmsnorm(X, w, 1e-6),
                "softmax": lambda: O.softmax(X), "l2norm": lambda: O.l2norm(X)}[op]()[0]
        out[f"rows_{op}"] = _close(got, want, 1e-5, 1e-30)

    # GEMM: row blocks of A, B replicated
    m, nn, k = 515, 384, 256
    rng = np.random.default_rng(21)
    A = (rng.standard_normal((m, k)) / math.sqrt(k)).astype(np.float16)
    B = (rng.standard_normal((k, nn)) / math.sqrt(k)).astype(np.float16)
    start, r = D.shard(m, world, rank)
    lc = torch.empty(r, nn, device="cuda")
    D.sharded_gemm("f16", m, nn, k, cuda(A[start:start + r]), cuda(B), lc)
    got = D.gather(lc, m).cpu().numpy()
    out["gemm_f16"] = _close16(got, A.astype(np.float64) @ B.astype(np.float64), 1e-5)

    # SDPA: (batch, head) ranges
    bh, s, d = 5, 384, 128
    q, kk, v = (O.normal((bh, s, d), 30 + i).astype(np.float16) for i in range(3))
    start, r = D.shard(bh, world, rank)
    lo = torch.empty(r, s, d, device="cuda", dtype=torch.float16)
    D.sharded_sdpa(bh, s, s, d, cuda(q[start:start + r]), cuda(kk[start:start + r]), cuda(v[start:start + r]),
                   lo, 1 / math.sqrt(d))
    got = D.gather(lo, bh).float().cpu().numpy()
    want = O.sdpa_f16(q.astype(np.float32), kk.astype(np.float32), v.astype(np.float32), 1 / math.sqrt(d))[0]
    out["sdpa_f16"] = _close16(got, want, 5e-3)

    torch.cuda.synchronize()
    dist.barrier()
    results[rank] = out
    dist.destroy_process_group()


def test_partitioned_classes_two_gpus_match_oracle(cuda_device):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with mp.get_context("spawn").Manager() as manager:
        results = manager.dict()
        mp.spawn(_worker, args=(2, _port(), results), nprocs=2, join=True)
        got = dict(results)
    assert sorted(got) == [0, 1]
    for rank, checks in got.items():
        failed = [name for name, ok in checks.items() if not ok]
        assert not failed, (rank, failed)


def test_peer_sum_single_rank(cuda_device):
    """World of one: the fused exchange degenerates to the rank's own shard sum."""
    import torch

    from lazy_compiler_b200 import runtime
    from lazy_compiler_b200.dist import PeerSum
    n = (1 << 22) + 7
    x = O.uniform(n, seed=8)
    xs = torch.from_numpy(x).cuda()
    peer = PeerSum.shared()
    out = torch.full((3,), float("nan"), device="cuda")
    count = torch.tensor([float(n)], device="cuda")
    for i in range(3):
        peer(xs, n, out[i:i + 1], count if i == 1 else None)
    runtime.call("lc_device_status", None)
    got = out.cpu().numpy()
    assert _close(got[[0, 2]], [O.sum_(x)[0]] * 2, 1e-5)
    assert _close(got[1], O.mean(x)[0], 1e-5)


def test_peer_sum_reports_a_peer_that_never_arrives(cuda_device):
    """A declared second rank whose flags nothing sets: the bounded wait gives up.

    The second mailbox is plain local memory that no process writes, so the
    kernel's wait for rank 1's flag runs out (5 s); the result is NaN,
    lc_device_status reports LC_ERR_TIMEOUT, and after lc_peer_reset the
    context and the exchange work again.
    """
    import ctypes

    import torch

    from lazy_compiler_b200 import runtime
    from lazy_compiler_b200.dist import PeerSum
    n = 1 << 20
    xs = torch.ones(n, device="cuda")
    own = PeerSum.shared()
    silent = torch.zeros(64, dtype=torch.float32, device="cuda")  # 256 bytes, nobody's mailbox
    boxes = (ctypes.c_void_p * 2)(own._boxes[0], silent.data_ptr())
    out = torch.zeros(1, device="cuda")
    runtime.call("lc_sum_peer_f32", ctypes.c_void_p(xs.data_ptr()), n, ctypes.c_void_p(0),
                 ctypes.c_void_p(out.data_ptr()), boxes, 2, 0, None)
    with pytest.raises(runtime.LcError) as err:
        runtime.call("lc_device_status", None)
    assert err.value.status == -4
    assert math.isnan(float(out.item()))
    torch.cuda.synchronize()
    own.reset()
    torch.cuda.synchronize()
    again = torch.zeros(1, device="cuda")
    own(xs, n, again)
    runtime.call("lc_device_status", None)
    assert float(again.item()) == float(n)
