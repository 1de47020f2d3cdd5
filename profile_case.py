"""Runs one kernel of the library on a chosen size, for profiling and timing.

    python profile_case.py OP [--n N] [--rows R --cols C]
           [--m M --n N --k K] [--bh B --seq S] [--warmup W] [--repeat R]

OP is one of add, axpb, relumul, gelu_erf, gelu_tanh, sum, mean, rowsum,
rmsnorm, softmax, l2norm, gemm_f16, gemm_bf16, gemm_f32, attention_f32, sdpa,
general_paths (each golden package's fixed-class plan against the same
package run as a block program, natively compiled and interpreted; host call
included), or sum_graph (``--repeat`` back-to-back lc_sum_f32 launches on
``--n`` elements replayed from one CUDA graph over enough rotating copies of
the input that the others exceed twice the L2, as bench.py times the reduce
configuration; prints the mean time per launch).  Inputs are seeded device tensors; every launch goes through the
C ABI.  The mean CUDA-event time of the repeated launches is printed
(``--repeat`` launches after ``--warmup``), so the same command line serves
an ncu capture (``-k`` the kernel, ``-s`` the warm-up launches, ``-c`` one to
three launches).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from lazy_compiler_b200 import runtime  # noqa: E402

GENERAL_PACKAGES = ["r01_array_sum", "r04_row_sum", "f01_rmsnorm", "f02_row_softmax", "phase9_gelu_attention",
                    "a02_attention_128", "m02_matmul_rect", "m01_matmul_512"]


def sum_graph(n: int, repeat: int) -> None:
    """Per-launch time of lc_sum_f32 on n elements, launched back to back from one CUDA graph."""
    import torch
    copies = max(1, -(-2 * 126 * 10 ** 6 // (4 * n)) + 1) if 4 * n < 2 * 126 * 10 ** 6 else 1
    xs = [torch.rand(n, device="cuda") * 2 - 1 for _ in range(copies)]
    out = torch.empty(1, device="cuda")
    stream = torch.cuda.Stream()
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def launch(i):
        runtime.call("lc_sum_f32", P(xs[i % copies]), P(out), n,
                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    with torch.cuda.stream(stream):
        for i in range(3):
            launch(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(repeat):
            launch(i)
    times = []
    for _ in range(5):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record(stream)
            graph.replay()
            end.record(stream)
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end) / repeat)
    ms = sorted(times)[len(times) // 2]
    print(json.dumps({"op": "sum_graph", "n": n, "copies": copies, "us_per_launch": round(ms * 1e3, 3),
                      "GB/s": round(4 * n / (ms / 1e3) / 1e9, 1)}))


def general_paths(repeat: int) -> None:
    """Fixed-class plan vs the block program (native and interpreted) per golden package."""
    import torch

    from lazy_compiler_b200.blockprog import compile_blockprog
    from lazy_compiler_b200.compiler import compile_file
    from lazy_compiler_b200.ir import load_package
    from lazy_compiler_b200.runner import _torch_dtype, seeded_input

    golden = ROOT / "tests" / "golden" / "packages"
    stream = torch.cuda.current_stream().cuda_stream

    def time_plan(plan, ptrs, n):
        for _ in range(3):
            runtime.launch(plan, ptrs, stream)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(n):
            runtime.launch(plan, ptrs, stream)
        end.record()
        torch.cuda.synchronize()
        return start.elapsed_time(end) / n * 1000

    for name in GENERAL_PACKAGES:
        (ir,) = sorted((golden / name).glob("*.ir.json"))
        meta = json.loads((golden / name / "meta.json").read_text())
        bufs = {}
        for arg in meta["kernels"][0]["args"]:
            shape = tuple(arg.get("shape") or [1])
            if arg.get("output"):
                bufs[arg["name"]] = torch.zeros(shape, device="cuda", dtype=_torch_dtype(arg["dtype"]))
            else:
                bufs[arg["name"]] = torch.as_tensor(seeded_input(arg, 0)).to("cuda", _torch_dtype(arg["dtype"]))
        ptrs = {n: t.data_ptr() for n, t in bufs.items()}
        fixed = compile_file(ir)
        pkg = load_package(ir)
        native = compile_blockprog(pkg, pkg.body[0]).to_json()
        interpreted = json.loads(json.dumps(native))
        row = {"package": name, "fixed_op": fixed["op"], "fixed_us": round(time_plan(fixed, ptrs, repeat), 2)}
        row["block_native_us"] = round(time_plan(native, ptrs, repeat), 2)
        os.environ["LC_JIT"] = "0"
        row["block_interpreted_us"] = round(time_plan(interpreted, ptrs, max(3, repeat // 10)), 2)
        os.environ["LC_JIT"] = "1"
        print(json.dumps(row), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("op")
    ap.add_argument("--n", type=int, default=None)
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--cols", type=int, default=4096)
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--k", type=int, default=8192)
    ap.add_argument("--bh", type=int, default=128)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--epi", default="none", choices=["none", "gelu_erf", "gelu_tanh"],
                    help="fused epilogue of gemm_f16 / gemm_bf16")
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--repeat", type=int, default=1)
    a = ap.parse_args()

    import torch
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    op = a.op
    if op == "general_paths":
        general_paths(max(a.repeat, 10))
        return
    if op == "sum_graph":
        for n in ([a.n] if a.n else [1024, 1 << 20, 1 << 22, 1 << 23, 1 << 24, 1 << 25, 1 << 26, 1 << 28]):
            sum_graph(n, max(a.repeat, 20))
        return
    if op in ("add", "axpb", "relumul", "gelu_erf", "gelu_tanh", "sum", "mean"):
        n = a.n or (1 << 28 if op not in ("sum", "mean") else 1 << 24)
        x = torch.randn(n, device="cuda", generator=g)
        y = torch.randn(n, device="cuda", generator=g) if op in ("add", "relumul") else x
        out = torch.empty(n if op not in ("sum", "mean") else 1, device="cuda")
        c1, c2 = torch.tensor([1.5], device="cuda"), torch.tensor([float(n)], device="cuda")
        fn = {
            "add": lambda: runtime.call("lc_add_f32", P(x), P(y), P(out), n, s),
            "axpb": lambda: runtime.call("lc_axpb_f32", P(c1), P(c1), P(x), P(out), n, s),
            "relumul": lambda: runtime.call("lc_relumul_f32", P(x), P(y), P(out), n, s),
            "gelu_erf": lambda: runtime.call("lc_gelu", 0, 0, P(x), P(out), n, s),
            "gelu_tanh": lambda: runtime.call("lc_gelu", 0, 1, P(x), P(out), n, s),
            "sum": lambda: runtime.call("lc_sum_f32", P(x), P(out), n, s),
            "mean": lambda: runtime.call("lc_mean_f32", P(x), P(c2), P(out), n, s),
        }[op]
        work, unit = (3 if op in ("add", "relumul") else (1 if op in ("sum", "mean") else 2)) * 4 * n, "GB/s"
    elif op in ("rowsum", "rmsnorm", "softmax", "l2norm"):
        r, c = a.rows, a.cols
        x = torch.randn(r, c, device="cuda", generator=g)
        w = torch.randn(c, device="cuda", generator=g) * 0.1 + 1
        out = torch.empty_like(x)
        cnt, eps = torch.tensor([float(c)], device="cuda"), torch.tensor([1e-6], device="cuda")
        fn = {
            "rowsum": lambda: runtime.call("lc_rowsum_f32", P(x), P(out), r, c, s),
            "rmsnorm": lambda: runtime.call("lc_rmsnorm_f32", P(cnt), P(eps), P(x), P(w), P(out), r, c, s),
            "softmax": lambda: runtime.call("lc_softmax_f32", P(x), P(out), r, c, s),
            "l2norm": lambda: runtime.call("lc_l2norm_f32", P(x), P(out), r, c, s),
        }[op]
        work, unit = (1 if op == "rowsum" else 2) * 4 * r * c, "GB/s"
    elif op in ("gemm_f16", "gemm_bf16"):
        m, n, k = a.m, a.n or 8192, a.k
        dt = torch.float16 if op == "gemm_f16" else torch.bfloat16
        A = (torch.randn(m, k, device="cuda", generator=g) / k ** 0.5).to(dt)
        B = (torch.randn(k, n, device="cuda", generator=g) / k ** 0.5).to(dt)
        C = torch.empty(m, n, device="cuda")
        code = 1 if op == "gemm_f16" else 2
        epi = runtime.EPILOGUES[a.epi]
        fn = lambda: runtime.call("lc_gemm", code, 0, 0, epi, P(A), P(B), P(C), m, n, k, s)  # noqa: E731
        work, unit = 2 * m * n * k, "TFLOP/s"
    elif op == "gemm_f32":
        m, n, k = a.m, a.n or 8192, a.k
        A = torch.randn(m, k, device="cuda", generator=g)
        B = torch.randn(k, n, device="cuda", generator=g)
        C = torch.empty(m, n, device="cuda")
        fn = lambda: runtime.call("lc_gemm", 0, 0, 0, 0, P(A), P(B), P(C), m, n, k, s)  # noqa: E731
        work, unit = 2 * m * n * k, "TFLOP/s"
    elif op == "attention_f32":
        bh, sq, d = a.bh, a.seq, 128
        q = torch.randn(bh, sq, d, device="cuda", generator=g)
        kt = torch.randn(bh, d, sq, device="cuda", generator=g)
        v = torch.randn(bh, sq, d, device="cuda", generator=g)
        o = torch.empty_like(q)
        c = torch.tensor([d ** -0.5], device="cuda")
        fn = lambda: runtime.call("lc_attention_f32", 0, 0, P(c), P(q), P(kt), P(v), P(o),  # noqa: E731
                                  bh, sq, sq, d, d, s)
        work, unit = 4 * bh * sq * sq * d, "TFLOP/s"
    elif op == "sdpa":
        bh, sq, d = a.bh, a.seq, 128
        q = torch.randn(bh, sq, d, device="cuda", generator=g).half()
        k_ = torch.randn(bh, sq, d, device="cuda", generator=g).half()
        v = torch.randn(bh, sq, d, device="cuda", generator=g).half()
        o = torch.empty_like(q)
        scale = ctypes.c_float(d ** -0.5)
        fn = lambda: runtime.call("lc_sdpa_f16", P(q), P(k_), P(v), P(o), bh, sq, sq, d, scale, s)  # noqa: E731
        work, unit = 4 * bh * sq * sq * d, "TFLOP/s"
    else:
        raise SystemExit(f"unknown op {op}")
    for _ in range(a.warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(a.repeat):
        fn()
    end.record()
    torch.cuda.synchronize()
    runtime.call("lc_device_status", s)
    ms = start.elapsed_time(end) / a.repeat
    rate = work / (ms / 1e3) / (1e12 if unit == "TFLOP/s" else 1e9)
    print(json.dumps({"op": op, "ms": round(ms, 4), "rate": round(rate, 1), "unit": unit}))


if __name__ == "__main__":
    main()
