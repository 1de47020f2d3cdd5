#!/usr/bin/env python3
"""Benchmark of the B200 operator backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

Configurations (BASELINE.json ``configs``):

* ``elementwise`` (default, the headline): 2^28 fp32 N(0,1) elements per
  GPU; one step = add, scale-shift (a=1.5, b=-0.25), relu*mul, erf-GELU and
  tanh-GELU, each one HBM pass.  Metric: HBM GB/s of algorithmic bytes.
* ``reduce``: whole-array sum and mean of 2^24 fp32 U[-1,1] per GPU; across
  GPUs the f64 partials are all-reduced over NCCL.  L2 is flushed between steps.
* ``rows``: RMSNorm (eps 1e-6, w ~ N(1, 0.1)), softmax, L2 norm and row sums
  of X[16384, 4096] fp32 per GPU.

Multi-GPU runs are weak scaling: every rank processes its own full-size
shard; ``value`` is the whole-job aggregate over the max-over-ranks device
time.  ``--impl reference`` times the reference's CPU implementation of the
path (its numpy formula oracle, restated in C over POSIX threads in
``oracle/c``) on the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "HBM GB/s (elementwise/reduce/norm) & dense TFLOPS (GEMM/attn), 1–8 B200"
FALLBACK_HBM_GBS = 6650.0
N_ELEMENTWISE = 1 << 28
N_REDUCE = 1 << 24
ROWS, COLS = 16384, 4096
L2_FLUSH_BYTES = 512 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=["elementwise", "reduce", "rows", "gemm_f16", "gemm_bf16", "sdpa"],
                    default="elementwise")
    ap.add_argument("--no-suite", action="store_true", help="skip the secondary configurations")
    ap.add_argument("--no-e2e", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    return args


# ---------------------------------------------------------------- environment

FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["bf16_tflops"]), float(data.get("bf16_tflops_sustained", 0)) or None, "measured"
    return FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


SUITE = ("reduce", "rows", "elementwise", "gemm_f16", "gemm_bf16", "sdpa")
SDPA_SHAPE = (8 * 16, 4096, 128)
GEMM_SHAPES = {"gemm_f16": ("f16", 8192, 8192, 8192), "gemm_bf16": ("bf16", 4096, 16384, 2048)}


def traffic_table():
    path = ROOT / "profiles" / "traffic.json"
    return json.loads(path.read_text()) if path.exists() else {}


class Dist:
    def __init__(self, gpus: int):
        import torch
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = False
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = True
        self.device = torch.device("cuda", self.local)

    def barrier(self):
        import torch
        if self.pg:
            import torch.distributed as dist
            dist.barrier(device_ids=[self.local])
        torch.cuda.synchronize(self.device)

    def max(self, value: float) -> float:
        if not self.pg:
            return value
        import torch
        import torch.distributed as dist
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist
            dist.destroy_process_group()


class Clocks:
    """SM clock and throttle reasons sampled during the timed region.

    Polls NVML (read-only queries) every millisecond from a background thread,
    so even a 20 ms timed region yields tens of samples; falls back to
    ``nvidia-smi -lms 100`` when NVML is unavailable.
    """

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        import torch
        self.samples = []
        self.max_mhz = None
        self.stop = False
        self.thread = None
        self.proc = None
        try:
            self.uuid = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
        except Exception:
            self.uuid = None
        self.index = device.index or 0

    def _poll(self, nvml, handle):
        get_reasons = getattr(nvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nvml.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop:
            try:
                self.samples.append((nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM),
                                     int(get_reasons(handle))))
            except Exception:
                pass
            time.sleep(0.001)

    def __enter__(self):
        import threading
        try:
            import pynvml as nvml
            nvml.nvmlInit()
            handle = (nvml.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid
                      else nvml.nvmlDeviceGetHandleByIndex(self.index))
            self.max_mhz = nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM)
            self.thread = threading.Thread(target=self._poll, args=(nvml, handle), daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", "-i", self.uuid or str(self.index),
                     "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                     "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                     "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                    stdout=self.file, stderr=subprocess.DEVNULL)
            except OSError:
                self.proc = None
        time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        self.stop = True
        if self.thread is not None:
            self.thread.join(timeout=2)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.file.flush()
            self.file.seek(0)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            bits = [0x8, 0x40, 0x20, 0x4]
            for line in self.file.read().splitlines():
                parts = [x.strip() for x in line.split(",")]
                try:
                    mask = sum(b for b, f in zip(bits, parts[2:6]) if f.lower().startswith("active"))
                    self.samples.append((float(parts[0]), mask))
                    self.max_mhz = float(parts[1])
                except (ValueError, IndexError):
                    continue
            os.unlink(self.file.name)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"], "samples": 0}
        reasons = sorted({name for _, mask in self.samples for bit, name in self.REASONS.items() if mask & bit})
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "sm_mhz_min": min(c for c, _ in self.samples), "reasons": reasons,
                "samples": len(self.samples), "source": "nvml" if self.proc is None else "nvidia-smi"}


# ---------------------------------------------------------------- our kernels

def P(t):
    return ctypes.c_void_p(t.data_ptr())


def elementwise_ops(n, tensors, stream):
    from lazy_compiler_b200 import runtime
    x, y, a, b, out = tensors
    s = ctypes.c_void_p(stream)
    return [
        ("add", 3 * 4 * n, lambda: runtime.call("lc_add_f32", P(x), P(y), P(out), n, s)),
        ("axpb", 2 * 4 * n, lambda: runtime.call("lc_axpb_f32", P(a), P(b), P(x), P(out), n, s)),
        ("relumul", 3 * 4 * n, lambda: runtime.call("lc_relumul_f32", P(x), P(y), P(out), n, s)),
        ("gelu_erf", 2 * 4 * n, lambda: runtime.call("lc_gelu", 0, 0, P(x), P(out), n, s)),
        ("gelu_tanh", 2 * 4 * n, lambda: runtime.call("lc_gelu", 0, 1, P(x), P(out), n, s)),
    ]


def timed_steps(dist, ops, steps, warmup, flush=None):
    """Runs warmup + timed steps; per-op CUDA-event durations over the timed region.

    Returns (max-over-ranks seconds of the timed region, per-op mean ms, launches).
    With ``flush`` (an L2-clearing callable run between steps) the region time
    is the sum of the op durations, so the flush itself is not counted.
    """
    import torch
    for _ in range(warmup):
        if flush:
            flush()
        for _, _, fn in ops:
            fn()
    dist.barrier()
    per_op = {name: [] for name, _, _ in ops}
    marks = []
    region_start = torch.cuda.Event(enable_timing=True)
    region_end = torch.cuda.Event(enable_timing=True)
    region_start.record()
    for _ in range(steps):
        if flush:
            flush()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(ops) + 1)]
        evs[0].record()
        for i, (_, _, fn) in enumerate(ops):
            fn()
            evs[i + 1].record()
        marks.append(evs)
    region_end.record()
    torch.cuda.synchronize()
    for evs in marks:
        for i, (name, _, _) in enumerate(ops):
            per_op[name].append(evs[i].elapsed_time(evs[i + 1]))
    if flush:
        local = sum(sum(v) for v in per_op.values()) / 1e3
    else:
        local = region_start.elapsed_time(region_end) / 1e3
    dist.barrier()
    return dist.max(local), {k: statistics.mean(v) for k, v in per_op.items()}, steps * len(ops)


def roofline(ops, per_op_ms, peak, peak_kind, traffic):
    name, nbytes, _ = max(ops, key=lambda o: per_op_ms[o[0]])
    if name.startswith("gemm") or name.startswith("sdpa"):
        tpeak, sustained, kind = tensor_peak()
        achieved = nbytes / (per_op_ms[name] / 1e3) / 1e12
        return {"bound": "tensor", "kernel": name, "achieved": round(achieved, 1), "peak": tpeak,
                "peak_kind": f"bf16_tflops burst of {kind}", "unit": "TFLOP/s",
                "frac": round(achieved / tpeak, 4),
                "frac_of_sustained": round(achieved / sustained, 4) if sustained else None,
                "traffic": traffic.get(name), "algorithmic_flops": nbytes}
    achieved = nbytes / (per_op_ms[name] / 1e3) / 1e9
    return {"bound": "hbm", "kernel": name, "achieved": round(achieved, 1), "peak": peak,
            "peak_kind": f"hbm_gbs of {peak_kind}", "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": traffic.get(name), "algorithmic_bytes": nbytes}


def run_ours(args):
    import torch
    from lazy_compiler_b200 import runtime
    runtime.library()
    dist = Dist(args.gpus)
    torch.cuda.set_device(dist.device)
    peak, peak_kind = peaks()
    traffic = traffic_table()
    stream = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=dist.device).manual_seed(1234 + dist.rank)
    result = {}

    def measure(config):
        if config == "elementwise":
            n = N_ELEMENTWISE
            x = torch.randn(n, device=dist.device, generator=g)
            y = torch.randn(n, device=dist.device, generator=g)
            a = torch.tensor([1.5], device=dist.device)
            b = torch.tensor([-0.25], device=dist.device)
            out = torch.empty_like(x)
            ops = elementwise_ops(n, (x, y, a, b, out), stream)
            cfg = {"workload": "elementwise set: add, scale-shift(a=1.5,b=-0.25), relu*mul, "
                               "erf-GELU, tanh-GELU over 2^28 fp32 N(0,1) per GPU",
                   "elements_per_gpu": n, "l2": "inputs larger than L2 (1 GiB per array)"}
            return ops, cfg, None, ((x, y), out)
        if config == "reduce":
            n = N_REDUCE
            x = torch.rand(n, device=dist.device, generator=g) * 2 - 1
            count = torch.tensor([float(n * dist.world)], device=dist.device)
            out = torch.empty(2, device=dist.device)
            part = torch.zeros(1, dtype=torch.float64, device=dist.device)
            s = ctypes.c_void_p(stream)
            if dist.world == 1:
                ops = [("sum", 4 * n, lambda: runtime.call("lc_sum_f32", P(x), P(out), n, s)),
                       ("mean", 4 * n, lambda: runtime.call("lc_mean_f32", P(x), P(count), P(out[1:]), n, s))]
            else:
                from lazy_compiler_b200.dist import sharded_sum
                ops = [("sum", 4 * n, lambda: sharded_sum(x, n, out[:1], None, stream=stream)),
                       ("mean", 4 * n, lambda: sharded_sum(x, n, out[1:], count, stream=stream))]
            scratch = torch.empty(L2_FLUSH_BYTES // 4, device=dist.device)
            clean = torch.zeros(L2_FLUSH_BYTES // 8, device=dist.device)
            sink = torch.empty(1, device=dist.device)

            def flush():
                # write more than L2 holds, then read an unrelated buffer larger than
                # L2 so the lines the timed reduction evicts are clean (no
                # write-back of the flush's dirty lines inside the timed kernels)
                scratch.zero_()
                torch.sum(clean, dim=0, keepdim=True, out=sink)
            cfg = {"workload": "whole-array sum and mean of 2^24 fp32 U[-1,1] per GPU"
                               + (", f64 partials all-reduced over NCCL" if dist.world > 1 else ""),
                   "elements_per_gpu": n,
                   "l2": "flushed between steps (512 MiB write, then a 256 MiB read; not timed)"}
            return ops, cfg, flush, ((x,), out, part, count, scratch, clean, sink)
        if config == "rows":
            x = torch.randn(ROWS, COLS, device=dist.device, generator=g)
            w = torch.randn(COLS, device=dist.device, generator=g) * 0.1 + 1.0
            out = torch.empty_like(x)
            rs = torch.empty(ROWS, device=dist.device)
            count = torch.tensor([float(COLS)], device=dist.device)
            eps = torch.tensor([1e-6], device=dist.device)
            s = ctypes.c_void_p(stream)
            xb = 4 * ROWS * COLS
            ops = [("rmsnorm", 2 * xb + 4 * COLS, lambda: runtime.call(
                        "lc_rmsnorm_f32", P(count), P(eps), P(x), P(w), P(out), ROWS, COLS, s)),
                   ("softmax", 2 * xb, lambda: runtime.call("lc_softmax_f32", P(x), P(out), ROWS, COLS, s)),
                   ("l2norm", 2 * xb, lambda: runtime.call("lc_l2norm_f32", P(x), P(out), ROWS, COLS, s)),
                   ("rowsum", xb + 4 * ROWS, lambda: runtime.call("lc_rowsum_f32", P(x), P(rs), ROWS, COLS, s))]
            cfg = {"workload": "RMSNorm, softmax, L2 norm, row sums of X[16384,4096] fp32 per GPU",
                   "rows": ROWS, "cols": COLS, "l2": "inputs larger than L2 (256 MiB)"}
            return ops, cfg, None, ((x, w), out, rs, count, eps)
        if config in GEMM_SHAPES:
            ab, m, n, k = GEMM_SHAPES[config]
            dt = torch.float16 if ab == "f16" else torch.bfloat16
            a = (torch.randn(m, k, device=dist.device, generator=g) / k ** 0.5).to(dt)
            b = (torch.randn(k, n, device=dist.device, generator=g) / k ** 0.5).to(dt)
            c = torch.empty(m, n, device=dist.device)
            s = ctypes.c_void_p(stream)
            code = 1 if ab == "f16" else 2
            flops = 2 * m * n * k
            ops = [(f"gemm_{ab}", flops, lambda: runtime.call("lc_gemm", code, 0, 0, 0, P(a), P(b), P(c), m, n, k, s))]
            cfg = {"workload": f"{ab} GEMM M{m} N{n} K{k}, B row-major [K,N], f32 out, A,B ~ N(0,1/sqrt(K))",
                   "m": m, "n": n, "k": k, "l2": f"inputs larger than L2 ({(m * k + k * n) * 2 >> 20} MiB)"}
            return ops, cfg, None, ((a, b), c)
        if config == "sdpa":
            bh, sq, d = SDPA_SHAPE
            q = torch.randn(bh, sq, d, device=dist.device, generator=g).half()
            k = torch.randn(bh, sq, d, device=dist.device, generator=g).half()
            v = torch.randn(bh, sq, d, device=dist.device, generator=g).half()
            o = torch.empty_like(q)
            s = ctypes.c_void_p(stream)
            flops = 4 * bh * sq * sq * d
            scale = ctypes.c_float(d ** -0.5)
            ops = [("sdpa_f16", flops, lambda: runtime.call("lc_sdpa_f16", P(q), P(k), P(v), P(o), bh, sq, sq, d, scale, s))]
            cfg = {"workload": "SDPA f16 B8 H16 S4096 D128, scale 1/sqrt(D), non-causal, f32 softmax statistics",
                   "batch_heads": bh, "seq": sq, "head_dim": d,
                   "l2": f"inputs larger than L2 ({3 * bh * sq * d * 2 >> 20} MiB)"}
            return ops, cfg, None, ((q, k, v), o)
        raise ValueError(config)

    def one(config, steps, warmup, with_clocks):
        ops, cfg, flush, keep = measure(config)
        clocks = None
        if with_clocks:
            with Clocks(dist.device) as c:
                seconds, per_op, launches = timed_steps(dist, ops, steps, warmup, flush)
            clocks = c.summary()
        else:
            seconds, per_op, launches = timed_steps(dist, ops, steps, warmup, flush)
        total = sum(o[1] for o in ops) * steps * dist.world
        tensor = config in GEMM_SHAPES or config == "sdpa"
        scale = 1e12 if tensor else 1e9
        return {"ops": ops, "cfg": cfg, "seconds": seconds, "per_op": per_op, "launches": launches,
                "value": total / seconds / scale, "unit": "TFLOP/s" if tensor else "GB/s",
                "clocks": clocks, "keep": keep}

    main = one(args.config, args.steps, args.warmup, True)
    line = {
        "metric": METRIC, "value": round(main["value"], 1), "unit": main["unit"], "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(main["seconds"] * 1e3 / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {"gemm_f16": "f16", "gemm_bf16": "bf16", "sdpa": "f16"}.get(args.config, "f32"),
        "data": "synthetic (seeded torch generator on device, N(0,1) / U[-1,1] as configured)",
        "config": {**main["cfg"], "parallelism": f"range shards x{dist.world}" if dist.world > 1 else "1 GPU"},
        "roofline": roofline(main["ops"], main["per_op"], peak, peak_kind, traffic),
        "kernels_ms": {k: round(v, 4) for k, v in main["per_op"].items()},
        "clocks": main["clocks"], "gpu_launches": main["launches"],
    }
    if not args.no_e2e:
        line["e2e"] = e2e(args, dist, main)
    del main
    torch.cuda.empty_cache()
    if not args.no_suite:
        suite = {}
        for config in SUITE:
            if config == args.config:
                continue
            r = one(config, max(5, min(args.steps, 20)), args.warmup, False)
            suite[config] = {"value": round(r["value"], 1), "unit": r["unit"],
                             "kernels_ms": {k: round(v, 4) for k, v in r["per_op"].items()},
                             "roofline": roofline(r["ops"], r["per_op"], peak, peak_kind, traffic),
                             "config": r["cfg"]}
            del r
            torch.cuda.empty_cache()
        line["suite"] = suite
    if dist.rank == 0 and dist.world == 1:
        line["cpu_baseline"] = cpu_baseline(args.config, sample_scale=16)
    if dist.rank == 0:
        emit(line)
    dist.close()


def e2e(args, dist, main):
    """Same metric through the C ABI with pinned host buffers; copies inside the timed region."""
    import torch
    ops = main["ops"]
    inputs, output = main["keep"][0], main["keep"][1]
    host_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in inputs]
    for h, t in zip(host_in, inputs):
        h.copy_(t)
    host_out = torch.empty(output.shape, dtype=output.dtype, pin_memory=True)
    steps = max(1, min(args.steps, 3))

    def step():
        for h, t in zip(host_in, inputs):
            t.copy_(h, non_blocking=True)
        for _, _, fn in ops:
            fn()
            host_out.copy_(output, non_blocking=True)

    step()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    seconds = dist.max(start.elapsed_time(end) / 1e3)
    work = sum(o[1] for o in ops) * steps * dist.world
    h2d = sum(h.numel() * h.element_size() for h in host_in)
    d2h = host_out.numel() * host_out.element_size() * len(ops)
    scale = 1e12 if main["unit"] == "TFLOP/s" else 1e9
    return {"value": round(work / seconds / scale, 3), "unit": main["unit"], "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps,
            "path": "ctypes C-ABI calls (lc_*) with pinned host inputs copied in and every result copied out"}


# ---------------------------------------------------------------- CPU reference / baseline

def oracle_lib():
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    lib = ctypes.CDLL(str(ROOT / "oracle" / "_build" / "liboracle.so"))
    lib.oc_sum.restype = ctypes.c_double
    return lib


def cpu_run(config, sample_scale):
    """One bounded CPU sample of the configuration.

    Returns (ops [(work, fn)], description, threads, unit, keep-alive arrays).
    """
    import numpy as np
    rng = np.random.default_rng(0)
    if config == "sdpa":
        bh, sq, d = SDPA_SHAPE
        rows = max(1, sq // sample_scale)
        q = rng.standard_normal((rows, d)).astype(np.float16).astype(np.float64)
        k = rng.standard_normal((sq, d)).astype(np.float16).astype(np.float64)
        v = rng.standard_normal((sq, d)).astype(np.float16).astype(np.float64)
        scale = d ** -0.5

        def attn():
            sc = (q @ k.T) * scale
            sc -= sc.max(-1, keepdims=True)
            p = np.exp(sc)
            p /= p.sum(-1, keepdims=True)
            return p @ v
        threads = blas_threads()
        desc = (f"{rows} query rows of one head against 4096 keys (1/{bh * sample_scale} of a step), "
                f"float64 numpy/BLAS softmax attention, {threads} threads")
        return [(4 * rows * sq * d, attn)], desc, threads, "TFLOP/s", (q, k, v)
    if config in GEMM_SHAPES:
        ab, m, n, k = GEMM_SHAPES[config]
        rows = max(1, m // sample_scale)
        a = (rng.standard_normal((rows, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
        a64, b64 = a.astype(np.float64), b.astype(np.float64)
        ops = [(2 * rows * n * k, lambda: a64 @ b64)]
        threads = blas_threads()
        desc = (f"{rows} of {m} rows of the {ab} GEMM (1/{sample_scale} of a step) in float64 "
                f"numpy/BLAS, {threads} threads")
        return ops, desc, threads, "TFLOP/s", (a64, b64)
    lib = oracle_lib()
    threads = lib.oc_threads()
    i64 = ctypes.c_int64
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if config == "elementwise":
        n = N_ELEMENTWISE // sample_scale
        x = rng.standard_normal(n, dtype=np.float32)
        y = rng.standard_normal(n, dtype=np.float32)
        out = np.empty_like(x)
        ops = [(3 * 4 * n, lambda: lib.oc_add(ptr(x), ptr(y), ptr(out), i64(n))),
               (2 * 4 * n, lambda: lib.oc_axpb(ctypes.c_float(1.5), ctypes.c_float(-0.25), ptr(x), ptr(out), i64(n))),
               (3 * 4 * n, lambda: lib.oc_relumul(ptr(x), ptr(y), ptr(out), i64(n))),
               (2 * 4 * n, lambda: lib.oc_gelu(0, ptr(x), ptr(out), i64(n))),
               (2 * 4 * n, lambda: lib.oc_gelu(1, ptr(x), ptr(out), i64(n)))]
        desc = f"5 elementwise ops over 2^{(n).bit_length() - 1} fp32 elements each (1/{sample_scale} of a step)"
        keep = (x, y, out)
    elif config == "reduce":
        n = N_REDUCE
        x = rng.uniform(-1, 1, n).astype(np.float32)
        ops = [(4 * n, lambda: lib.oc_sum(ptr(x), i64(n))), (4 * n, lambda: lib.oc_sum(ptr(x), i64(n)))]
        desc = "sum and mean of 2^24 fp32 (a full step)"
        keep = (x,)
    else:
        r = ROWS // sample_scale
        x = rng.standard_normal((r, COLS), dtype=np.float32)
        w = (rng.standard_normal(COLS) * 0.1 + 1).astype(np.float32)
        out = np.empty_like(x)
        rs = np.empty(r, np.float32)
        xb = 4 * r * COLS
        ops = [(2 * xb, lambda: lib.oc_rmsnorm(ptr(x), ptr(w), ptr(out), i64(r), i64(COLS),
                                               ctypes.c_double(1e-6), ctypes.c_double(COLS))),
               (2 * xb, lambda: lib.oc_softmax(ptr(x), ptr(out), i64(r), i64(COLS))),
               (2 * xb, lambda: lib.oc_l2norm(ptr(x), ptr(out), i64(r), i64(COLS))),
               (xb, lambda: lib.oc_rowsum(ptr(x), ptr(rs), i64(r), i64(COLS)))]
        desc = f"4 row ops over {r} x {COLS} fp32 rows (1/{sample_scale} of a step)"
        keep = (x, w, out, rs)
    return ops, desc, threads, "GB/s", keep


def blas_threads():
    try:
        from threadpoolctl import threadpool_info
        counts = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if counts:
            return max(counts)
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_time(ops, repeats):
    best = []
    for _ in range(repeats):
        t0 = time.perf_counter()
        for _, fn in ops:
            fn()
        best.append(time.perf_counter() - t0)
    return best


def cpu_baseline(config, sample_scale):
    if config in GEMM_SHAPES:
        sample_scale = 64
    if config == "sdpa":
        sample_scale = 8
    ops, desc, threads, unit, keep = cpu_run(config, sample_scale)
    cpu_time(ops, 1)
    times = cpu_time(ops, 3)
    work = sum(o[0] for o in ops)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    how = ("the reference's float64 numpy oracle" if config in GEMM_SHAPES or config == "sdpa" else
           f"C restatement of the reference's numpy formula oracle, {threads} POSIX threads")
    return {"value": round(work / statistics.median(times) / scale, 4), "unit": unit,
            "cores": threads, "kind": "port",
            "sample": desc + f"; {how}, median of 3 after 1 warm-up"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    scale = {"elementwise": 16, "reduce": 1, "rows": 4, "sdpa": 8}.get(args.config, 64)
    ops, desc, threads, unit, keep = cpu_run(args.config, scale)
    cpu_time(ops, args.warmup)
    times = cpu_time(ops, args.steps)
    work = sum(o[0] for o in ops)
    value = work * args.steps / sum(times) / (1e12 if unit == "TFLOP/s" else 1e9)
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(times) * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "data": "synthetic (seeded numpy)",
        "dtype": {"gemm_f16": "f64 (f16 inputs)", "gemm_bf16": "f64 (bf16 inputs)",
                  "sdpa": "f64 (f16 inputs)"}.get(args.config, "f32"),
        "config": {"workload": args.config, "sample": desc},
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


_RESULT_FD = None


def emit(line: dict) -> None:
    """Writes the one JSON result line to the real stdout."""
    data = (json.dumps(line) + "\n").encode()
    if _RESULT_FD is not None:
        os.write(_RESULT_FD, data)
    else:
        sys.stdout.write(data.decode())
        sys.stdout.flush()


def main():
    global _RESULT_FD
    args = parse_args()
    # Libraries (NCCL, torch) may print to fd 1; keep stdout for the result line only.
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
