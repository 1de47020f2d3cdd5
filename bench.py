#!/usr/bin/env python3
"""Benchmark of the B200 operator backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

Configurations (BASELINE.json ``configs``):

* ``elementwise`` (default, the headline): 2^28 fp32 N(0,1) elements; one
  step = add, scale-shift (a=1.5, b=-0.25), relu*mul, erf-GELU and tanh-GELU,
  each one HBM pass.  Metric: HBM GB/s of algorithmic bytes.
* ``reduce``: whole-array sum and mean of 2^24 fp32 U[-1,1].
* ``rows``: RMSNorm (eps 1e-6, w ~ N(1, 0.1)), softmax, L2 norm and row sums
  of X[16384, 4096] fp32.
* ``gemm_f16`` (8192^3), ``gemm_f16_gelu`` (the same with the optional fused
  erf-GELU epilogue), ``gemm_bf16`` (M4096 N16384 K2048): f32 out.
* ``sdpa``: f16 B8 H16 S4096 D128, non-causal.

Timing: the K timed steps are captured in one CUDA graph and replayed between
two CUDA events on the launching stream (W eager warm-up steps first), so the
inter-kernel gaps are the device's, not the host launch path's.  Every
operation's inputs rotate over enough copies that the set a launch does not
read is larger than twice the L2 (a launch never finds its inputs in L2).
Per-operation times for the roofline come from a second graph per operation
(K launches of that operation alone, or as many more as make the graph run
2 ms, so that the replay's start cost is not charged to a 15 µs kernel).

Multi-GPU (one process per GPU, torchrun): strong scaling.  The fixed
BASELINE configuration is partitioned across the ranks (element ranges for
pointwise and sum/mean, row blocks for the row operations, M blocks of A and
C with B replicated for GEMM, (batch, head) ranges for SDPA);
``value`` = the whole configuration's work / the max-over-ranks device time.
The sum and mean exchange their f64 shard sums inside the kernel over NVLink
peer memory (``lazy_compiler_b200.dist.PeerSum``); an NCCL all-reduce of the
same partials is timed beside it.  The weak-scaled figure (every rank a
full-size problem) is reported under ``weak``.

``--impl reference`` times the reference's CPU implementation of the path
(its numpy formula oracle, restated in C over POSIX threads in ``oracle/c``,
and the numpy formulas themselves) on the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
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
FALLBACK_BF16_TFLOPS = 1590.0
N_ELEMENTWISE = 1 << 28
N_REDUCE = 1 << 24
ROWS, COLS = 16384, 4096
L2_BYTES = 126 * 10 ** 6
# a per-operation timing graph runs at least this long (more launches when K are shorter)
PER_OP_GRAPH_S = 2e-3
SUITE = ("reduce", "rows", "elementwise", "gemm_f16", "gemm_f16_gelu", "gemm_bf16", "sdpa")
SDPA_SHAPE = (8 * 16, 4096, 128)
GEMM_SHAPES = {"gemm_f16": ("f16", 8192, 8192, 8192), "gemm_f16_gelu": ("f16", 8192, 8192, 8192),
               "gemm_bf16": ("bf16", 4096, 16384, 2048)}
# the configuration's optional fused epilogue, measured as its own suite entry
GEMM_EPILOGUE = {"gemm_f16_gelu": "gelu_erf"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=list(SUITE), default="elementwise")
    ap.add_argument("--no-suite", action="store_true", help="skip the secondary configurations")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-ref-ptx", action="store_true", help="skip the reference-PTX baseline leg")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    return args


# ---------------------------------------------------------------- environment

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

    Polls NVML (read-only queries) every millisecond from a background thread;
    falls back to ``nvidia-smi -lms 100`` when NVML is unavailable.
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


# ---------------------------------------------------------------- workloads

def P(t):
    return ctypes.c_void_p(t.data_ptr())


def S():
    """The current stream, read at call time (the capture stream inside a graph)."""
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def rotation(slot_bytes: int) -> int:
    """Copies of a launch's inputs so that the other copies exceed twice the L2."""
    return max(1, math.ceil(2 * L2_BYTES / max(1, slot_bytes)) + (1 if slot_bytes < 2 * L2_BYTES else 0))


class Op:
    """One library call of a step: ``fn(slot_inputs)`` launches it on the current stream."""

    def __init__(self, name, work, fn, kernels=1):
        self.name, self.work, self.fn, self.kernels = name, work, fn, kernels


class Workload:
    def __init__(self, config, unit, ops, slots, full_work, cfg, keep, e2e_io, dtype):
        self.config, self.unit, self.ops, self.slots = config, unit, ops, slots
        self.full_work, self.cfg, self.keep, self.e2e_io, self.dtype = full_work, cfg, keep, e2e_io, dtype

    @property
    def tensor(self):
        return self.unit == "TFLOP/s"

    def launch(self, i: int, j: int) -> None:
        """Operation j of step i, on the inputs of its rotation slot."""
        n_ops = len(self.ops)
        self.ops[j].fn(self.slots[(i * n_ops + j) % len(self.slots)])


def build(config: str, dist, strong: bool, g):
    """The workload of one configuration: this rank's shard (strong) or a full copy (weak)."""
    import torch
    from lazy_compiler_b200 import runtime
    from lazy_compiler_b200.dist import PeerSum, shard
    dev = dist.device
    world, rank = dist.world, dist.rank
    part = (lambda n: shard(n, world, rank)[1]) if strong else (lambda n: n)
    label = f" ({'this rank' if strong and world > 1 else 'per GPU'})"
    if config == "elementwise":
        n = part(N_ELEMENTWISE)
        r = rotation(8 * n)
        slots = [(torch.randn(n, device=dev, generator=g), torch.randn(n, device=dev, generator=g)) for _ in range(r)]
        a, b = torch.tensor([1.5], device=dev), torch.tensor([-0.25], device=dev)
        outs = [torch.empty(n, device=dev) for _ in range(5)]
        ops = [
            Op("add", 12 * n, lambda s: runtime.call("lc_add_f32", P(s[0]), P(s[1]), P(outs[0]), n, S())),
            Op("axpb", 8 * n, lambda s: runtime.call("lc_axpb_f32", P(a), P(b), P(s[0]), P(outs[1]), n, S())),
            Op("relumul", 12 * n, lambda s: runtime.call("lc_relumul_f32", P(s[0]), P(s[1]), P(outs[2]), n, S())),
            Op("gelu_erf", 8 * n, lambda s: runtime.call("lc_gelu", 0, 0, P(s[0]), P(outs[3]), n, S())),
            Op("gelu_tanh", 8 * n, lambda s: runtime.call("lc_gelu", 0, 1, P(s[0]), P(outs[4]), n, S())),
        ]
        full = 48 * N_ELEMENTWISE
        cfg = {"workload": "elementwise set: add, scale-shift(a=1.5,b=-0.25), relu*mul, erf-GELU, tanh-GELU "
                           "over 2^28 fp32 N(0,1)", "elements": N_ELEMENTWISE, "elements_local": n}
        return Workload(config, "GB/s", ops, slots, full, cfg, (a, b), (slots[0], outs), "f32")
    if config == "reduce":
        n = part(N_REDUCE)
        r = rotation(4 * n)
        slots = [(torch.rand(n, device=dev, generator=g) * 2 - 1,) for _ in range(r)]
        count = torch.tensor([float(N_REDUCE if strong else n * world)], device=dev)
        outs = [torch.empty(1, device=dev) for _ in range(2)]
        if world == 1:
            ops = [Op("sum", 4 * n, lambda s: runtime.call("lc_sum_f32", P(s[0]), P(outs[0]), n, S())),
                   Op("mean", 4 * n, lambda s: runtime.call("lc_mean_f32", P(s[0]), P(count), P(outs[1]), n, S()))]
            keep = (count,)
        else:
            peer = PeerSum.shared()
            ops = [Op("sum", 4 * n, lambda s: peer(s[0], n, outs[0])),
                   Op("mean", 4 * n, lambda s: peer(s[0], n, outs[1], count))]
            keep = (count, peer)
        full = 8 * N_REDUCE
        cfg = {"workload": "whole-array sum and mean of 2^24 fp32 U[-1,1]"
                           + (", f64 shard sums exchanged inside the kernel over NVLink peer memory"
                              if world > 1 else ""), "elements": N_REDUCE, "elements_local": n}
        return Workload(config, "GB/s", ops, slots, full, cfg, keep, (slots[0], outs), "f32")
    if config == "rows":
        rows = part(ROWS)
        r = rotation(4 * rows * COLS)
        slots = [(torch.randn(rows, COLS, device=dev, generator=g),) for _ in range(r)]
        w = torch.randn(COLS, device=dev, generator=g) * 0.1 + 1.0
        count, eps = torch.tensor([float(COLS)], device=dev), torch.tensor([1e-6], device=dev)
        outs = [torch.empty(rows, COLS, device=dev) for _ in range(3)] + [torch.empty(rows, device=dev)]
        xb = 4 * rows * COLS
        ops = [Op("rmsnorm", 2 * xb + 4 * COLS, lambda s: runtime.call(
                   "lc_rmsnorm_f32", P(count), P(eps), P(s[0]), P(w), P(outs[0]), rows, COLS, S())),
               Op("softmax", 2 * xb, lambda s: runtime.call("lc_softmax_f32", P(s[0]), P(outs[1]), rows, COLS, S())),
               Op("l2norm", 2 * xb, lambda s: runtime.call("lc_l2norm_f32", P(s[0]), P(outs[2]), rows, COLS, S())),
               Op("rowsum", xb + 4 * rows, lambda s: runtime.call("lc_rowsum_f32", P(s[0]), P(outs[3]), rows, COLS,
                                                                  S()))]
        fb = 4 * ROWS * COLS
        full = (2 * fb + 4 * COLS) + 2 * fb + 2 * fb + (fb + 4 * ROWS)
        cfg = {"workload": "RMSNorm, softmax, L2 norm, row sums of X[16384,4096] fp32", "rows": ROWS, "cols": COLS,
               "rows_local": rows}
        return Workload(config, "GB/s", ops, slots, full, cfg, (w, count, eps), (slots[0], outs), "f32")
    if config in GEMM_SHAPES:
        ab, m, n, k = GEMM_SHAPES[config]
        rows = part(m)
        dt = torch.float16 if ab == "f16" else torch.bfloat16
        r = rotation(2 * (rows * k + k * n))
        slots = [((torch.randn(rows, k, device=dev, generator=g) / k ** 0.5).to(dt),
                  (torch.randn(k, n, device=dev, generator=g) / k ** 0.5).to(dt)) for _ in range(r)]
        c = torch.empty(rows, n, device=dev)
        code = 1 if ab == "f16" else 2
        epi = GEMM_EPILOGUE.get(config, "none")
        epi_code = runtime.EPILOGUES[epi]
        name = f"gemm_{ab}" + ("" if epi == "none" else f"_{epi}")
        ops = [Op(name, 2 * rows * n * k,
                  lambda s: runtime.call("lc_gemm", code, 0, 0, epi_code, P(s[0]), P(s[1]), P(c), rows, n, k,
                                         S()))]
        cfg = {"workload": f"{ab} GEMM M{m} N{n} K{k}, B row-major [K,N], f32 out, A,B ~ N(0,1/sqrt(K))"
                           + ("" if epi == "none" else ", fused erf-GELU epilogue")
                           + (", M split in row blocks, B replicated" if strong and world > 1 else ""),
               "m": m, "n": n, "k": k, "m_local": rows}
        return Workload(config, "TFLOP/s", ops, slots, 2 * m * n * k, cfg, (), (slots[0], [c]), ab)
    if config == "sdpa":
        bh_all, sq, d = SDPA_SHAPE
        bh = part(bh_all)
        r = rotation(3 * 2 * bh * sq * d)
        slots = [tuple(torch.randn(bh, sq, d, device=dev, generator=g).half() for _ in range(3)) for _ in range(r)]
        o = torch.empty(bh, sq, d, device=dev, dtype=torch.float16)
        scale = ctypes.c_float(d ** -0.5)
        ops = [Op("sdpa_f16", 4 * bh * sq * sq * d, lambda s: runtime.call(
            "lc_sdpa_f16", P(s[0]), P(s[1]), P(s[2]), P(o), bh, sq, sq, d, scale, S()))]
        cfg = {"workload": "SDPA f16 B8 H16 S4096 D128, scale 1/sqrt(D), non-causal, f32 softmax statistics"
                           + (", (batch, head) pairs split across ranks" if strong and world > 1 else ""),
               "batch_heads": bh_all, "seq": sq, "head_dim": d, "batch_heads_local": bh}
        return Workload(config, "TFLOP/s", ops, slots, 4 * bh_all * sq * sq * d, cfg, (), (slots[0], [o]), "f16")
    raise ValueError(config)


def graph_time(dist, wl: Workload, steps: int, warmup: int, clocks: bool = False):
    """Max-over-ranks device seconds of K steps replayed from one CUDA graph, and per-op means (ms)."""
    import torch
    stream = torch.cuda.Stream(dist.device)
    n_ops = len(wl.ops)
    with torch.cuda.stream(stream):
        for i in range(warmup):
            for j in range(n_ops):
                wl.launch(i, j)
    torch.cuda.synchronize(dist.device)
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph, stream=stream):
        for i in range(steps):
            for j in range(n_ops):
                wl.launch(i, j)
    op_graphs = []
    for j in range(n_ops):
        gj = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gj, stream=stream):
            for i in range(steps):
                wl.launch(i, j)
        op_graphs.append(gj)

    token = torch.zeros(1, device=dist.device)

    def replay(graph):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            if dist.pg:
                # device-side rendezvous on the timing stream: every GPU starts the
                # timed region when the all-reduce completes, not when its host got here
                import torch.distributed as tdist
                tdist.all_reduce(token)
            start.record(stream)
            graph.replay()
            end.record(stream)
        torch.cuda.synchronize(dist.device)
        return start.elapsed_time(end) / 1e3

    # one untimed replay of each graph (upload), identical on every rank
    replay(step_graph)
    reps = []
    for j, gj in enumerate(op_graphs):
        # A replay pays a few microseconds before its first kernel starts; a
        # per-operation graph shorter than PER_OP_GRAPH_S is re-captured with
        # more launches (the same rotation of inputs) so that this start cost
        # does not enter the per-launch duration.  Every rank takes the same count.
        t = dist.max(replay(gj))
        r = steps
        if t < PER_OP_GRAPH_S:
            r = min(steps * 64, math.ceil(steps * PER_OP_GRAPH_S / max(t, 1e-7)))
            longer = torch.cuda.CUDAGraph()
            with torch.cuda.graph(longer, stream=stream):
                for i in range(r):
                    wl.launch(i, j)
            op_graphs[j] = longer
            replay(longer)
        reps.append(r)
    dist.barrier()
    clock_summary = None
    if clocks:
        with Clocks(dist.device) as c:
            local = replay(step_graph)
        clock_summary = c.summary()
    else:
        local = replay(step_graph)
    seconds = dist.max(local)
    per_op = {}
    for op, gj, r in zip(wl.ops, op_graphs, reps):
        dist.barrier()
        per_op[op.name] = dist.max(replay(gj)) * 1e3 / r
    dist.barrier()
    del step_graph, op_graphs
    launches = steps * sum(op.kernels for op in wl.ops)
    return seconds, per_op, launches, clock_summary


def roofline(wl: Workload, per_op_ms, peak, peak_kind, traffic):
    op = max(wl.ops, key=lambda o: per_op_ms[o.name])
    if wl.tensor:
        tpeak, sustained, kind = tensor_peak()
        achieved = op.work / (per_op_ms[op.name] / 1e3) / 1e12
        return {"bound": "tensor", "kernel": op.name, "achieved": round(achieved, 1), "peak": tpeak,
                "peak_kind": f"bf16_tflops burst of {kind}", "unit": "TFLOP/s",
                "frac": round(achieved / tpeak, 4),
                "frac_of_sustained": round(achieved / sustained, 4) if sustained else None,
                "traffic": traffic.get(op.name), "algorithmic_flops": op.work}
    achieved = op.work / (per_op_ms[op.name] / 1e3) / 1e9
    return {"bound": "hbm", "kernel": op.name, "achieved": round(achieved, 1), "peak": peak,
            "peak_kind": f"hbm_gbs of {peak_kind}", "unit": "GB/s", "frac": round(achieved / peak, 4),
            "traffic": traffic.get(op.name), "algorithmic_bytes": op.work}


def measure(config, dist, strong, steps, warmup, clocks, g):
    import torch
    wl = build(config, dist, strong, g)
    seconds, per_op, launches, clock_summary = graph_time(dist, wl, steps, warmup, clocks)
    scale = 1e12 if wl.tensor else 1e9
    total = wl.full_work * steps if strong else sum(o.work for o in wl.ops) * steps * dist.world
    slot_bytes = sum(t.numel() * t.element_size() for t in wl.slots[0])
    result = {"wl": wl, "seconds": seconds, "per_op": per_op, "launches": launches, "clocks": clock_summary,
              "value": total / seconds / scale, "rotation": len(wl.slots), "slot_bytes": slot_bytes}
    torch.cuda.synchronize(dist.device)
    return result


def collective_compare(dist, g, steps):
    """Sum of this rank's 2^24/N shard: fused peer exchange vs NCCL all-reduce of the partials (eager)."""
    import torch
    from lazy_compiler_b200.dist import PeerSum, shard, sharded_sum
    n = shard(N_REDUCE, dist.world, dist.rank)[1]
    x = torch.rand(n, device=dist.device, generator=g) * 2 - 1
    out = torch.empty(2, device=dist.device)
    peer = PeerSum.shared()
    variants = {"peer_kernel": lambda: peer(x, n, out[:1]), "nccl_allreduce": lambda: sharded_sum(x, n, out[1:])}
    res = {}
    for name, fn in variants.items():
        for _ in range(3):
            fn()
        dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        res[f"{name}_us"] = round(dist.max(start.elapsed_time(end) / steps) * 1e3, 2)
    dist.barrier()
    got = out.cpu().tolist()
    res["agree"] = got[0] == got[1]
    res["note"] = "eager launches (host launch path included), this rank's 2^24/N shard, max over ranks"
    return res


def run_ours(args):
    import torch
    from lazy_compiler_b200 import runtime
    runtime.library()
    dist = Dist(args.gpus)
    torch.cuda.set_device(dist.device)
    peak, peak_kind = peaks()
    traffic = traffic_table()
    g = torch.Generator(device=dist.device).manual_seed(1234 + dist.rank)
    strong = dist.world > 1

    main = measure(args.config, dist, strong, args.steps, args.warmup, True, g)
    wl = main["wl"]
    line = {
        "metric": METRIC, "value": round(main["value"], 1), "unit": wl.unit, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(main["seconds"] * 1e3 / args.steps, 4),
        "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic (seeded torch generator on device, N(0,1) / U[-1,1] as configured)",
        "config": {**wl.cfg,
                   "parallelism": (f"{dist.world} ranks, " + {"elementwise": "element ranges", "reduce": "element ranges",
                                   "rows": "row blocks", "sdpa": "(batch, head) ranges"}.get(
                                       args.config, "M row blocks, B replicated")) if strong else "1 GPU",
                   "l2": (f"inputs rotate over {main['rotation']} copies of {main['slot_bytes'] >> 20} MiB "
                          f"(the copies a launch does not read exceed twice the 126 MB L2)"
                          if main["rotation"] > 1 else
                          f"inputs larger than L2 ({main['slot_bytes'] >> 20} MiB per step, 126 MB L2)"),
                   "timing": "K steps captured in one CUDA graph, CUDA events around the replay"},
        "roofline": roofline(wl, main["per_op"], peak, peak_kind, traffic),
        "kernels_ms": {k: round(v, 4) for k, v in main["per_op"].items()},
        "clocks": main["clocks"], "gpu_launches": main["launches"],
    }
    if not args.no_e2e:
        line["e2e"] = e2e(args, dist, wl, strong)
    del main, wl
    torch.cuda.empty_cache()
    if strong:
        weak = measure(args.config, dist, False, args.steps, args.warmup, False, g)
        line["weak"] = {"value": round(weak["value"], 1), "unit": weak["wl"].unit,
                        "ms_per_step": round(weak["seconds"] * 1e3 / args.steps, 4),
                        "note": "every rank a full-size configuration (aggregate over ranks)"}
        del weak
        torch.cuda.empty_cache()
        if args.config == "reduce" or not args.no_suite:
            line["collective"] = collective_compare(dist, g, max(args.steps, 20))
    if not args.no_suite:
        suite = {}
        for config in SUITE:
            if config == args.config:
                continue
            r = measure(config, dist, strong, max(5, min(args.steps, 20)), args.warmup, True, g)
            suite[config] = {"value": round(r["value"], 1), "unit": r["wl"].unit,
                             "kernels_ms": {k: round(v, 4) for k, v in r["per_op"].items()},
                             "roofline": roofline(r["wl"], r["per_op"], peak, peak_kind, traffic),
                             "config": r["wl"].cfg, "clocks": r["clocks"]}
            del r
            torch.cuda.empty_cache()
        line["suite"] = suite
    if dist.rank == 0 and dist.world == 1:
        if not args.no_ref_ptx:
            line["ref_ptx"] = ref_ptx_baseline(args.config, line["kernels_ms"])
            if "suite" in line:
                for config, row in line["suite"].items():
                    row["ref_ptx"] = ref_ptx_baseline(config, row["kernels_ms"])
        line["cpu_baseline"] = cpu_baseline(args.config, sample_scale=16)
    if dist.rank == 0:
        emit(line)
    dist.close()


def e2e(args, dist, wl: Workload, strong: bool):
    """The same step through the C ABI with pinned host buffers, copies inside the timed region.

    Three streams overlap the two PCIe directions with the kernels: step i's
    inputs are copied into one of two device input sets while step i-1
    computes, and each operation's result is copied out while the next
    operation runs.
    """
    import torch
    inputs, outs = wl.e2e_io
    host_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in inputs]
    for h, t in zip(host_in, inputs):
        h.copy_(t)
    dev_in = [inputs, tuple(torch.empty_like(t) for t in inputs)]
    host_out = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
    op_out = list(range(len(wl.ops))) if len(outs) == len(wl.ops) else [0] * len(wl.ops)
    s_in, s_run, s_out = (torch.cuda.Stream(dist.device) for _ in range(3))
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready, in_free = [ev(), ev()], [ev(), ev()]
    out_ready, out_free = [ev() for _ in outs], [ev() for _ in outs]
    for e in in_free + out_free:
        e.record(s_run)
    steps = max(10, args.steps)

    def step(i):
        b = i % 2
        s_in.wait_event(in_free[b])
        with torch.cuda.stream(s_in):
            for h, t in zip(host_in, dev_in[b]):
                t.copy_(h, non_blocking=True)
        in_ready[b].record(s_in)
        s_run.wait_event(in_ready[b])
        for j, op in enumerate(wl.ops):
            k = op_out[j]
            s_run.wait_event(out_free[k])
            with torch.cuda.stream(s_run):
                op.fn(dev_in[b])
            out_ready[k].record(s_run)
            s_out.wait_event(out_ready[k])
            with torch.cuda.stream(s_out):
                host_out[k].copy_(outs[k], non_blocking=True)
            out_free[k].record(s_out)
        in_free[b].record(s_run)

    step(0)
    step(1)
    torch.cuda.synchronize(dist.device)
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s_in)
    s_run.wait_stream(s_in)
    s_out.wait_stream(s_in)
    for i in range(steps):
        step(i)
    s_in.wait_stream(s_run)
    s_in.wait_stream(s_out)
    end.record(s_in)
    torch.cuda.synchronize(dist.device)
    seconds = dist.max(start.elapsed_time(end) / 1e3)
    work = (wl.full_work if strong else sum(o.work for o in wl.ops) * dist.world) * steps
    h2d = sum(h.numel() * h.element_size() for h in host_in)
    d2h = sum(host_out[op_out[j]].numel() * host_out[op_out[j]].element_size() for j in range(len(wl.ops)))
    scale = 1e12 if wl.tensor else 1e9
    return {"value": round(work / seconds / scale, 3), "unit": wl.unit, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps,
            "path": "ctypes C-ABI calls (lc_*) with pinned host inputs copied in and every result copied out; "
                    "H2D, kernels and D2H on three streams (double-buffered inputs)"}


# ---------------------------------------------------------------- the reference's own PTX on this B200

REF_PTX = {
    "elementwise": [("add", "p01_vector_add", 12 << 28), ("axpb", "p02_scale_shift", 8 << 28),
                    ("relumul", "p03_relu_mul", 12 << 28), ("gelu_erf", "phase9_gelu_erf_tail", 8 << 28),
                    ("gelu_tanh", "phase9_gelu_tanh_matrix", 8 << 28)],
    "reduce": [("sum", "r02_big_sum", 4 << 24), ("mean", "r03_mean", 4 << 24)],
    "rows": [("rmsnorm", "f01_rmsnorm", 8 * ROWS * COLS + 4 * COLS), ("softmax", "f02_row_softmax", 8 * ROWS * COLS),
             ("l2norm", "f03_l2norm", 8 * ROWS * COLS), ("rowsum", "r04_row_sum", 4 * ROWS * COLS + 4 * ROWS)],
    # the reference's mma.sync GEMM (tanh-GELU epilogue, f16 out) rescaled to 8192^3; ours is timed
    # on the same buffers through the plan of the same rescaled package (same epilogue and output)
    "gemm_f16": [("gemm_f16 (tanh-GELU, f16 out)", "phase9_half_gelu_gemm", 2 * 8192 ** 3)],
    # the reference's scalar attention (a02 schedule, f16 loads, D = 128, 4096 keys) on a slice of
    # 512 query rows of one head; its rate stands for the whole configuration (linear in rows, heads)
    "sdpa": [("sdpa_f16", "a02_attention_f16_slice", 4 * 512 * 4096 * 128)],
}


REF_PTX_REPEATS = 10


def ref_ptx_baseline(config, ours_ms):
    """The reference compiler's own PTX for the configuration (rescaled public packages), timed here.

    Baseline leg: the PTX that the reference's unchanged compiler emitted
    (``oracle/_ref``, built in the development container) is JIT-loaded and
    launched under its meta.json geometry on this B200, on seeded device
    inputs: after at least 0.3 s of warm-up launches, the median of
    REF_PTX_REPEATS launches each between its own CUDA events.
    """
    if config not in REF_PTX:
        return {"unavailable": f"no rescaled reference package for the {config} configuration"}
    try:
        import torch

        from oracle.ref_launch import RefKernel, manifest_rescaled
        rows = manifest_rescaled()
        ops, total_bytes, total_ms = {}, 0, 0.0
        for op, name, nbytes in REF_PTX[config]:
            if name not in rows:
                return {"unavailable": f"oracle/_ref has no rescaled PTX for {name}"}
            kernel = RefKernel(name, rescaled=True)
            g = torch.Generator(device="cuda").manual_seed(7)
            inputs = {}
            for arg in kernel.kernel_meta["args"]:
                if arg.get("output") or "data" in arg:
                    continue
                shape = tuple(arg["shape"])
                if config == "reduce":
                    inputs[arg["name"]] = torch.rand(shape, device="cuda", generator=g) * 2 - 1
                elif arg["name"] == "w":
                    inputs[arg["name"]] = torch.randn(shape, device="cuda", generator=g) * 0.1 + 1
                else:
                    inputs[arg["name"]] = torch.randn(shape, device="cuda", generator=g)
            _, buffers = kernel.run(inputs, keep=True)
            ptrs = {n: t.data_ptr() for n, t in buffers.items()}
            stream = torch.cuda.current_stream().cuda_stream
            tensor = config in GEMM_SHAPES or config == "sdpa"
            # warm the GPU (clocks ramp down while idle): launch for at least 0.3 s first
            t0 = time.perf_counter()
            while time.perf_counter() - t0 < 0.3:
                kernel.launch(ptrs, stream)
                torch.cuda.synchronize()
            times = []
            for _ in range(REF_PTX_REPEATS):
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                kernel.launch(ptrs, stream)
                end.record()
                torch.cuda.synchronize()
                times.append(start.elapsed_time(end))
            ms = statistics.median(times)
            if config == "sdpa":
                # ours: the configuration's own kernel, compared per flop
                bh, sq, d = SDPA_SHAPE
                ours_ms = {op: ours_ms[op] * nbytes / (4 * bh * sq * sq * d)} if op in ours_ms else {}
            elif tensor:
                # ours on the same buffers: the plan this backend makes of the same rescaled package
                from lazy_compiler_b200.compiler import compile_file
                from lazy_compiler_b200.runtime import launch
                from oracle.ref_launch import REF
                (ir,) = sorted((REF.parent.parent / rows[name]["package"]).glob("*.ir.json"))
                plan = compile_file(ir)
                for _ in range(3):
                    launch(plan, ptrs, stream)
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                for _ in range(REF_PTX_REPEATS):
                    launch(plan, ptrs, stream)
                end.record()
                torch.cuda.synchronize()
                ours_ms = {op: start.elapsed_time(end) / REF_PTX_REPEATS}
            rate = {"TFLOP/s": sig(nbytes / ms / 1e9)} if tensor else {"GB/s": sig(nbytes / ms / 1e6)}
            ops[op] = {"package": f"{name} (rescaled)", "ms": sig(ms), **rate,
                       "ours_ms": sig(ours_ms.get(op, float("nan"))),
                       "speedup": round(ms / ours_ms[op], 2) if op in ours_ms else None,
                       "grid": kernel.kernel_meta["grid"], "block": kernel.kernel_meta["block"]}
            total_bytes += nbytes
            total_ms += ms
            del buffers, inputs
        torch.cuda.empty_cache()
        tensor = config in GEMM_SHAPES or config == "sdpa"
        note = ("; sdpa: a slice of 512 query rows of one head, its rate extrapolated to the whole "
                "configuration, ours_ms scaled to the slice's flops" if config == "sdpa" else "")
        return {"kind": "the reference compiler's own PTX (public IR packages rescaled to the configuration "
                        "size, its meta.json geometry) on this B200" + note,
                "value": sig(total_bytes / total_ms / (1e9 if tensor else 1e6)),
                "unit": "TFLOP/s" if tensor else "GB/s", "ops": ops}
    except Exception as exc:  # the leg is a baseline: report, never fail the bench
        return {"unavailable": f"{type(exc).__name__}: {exc}"}


def sig(x, digits=4):
    """x to `digits` significant figures (the baselines span six decades)."""
    return float(f"{x:.{digits}g}")


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
        if GEMM_EPILOGUE.get(config) == "gelu_erf":
            from scipy.special import erf

            def gemm_gelu():
                y = a64 @ b64
                return 0.5 * y * (1.0 + erf(y / np.sqrt(2.0)))
            ops = [(2 * rows * n * k, gemm_gelu)]
        else:
            ops = [(2 * rows * n * k, lambda: a64 @ b64)]
        threads = blas_threads()
        desc = (f"{rows} of {m} rows of the {ab} GEMM (1/{sample_scale} of a step) in float64 "
                f"numpy/BLAS" + (" with the erf-GELU" if config in GEMM_EPILOGUE else "") + f", {threads} threads")
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
        frac = "a full step" if sample_scale == 1 else f"1/{sample_scale} of a step"
        desc = f"5 elementwise ops over 2^{(n).bit_length() - 1} fp32 elements each ({frac})"
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
        frac = "a full step" if sample_scale == 1 else f"1/{sample_scale} of a step"
        desc = f"4 row ops over {r} x {COLS} fp32 rows ({frac})"
        keep = (x, w, out, rs)
    return ops, desc, threads, "GB/s", keep


def numpy_run(config, sample_scale):
    """The numpy formula oracle itself (float64 upcast, single-threaded) on a bounded sample."""
    import numpy as np

    from oracle import expressions as O
    rng = np.random.default_rng(0)
    if config == "elementwise":
        n = N_ELEMENTWISE // sample_scale
        x = rng.standard_normal(n, dtype=np.float32)
        y = rng.standard_normal(n, dtype=np.float32)
        ops = [(12 * n, lambda: (x.astype(np.float64) + y).astype(np.float32)),
               (8 * n, lambda: (1.5 * x.astype(np.float64) - 0.25).astype(np.float32)),
               (12 * n, lambda: (np.maximum(x.astype(np.float64), 0) * y).astype(np.float32)),
               (8 * n, lambda: O.gelu(x, "none")), (8 * n, lambda: O.gelu(x, "tanh"))]
        return ops, f"5 elementwise ops over {n} fp32 elements (1/{sample_scale} of a step)", (x, y)
    if config == "reduce":
        x = rng.uniform(-1, 1, N_REDUCE).astype(np.float32)
        return [(4 * N_REDUCE, lambda: O.sum_(x)), (4 * N_REDUCE, lambda: O.mean(x))], \
            "sum and mean of 2^24 fp32 (a full step)", (x,)
    if config == "rows":
        r = ROWS // sample_scale
        x = rng.standard_normal((r, COLS), dtype=np.float32)
        w = (rng.standard_normal(COLS) * 0.1 + 1).astype(np.float32)
        xb = 4 * r * COLS
        return [(2 * xb, lambda: O.rmsnorm(x, w, 1e-6)), (2 * xb, lambda: O.softmax(x)),
                (2 * xb, lambda: O.l2norm(x)), (xb, lambda: O.rowsum(x))], \
            f"4 row ops over {r} x {COLS} fp32 rows (1/{sample_scale} of a step)", (x, w)
    return None, None, None


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
    # the memory-bound configurations run whole (same configuration as ours); the
    # float64 BLAS GEMM / attention run a bounded slice of the step
    scale = {"elementwise": 1, "reduce": 1, "rows": 1, "sdpa": 8}.get(args.config, 64)
    ops, desc, threads, unit, keep = cpu_run(args.config, scale)
    cpu_time(ops, args.warmup)
    times = cpu_time(ops, args.steps)
    work = sum(o[0] for o in ops)
    value = work * args.steps / sum(times) / (1e12 if unit == "TFLOP/s" else 1e9)
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sum(times) * 1e3 / args.steps, 3), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "data": "synthetic (seeded numpy)",
        "dtype": {"gemm_f16": "f64 (f16 inputs)", "gemm_f16_gelu": "f64 (f16 inputs)", "gemm_bf16": "f64 (bf16 inputs)",
                  "sdpa": "f64 (f16 inputs)"}.get(args.config, "f32"),
        "config": {"workload": args.config, "sample": desc, "same_config": scale == 1},
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    np_ops, np_desc, np_keep = numpy_run(args.config, 16)
    if np_ops:
        cpu_time(np_ops, 1)
        np_times = cpu_time(np_ops, 3)
        np_work = sum(o[0] for o in np_ops)
        line["numpy_formulas"] = {
            "value": round(np_work / statistics.median(np_times) / 1e9, 4), "unit": "GB/s", "cores": 1,
            "sample": np_desc + "; the numpy float64 formula oracle itself (single-threaded numpy), median of 3",
            "cpu_count": os.cpu_count(), "affinity": len(os.sched_getaffinity(0)), "blas_threads": blas_threads()}
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
