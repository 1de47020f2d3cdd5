"""Runs an IR package on the GPU the way the reference's runner does.

Mirrors the reference's local runner (tools/check_compiler.py:291-422
``CudaDriver.run`` and :425-445 ``local_run``) and the organiser runner's
``/run`` semantics (docs/API.md:26-72, submit.py:112-135):

* every kernel of ``meta.json["kernels"]`` is compiled (``compile.py``'s
  ``compile_file``) and launched in order; ``intermediate`` arguments chain
  the outputs of earlier kernels;
* seeded inputs are ``default_rng(seed + offset).standard_normal(shape)``
  drawn in float64 then cast, ``data`` arguments are taken verbatim;
* outputs are prefilled with NaN (floating) or -1 (integer) so an element the
  kernel forgets to write cannot pass;
* ``zero_outputs`` are zeroed before every launch.

Device memory comes from PyTorch (plumbing only); the kernels are the
C-ABI entry points of ``liblazyb200.so`` reached through :mod:`.runtime`.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np

from .compiler import compile_file
from .ir import CompileError
from .runtime import launch

_NP = {"f32": np.float32, "f16": np.float16, "f64": np.float64, "i32": np.int32,
       "bf16": np.float32}


def _torch_dtype(kind: str):
    import torch
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16,
            "f64": torch.float64, "i32": torch.int32}[kind]


def seeded_input(arg: dict, seed_offset: int = 0) -> np.ndarray:
    """Host values of one non-output argument (runner convention, docs/API.md:46)."""
    kind = arg["dtype"]
    shape = tuple(arg.get("shape") or [1])
    if "data" in arg:
        return np.asarray(arg["data"], dtype=np.float64 if kind == "bf16" else _NP[kind]).reshape(shape)
    rng = np.random.default_rng(int(arg.get("seed", 0)) + seed_offset)
    values = rng.standard_normal(shape)
    return values if kind == "bf16" else values.astype(_NP[kind])


def _ir_for_entry(folder: Path, entry: str) -> Path:
    for path in sorted(folder.glob("*.ir.json")):
        graph = json.loads(path.read_text())
        for node in graph.get("nodes", {}).values():
            if node.get("op") == "KernelOp" and node.get("op_fields", {}).get("name") == entry:
                return path
    raise CompileError(f"no IR in {folder} defines kernel {entry}")


def run_package(folder: str | Path, seed_offset: int = 0, device: str = "cuda",
                inputs: dict | None = None) -> dict:
    """Compile and run every kernel of a package; returns graph outputs as numpy arrays.

    ``inputs`` optionally overrides argument values by name (host arrays or
    tensors, which are used in place when already on the device).
    """
    import torch

    folder = Path(folder)
    meta = json.loads((folder / "meta.json").read_text())
    dev = torch.device(device)
    stream = torch.cuda.current_stream(dev)
    buffers: dict[str, torch.Tensor] = {}
    for kernel in meta["kernels"]:
        plan = compile_file(_ir_for_entry(folder, kernel["entry"]), folder / "meta.json")
        by_name = {a["name"]: a for a in kernel["args"]}
        for name in kernel["arg_order"]:
            arg = by_name[name]
            if name in buffers and (arg.get("intermediate") or arg.get("output")):
                continue
            kind = arg["dtype"]
            shape = tuple(arg.get("shape") or [1])
            if arg.get("output"):
                t = torch.empty(shape, dtype=_torch_dtype(kind), device=dev)
                t.fill_(-1 if kind.startswith("i") else math.nan)
            elif arg.get("intermediate"):
                raise CompileError(f"intermediate {name} is used before it is produced")
            else:
                given = inputs.get(name) if inputs else None
                if isinstance(given, torch.Tensor):
                    t = given.to(dev, _torch_dtype(kind)).contiguous()
                else:
                    host = given if given is not None else seeded_input(arg, seed_offset)
                    t = torch.as_tensor(np.ascontiguousarray(host)).to(dev, _torch_dtype(kind))
            buffers[name] = t
        for name in kernel.get("zero_outputs", []):
            buffers[name].zero_()
        launch(plan, {n: buffers[n].data_ptr() for n in kernel["arg_order"]}, stream.cuda_stream)
    torch.cuda.synchronize(dev)
    out = {}
    for name in meta["graph_outputs"]:
        t = buffers[name]
        out[name] = (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy()
    return out


# ---------------------------------------------------------------- /run requests

_RUN_DTYPES = ("f32", "f16", "bf16", "f64", "i32")
_LIMITS = {"warmup": 20, "iters": 200, "elements": 1 << 26, "max_return": 1 << 22}


def _request_error(stage: str, message: str) -> dict:
    return {"ok": False, "stage": stage, "stderr": message}


def run_request(request: dict, device: str = "cuda") -> dict:
    """One launch with the request and response of the reference runner's ``POST /run``.

    The request carries, in place of ``ptx`` / ``cubin_id``, the ``plan`` that
    ``compile.py`` printed for the kernel; ``entry``, ``grid``, ``block``,
    ``smem_bytes``, ``zero_outputs``, ``warmup``, ``iters``, ``max_return`` and
    the positional ``args`` (``seed`` / ``data`` / ``output``) mean what they
    mean there (docs/API.md:26-72).  The launch geometry is checked against
    the plan's meta.json geometry, as the runner launches exactly that.

    Returns ``{"ok": True, "median_us", "iters", "outputs": {name: {"shape",
    "dtype", "sum", "values", "truncated"}}}``, or ``{"ok": False, "stage",
    "stderr"}`` with stage ``request`` (malformed or out-of-range request) or
    ``run`` (the launch failed).  Outputs are zeroed before the first launch
    and ``zero_outputs`` before every launch; ``median_us`` is the median of
    ``iters`` launches timed with CUDA events.
    """
    import torch

    from .runtime import LcError

    plan = request.get("plan")
    if not isinstance(plan, dict) or "op" not in plan:
        return _request_error("request", "the request carries no compiled plan")
    entry = request.get("entry")
    if entry != plan.get("entry"):
        return _request_error("run", f"entry {entry!r} is not the plan's kernel {plan.get('entry')!r}")
    geometry = plan.get("reference_launch") or {}
    for key in ("grid", "block"):
        if key in request and key in geometry and list(request[key]) != list(geometry[key]):
            return _request_error("request", f"{key} {request[key]} differs from the kernel's {geometry[key]}")
    warmup, iters = int(request.get("warmup", 0)), int(request.get("iters", 1))
    max_return = int(request.get("max_return", 4096))
    if not (0 <= warmup <= _LIMITS["warmup"] and 1 <= iters <= _LIMITS["iters"]
            and 0 <= max_return <= _LIMITS["max_return"]):
        return _request_error("request", "warmup, iters or max_return out of range")
    args = request.get("args")
    if not isinstance(args, list) or [a.get("name") for a in args] != list(plan["arg_order"]):
        return _request_error("request", f"args must be given in the kernel's order {plan['arg_order']}")
    total = 0
    for a in args:
        if a.get("dtype") not in _RUN_DTYPES:
            return _request_error("request", f"unsupported dtype {a.get('dtype')!r} for {a.get('name')}")
        total += math.prod(a.get("shape") or [1])
    if total > _LIMITS["elements"]:
        return _request_error("request", "buffers exceed 2^26 elements")
    dev = torch.device(device)
    stream = torch.cuda.current_stream(dev)
    buffers = {}
    for a in args:
        shape = tuple(a.get("shape") or [1])
        if a.get("output"):
            buffers[a["name"]] = torch.zeros(shape, dtype=_torch_dtype(a["dtype"]), device=dev)
        else:
            host = seeded_input(a)
            buffers[a["name"]] = torch.as_tensor(np.ascontiguousarray(host)).to(dev, _torch_dtype(a["dtype"]))
    pointers = {n: t.data_ptr() for n, t in buffers.items()}
    zero = [n for n in request.get("zero_outputs", []) if n in buffers]
    times = []
    try:
        for i in range(warmup + iters):
            for n in zero:
                buffers[n].zero_()
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            launch(plan, pointers, stream.cuda_stream)
            stop.record(stream)
            if i >= warmup:
                times.append((start, stop))
        torch.cuda.synchronize(dev)
    except (LcError, ValueError, KeyError) as err:
        return _request_error("run", str(err))
    median = float(np.median([s.elapsed_time(e) * 1000.0 for s, e in times]))
    outputs, budget = {}, max_return
    for a in args:
        if not a.get("output"):
            continue
        t = buffers[a["name"]]
        values = (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy().ravel()
        take = min(budget, values.size)
        budget -= take
        outputs[a["name"]] = {"shape": list(t.shape), "dtype": a["dtype"], "sum": float(values.astype(np.float64).sum()),
                              "values": values[:take].tolist(), "truncated": take < values.size}
    return {"ok": True, "median_us": round(median, 3), "iters": iters, "outputs": outputs}
