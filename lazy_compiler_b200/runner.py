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
