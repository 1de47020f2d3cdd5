"""Launches the reference compiler's PTX on the GPU — TEST AND BASELINE INFRASTRUCTURE ONLY.

The PTX in ``oracle/_ref/ptx`` is what the reference's own ``compile_file``
emitted for each package (``oracle/ref_ptx.py``, hashes checked against the
reference's records).  This module JIT-loads it with the CUDA driver
(``cuModuleLoadData``) and launches the entry under the package's meta.json
geometry with `.u64` arguments in ``arg_order`` — the reference's launcher
contract (tools/check_compiler.py:291-422): seeded inputs, outputs prefilled
with NaN / -1, ``zero_outputs`` zeroed before every launch.  Device memory
comes from PyTorch; the PTX text is never parsed or modified.  Used by the
tests (parity with this backend) and by ``bench.py``'s reference-PTX
baseline leg (the reference's own kernels timed on the same B200); never by
the product.
"""
from __future__ import annotations

import ctypes
import json
import math
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "oracle" / "_ref"
CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES = 8

_cuda = None


def driver():
    global _cuda
    if _cuda is None:
        _cuda = ctypes.CDLL("libcuda.so.1")
        _cuda.cuGetErrorString.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p)]
    return _cuda


def check(status: int, what: str) -> None:
    if status:
        msg = ctypes.c_char_p()
        driver().cuGetErrorString(status, ctypes.byref(msg))
        raise RuntimeError(f"{what}: CUDA driver error {status} ({(msg.value or b'').decode()})")


def manifest() -> dict:
    path = REF / "manifest.json"
    return json.loads(path.read_text()) if path.exists() else {}


def manifest_rescaled() -> dict:
    path = REF / "manifest_rescaled.json"
    return json.loads(path.read_text()) if path.exists() else {}


class RefKernel:
    """One reference-compiled PTX module, JIT-loaded on the current device."""

    def __init__(self, name: str, rescaled: bool = False):
        import torch
        torch.cuda.init()
        torch.cuda.current_stream()  # make the primary context current
        row = (manifest_rescaled() if rescaled else manifest())[name]
        self.meta = row["meta"]
        self.kernel_meta = self.meta["kernels"][0]
        folder = "ptx_rescaled" if rescaled else "ptx"
        image = (REF / folder / f"{name}.ptx").read_bytes() + b"\0"
        cu = driver()
        self.module = ctypes.c_void_p()
        check(cu.cuModuleLoadData(ctypes.byref(self.module), ctypes.c_char_p(image)), "cuModuleLoadData")
        self.function = ctypes.c_void_p()
        check(cu.cuModuleGetFunction(ctypes.byref(self.function), self.module,
                                     self.kernel_meta["entry"].encode()), "cuModuleGetFunction")
        smem = int(self.kernel_meta.get("smem_bytes", 0))
        if smem > 48 * 1024:
            check(cu.cuFuncSetAttribute(self.function, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                        ctypes.c_int(smem)), "cuFuncSetAttribute")

    def launch(self, pointers: dict, stream: int = 0) -> None:
        km = self.kernel_meta
        values = [ctypes.c_uint64(int(pointers[name])) for name in km["arg_order"]]
        params = (ctypes.c_void_p * len(values))(*[ctypes.cast(ctypes.byref(v), ctypes.c_void_p) for v in values])
        grid, block = km["grid"], km["block"]
        check(driver().cuLaunchKernel(self.function, *map(ctypes.c_uint, grid), *map(ctypes.c_uint, block),
                                      ctypes.c_uint(int(km.get("smem_bytes", 0))), ctypes.c_void_p(stream),
                                      params, None), "cuLaunchKernel")

    def run(self, inputs: dict | None = None, seed_offset: int = 0, keep: bool = False):
        """Allocate, launch once, return graph outputs (numpy; with ``keep`` also the buffers)."""
        import torch
        from lazy_compiler_b200.runner import _torch_dtype, seeded_input
        km = self.kernel_meta
        args = {a["name"]: a for a in km["args"]}
        buffers = {}
        for name in km["arg_order"]:
            arg = args[name]
            shape = tuple(arg.get("shape") or [1])
            if arg.get("output"):
                t = torch.empty(shape, dtype=_torch_dtype(arg["dtype"]), device="cuda")
                t.fill_(-1 if arg["dtype"].startswith("i") else math.nan)
            else:
                given = inputs.get(name) if inputs else None
                if isinstance(given, torch.Tensor):
                    t = given.to("cuda", _torch_dtype(arg["dtype"])).contiguous()
                else:
                    host = given if given is not None else seeded_input(arg, seed_offset)
                    t = torch.as_tensor(np.ascontiguousarray(host)).to("cuda", _torch_dtype(arg["dtype"]))
            buffers[name] = t
        for name in km.get("zero_outputs", []):
            buffers[name].zero_()
        self.launch({n: t.data_ptr() for n, t in buffers.items()},
                    torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        out = {}
        for name in self.meta["graph_outputs"]:
            t = buffers[name]
            out[name] = (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy()
        return (out, buffers) if keep else out
