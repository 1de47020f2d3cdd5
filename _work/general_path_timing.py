"""Times each package's fixed-class kernel against the same package run as a
block program (natively compiled, and through the interpreter) on the B200.

    python tests/general_path_timing.py [--repeat R]

Test infrastructure: one JSON object per package with the mean time per
launch through ``runtime.launch`` (host call included, after three warm-up
launches) of the plan ``compile.py`` prints, of the block program with
``LC_JIT`` on and of the block program through the interpreter.
"""
import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent))
sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from conftest import golden_ir, golden_meta  # noqa: E402
from lazy_compiler_b200.blockprog import compile_blockprog  # noqa: E402
from lazy_compiler_b200.compiler import compile_file  # noqa: E402
from lazy_compiler_b200.ir import load_package  # noqa: E402
from lazy_compiler_b200.runtime import launch  # noqa: E402
from oracle import expressions as O  # noqa: E402

PACKAGES = ["r01_array_sum", "r04_row_sum", "f01_rmsnorm", "f02_row_softmax", "phase9_gelu_attention",
            "a02_attention_128", "m02_matmul_rect", "m01_matmul_512"]


def buffers(meta):
    import torch
    types = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16, "s32": torch.int32}
    out = {}
    for a in meta["kernels"][0]["args"]:
        shape = tuple(a.get("shape") or [1])
        if a.get("output"):
            out[a["name"]] = torch.zeros(shape, device="cuda", dtype=types[a["dtype"]])
        else:
            out[a["name"]] = torch.as_tensor(np.ascontiguousarray(O.input_array(a, 0))).to("cuda", types[a["dtype"]])
    return out


def time_plan(plan, bufs, repeat):
    import torch
    ptrs = {n: t.data_ptr() for n, t in bufs.items()}
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        launch(plan, ptrs, stream)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(repeat):
        launch(plan, ptrs, stream)
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / repeat * 1000


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--repeat", type=int, default=50)
    args = ap.parse_args()
    for name in PACKAGES:
        meta = golden_meta(name)
        bufs = buffers(meta)
        fixed = compile_file(golden_ir(name))
        pkg = load_package(golden_ir(name))
        native = compile_blockprog(pkg, pkg.body[0]).to_json()
        interpreted = json.loads(json.dumps(native))
        row = {"package": name, "fixed_op": fixed["op"], "fixed_us": round(time_plan(fixed, bufs, args.repeat), 2)}
        row["block_native_us"] = round(time_plan(native, bufs, args.repeat), 2)
        os.environ["LC_JIT"] = "0"
        row["block_interpreted_us"] = round(time_plan(interpreted, bufs, max(3, args.repeat // 10)), 2)
        os.environ["LC_JIT"] = "1"
        print(json.dumps(row))


if __name__ == "__main__":
    main()
