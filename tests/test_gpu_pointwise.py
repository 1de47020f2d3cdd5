"""GPU parity of pointwise register programs (lc_pointwise) against the IR
oracle, on synthetic op mixes beyond the fixed classes, at each package's
stated tolerance; the C-ABI's validation of malformed programs."""
import ctypes
import json

import numpy as np
import pytest

import pw_packages as W
from lazy_compiler_b200 import runtime
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.runner import run_package
from oracle import expressions as O
from oracle import pointwise_ir

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(W.SYNTHETIC))
@pytest.mark.parametrize("offset", [0, 5])
def test_synthetic_program_on_gpu(name, offset, tmp_path, cuda_device):
    ir = W.SYNTHETIC[name](tmp_path / name)
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = pointwise_ir.evaluate(ir, arrays)
    out = run_package(tmp_path / name, inputs=arrays)
    for key, value in ref.items():
        row = O.compare(out[key], value, meta["rtol"], meta["atol"])
        assert row["pass"], (key, row)


def test_program_validation_rejects_bad_programs(tmp_path, cuda_device):
    import torch
    ir = W.SYNTHETIC["erf_log"](tmp_path / "erf_log")
    plan = compile_file(ir)
    prog = plan["params"]["program"]
    x = torch.zeros(4099, device="cuda")
    ptrs = (ctypes.c_void_p * runtime.PW_MAX_BUFFERS)(*[x.data_ptr()] * len(prog["buffers"]))
    lib = runtime.library()

    def status(g):
        return lib.lc_pointwise(ctypes.c_void_p(ctypes.addressof(g)), ptrs, None)

    good = runtime.pw_program(prog)
    assert status(good) == 0
    torch.cuda.synchronize()
    bad = runtime.pw_program(prog)
    bad.sizes[0] = 4098                      # a form would read past the buffer
    assert status(bad) == -1
    bad = runtime.pw_program(prog)
    bad.code[0][0] = (bad.code[0][0] & ~0xFF) | 250   # unknown opcode
    assert status(bad) == -1
    bad = runtime.pw_program(prog)
    bad.code[0][0] |= 60 << 8                # destination register beyond n_regs
    assert status(bad) == -1
    bad = runtime.pw_program(prog)
    bad.forms[0].dtype = runtime.LC_S32      # storage type disagrees with the load
    assert status(bad) == -1
    assert lib.lc_pointwise(None, ptrs, None) == -1
