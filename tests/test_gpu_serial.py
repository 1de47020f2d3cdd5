"""GPU parity of serial programs (per-point runtime loops) against the serial
oracle and the reference's golden vectors; validation of malformed loops."""
import ctypes
import json

import numpy as np
import pytest

import pw_packages as W
from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200 import runtime
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.ir import load_package
from lazy_compiler_b200.runner import run_package
from lazy_compiler_b200.serial import compile_serial
from oracle import expressions as O
from oracle import serial_ir
from test_gpu_lanes import run_plan
from test_serial_programs import changed_a02

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(W.SERIAL_SYNTHETIC))
@pytest.mark.parametrize("offset", [0, 6])
def test_synthetic_serial_on_gpu(name, offset, tmp_path, cuda_device):
    ir = W.SERIAL_SYNTHETIC[name](tmp_path / name)
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = serial_ir.evaluate(ir, arrays)
    out = run_package(tmp_path / name, inputs=arrays)
    for key, value in ref.items():
        row = O.compare(out[key], value, meta["rtol"], meta["atol"])
        assert row["pass"], (key, row)


def test_a02_as_serial_program_on_gpu(cuda_device):
    pkg = load_package(golden_ir("a02_attention_128"))
    plan = compile_serial(pkg, pkg.body[0]).to_json()
    meta = golden_meta("a02_attention_128")
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    got = run_plan(plan, meta, arrays)
    with np.load(golden("a02_attention_128") / "expected.npz") as z:
        for key in z.files:
            row = O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])
            assert row["pass"], row


def test_changed_attention_on_gpu(tmp_path, cuda_device):
    ir = changed_a02(tmp_path)
    meta = json.loads((ir.parent / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, 2) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = serial_ir.evaluate(ir, arrays)
    out = run_package(ir.parent, inputs=arrays)
    for key, value in ref.items():
        assert O.compare(out[key], value, 1e-4, 1e-5)["pass"]


def test_malformed_loops_are_rejected(tmp_path, cuda_device):
    import torch
    ir = W.SERIAL_SYNTHETIC["serial_nested"](tmp_path / "n")
    plan = compile_file(ir)
    prog = plan["params"]["program"]
    x = torch.zeros(1024, device="cuda")
    ptrs = (ctypes.c_void_p * runtime.PW_MAX_BUFFERS)(*[x.data_ptr()] * len(prog["buffers"]))
    lib = runtime.library()
    loopb = next(i for i, ins in enumerate(prog["code"]) if ins[0] == runtime_op("LOOPB"))
    bad = runtime.pw_program(prog)
    bad.code[loopb][1] = (bad.code[loopb][1] & 0xFF) | ((bad.code[loopb][1] >> 8 & 15) | (loopb + 1) << 4) << 8
    assert lib.lc_pointwise(ctypes.c_void_p(ctypes.addressof(bad)), ptrs, None) == -1   # target is not its LOOPE
    bad = runtime.pw_program(prog)
    bad.extents[bad.n_axes] = -1                                                      # negative loop extent
    assert lib.lc_pointwise(ctypes.c_void_p(ctypes.addressof(bad)), ptrs, None) == -1


def runtime_op(name):
    from lazy_compiler_b200.pointwise import OP
    return OP[name]
