"""GPU parity of row programs (lc_rowprog): synthetic op mixes against the
row oracle, the fixed reduction classes forced through the row compiler
against the reference's golden vectors, and the C-ABI's validation."""
import ctypes
import json

import numpy as np
import pytest

import pw_packages as W
from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200 import runtime
from lazy_compiler_b200.runner import run_package
from oracle import expressions as O
from oracle import rowprog_ir
from test_gpu_lanes import run_plan
from test_row_programs import REDUCTIONS, forced_plan

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(W.ROW_SYNTHETIC))
@pytest.mark.parametrize("offset", [0, 4])
def test_synthetic_row_program_on_gpu(name, offset, tmp_path, cuda_device):
    ir = W.ROW_SYNTHETIC[name](tmp_path / name)
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = rowprog_ir.evaluate(ir, arrays)
    out = run_package(tmp_path / name, inputs=arrays)
    for key, value in ref.items():
        row = O.compare(out[key], value, meta["rtol"], meta["atol"])
        assert row["pass"], (key, row)


@pytest.mark.parametrize("name", REDUCTIONS)
def test_fixed_reductions_as_row_programs_on_gpu(name, cuda_device):
    plan = forced_plan(golden_ir(name))
    meta = golden_meta(name)
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    got = run_plan(plan, meta, arrays)
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            row = O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])
            assert row["pass"], row


def test_row_program_validation(tmp_path, cuda_device):
    import torch
    plan = forced_plan(golden_ir("r04_row_sum"))
    prog, layout = plan["params"]["program"], plan["params"]["layout"]
    x = torch.zeros(64 * 512, device="cuda")
    ptrs = (ctypes.c_void_p * runtime.PW_MAX_BUFFERS)(*[x.data_ptr()] * len(prog["buffers"]))
    lib = runtime.library()

    def status(g, lay):
        return lib.lc_rowprog(ctypes.c_void_p(ctypes.addressof(g)), ctypes.c_void_p(ctypes.addressof(lay)), ptrs, None)

    assert status(runtime.pw_program(prog), runtime.rp_layout(layout)) == 0
    torch.cuda.synchronize()
    lay = runtime.rp_layout(layout)
    lay.end[0] = 10_000                     # a pass range past the program
    assert status(runtime.pw_program(prog), lay) == -1
    lay = runtime.rp_layout(layout)
    lay.state_pass[0] = 3                   # a state of a pass that does not exist
    assert status(runtime.pw_program(prog), lay) == -1
    # a pointwise launch may not use state operations
    assert lib.lc_pointwise(ctypes.c_void_p(ctypes.addressof(runtime.pw_program(prog))), ptrs, None) == -1


@pytest.mark.parametrize("name", sorted(W.ROW_COUPLED))
def test_online_softmax_variants_on_gpu(name, tmp_path, cuda_device):
    ir = W.ROW_COUPLED[name](tmp_path / name)
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    for offset in (0, 5):
        arrays = {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}
        ref = rowprog_ir.evaluate(ir, arrays)
        out = run_package(tmp_path / name, inputs=arrays)
        for key, value in ref.items():
            row = O.compare(out[key], value, 1e-5, 1e-6)
            assert row["pass"], (key, row)
