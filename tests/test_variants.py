"""Op-mix variants of the reference's own packages (a changed activation,
score scale or accumulated expression): a fixed class must not take them,
and the general path they fall to must compute what the changed IR says —
checked on CPU (compiled program in numpy against the IR oracles) and, with
-m gpu, on the device."""
import importlib
import json

import pytest

import pw_packages as W
import pw_vm
from lazy_compiler_b200.compiler import compile_file
from oracle import expressions as O


def check(ir, plan, got, offset):
    meta = json.loads((ir.parent / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}
    oracle = importlib.import_module("oracle." + W.VARIANTS[ir.parent.name][3])
    ref = oracle.evaluate(ir, arrays)
    out = got(plan, arrays)
    for key, value in ref.items():
        row = O.compare(out[key].reshape(value.shape), value, 1e-4, 1e-5)
        assert row["pass"], (key, row)


def cpu(plan, arrays):
    p = plan["params"]
    if plan["op"] == "rowprog":
        return pw_vm.run_rows(p["program"], p["layout"], arrays)
    if plan["op"] == "blockprog":
        return pw_vm.run_block(p["program"], p["layout"], arrays)
    return pw_vm.run(p["program"], arrays)


@pytest.mark.parametrize("name", sorted(W.VARIANTS))
def test_variant_runs_as_its_general_program(name, tmp_path):
    ir = W.variant(tmp_path / name, name)
    plan = compile_file(ir)
    assert plan["op"] == W.VARIANTS[name][2], plan["op"]
    check(ir, plan, cpu, 1)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(W.VARIANTS))
def test_variant_on_gpu(name, tmp_path, cuda_device):
    from lazy_compiler_b200.runner import run_package
    ir = W.variant(tmp_path / name, name)
    plan = compile_file(ir)
    check(ir, plan, lambda plan, arrays: run_package(ir.parent, inputs=arrays), 3)
