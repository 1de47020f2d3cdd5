"""Staged (cp.async, shared-memory) matmuls: the block oracle
(oracle/staged_ir.py) against the reference's golden vectors, and staged
matmuls whose Write stores an expression of the accumulator (an activation,
a scaled SiLU, a bias and residual) — the GEMM plus an epilogue program —
against that oracle: on CPU with the GEMM in float64 and the epilogue
program in numpy (tests/pw_vm.py), with -m gpu through the runner."""
import json

import numpy as np
import pytest

import pw_packages as W
import pw_vm
from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200.compiler import compile_file
from oracle import expressions as O
from oracle import staged_ir


def inputs_of(meta, offset=0):
    return {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}


@pytest.mark.parametrize("name", ["m01_matmul_512", "m02_matmul_rect"])
def test_staged_oracle_matches_golden(name):
    meta = golden_meta(name)
    got = staged_ir.evaluate(golden_ir(name), inputs_of(meta))
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]


def test_plain_staged_matmul_has_no_epilogue_program():
    plan = compile_file(golden_ir("m01_matmul_512"))
    assert plan["op"] == "gemm" and "post" not in plan["params"]


def cpu(plan, arrays):
    p = plan["params"]
    a = arrays[plan["bind"]["a"]].astype(np.float64)
    b = arrays[plan["bind"]["b"]].astype(np.float64)
    c = a @ (b if p["b_layout"] == "kn" else b.T)
    return pw_vm.run(p["post"]["program"], {**arrays, plan["bind"]["c"]: c.astype(np.float32)})


@pytest.mark.parametrize("name", sorted(W.STAGED_EPILOGUES))
def test_staged_epilogue_matches_oracle(name, tmp_path):
    ir = W.STAGED_EPILOGUES[name](tmp_path / name)
    plan = compile_file(ir)
    assert plan["op"] == "gemm" and plan["params"]["epilogue"] == "none" and "post" in plan["params"]
    meta = json.loads((ir.parent / "meta.json").read_text())
    arrays = inputs_of(meta, 1)
    ref = staged_ir.evaluate(ir, arrays)
    got = cpu(plan, arrays)
    for key, value in ref.items():
        assert O.compare(got[key].reshape(value.shape), value, meta["rtol"], meta["atol"])["pass"]


def test_epilogue_reading_two_accumulators_is_not_a_gemm(tmp_path):
    """acc(r, c) + acc(r, c+1) stored at (r, c+1): not an expression of one
    element's accumulator, so not a GEMM plus epilogue; it runs as the block
    program it is."""
    names = []

    def epi(acc, t, row, col):
        names.append(acc)
        if len(names) % 2 == 0:
            return [W.assign(t, "add", [names[-2], acc])], t
        return [W.assign(t, "copy", [acc])], t
    ir = W.staged_epilogue(tmp_path / "mixed", epi)
    assert compile_file(ir)["op"] == "blockprog"


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(W.STAGED_EPILOGUES))
def test_staged_epilogue_on_gpu(name, tmp_path, cuda_device):
    from lazy_compiler_b200.runner import run_package
    ir = W.STAGED_EPILOGUES[name](tmp_path / name)
    meta = json.loads((ir.parent / "meta.json").read_text())
    arrays = inputs_of(meta, 2)
    ref = staged_ir.evaluate(ir, arrays)
    got = run_package(ir.parent, inputs=arrays)
    for key, value in ref.items():
        assert O.compare(np.asarray(got[key]).reshape(value.shape), value, meta["rtol"], meta["atol"])["pass"]
