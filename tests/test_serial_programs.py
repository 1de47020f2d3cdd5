"""Serial programs (per-point bodies with runtime loops: small contractions,
the scalar attention schedule, their op mixes), on CPU: the compiled
program, interpreted in numpy (tests/pw_vm.py), against the serial oracle
(oracle/serial_ir.py) and the reference's golden vectors."""
import json
import shutil

import numpy as np
import pytest

import pw_packages as W
import pw_vm
from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.ir import CompileError, load_package
from lazy_compiler_b200.serial import compile_serial
from oracle import expressions as O
from oracle import serial_ir


def inputs_of(meta, offset=0):
    return {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}


def test_a02_as_serial_program_matches_golden():
    pkg = load_package(golden_ir("a02_attention_128"))
    plan = compile_serial(pkg, pkg.body[0]).to_json()
    assert plan["params"]["program"]["loops"] == [128, 32]
    meta = golden_meta("a02_attention_128")
    got = pw_vm.run(plan["params"]["program"], inputs_of(meta))
    with np.load(golden("a02_attention_128") / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]


def test_serial_oracle_matches_golden():
    meta = golden_meta("a02_attention_128")
    got = serial_ir.evaluate(golden_ir("a02_attention_128"), inputs_of(meta))
    with np.load(golden("a02_attention_128") / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]


@pytest.mark.parametrize("name", sorted(W.SERIAL_SYNTHETIC))
def test_synthetic_serial_program_matches_oracle(name, tmp_path):
    ir = W.SERIAL_SYNTHETIC[name](tmp_path / name)
    plan = compile_file(ir)
    assert plan["op"] == "pointwise" and plan["params"]["serial"]
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    for offset in (0, 2):
        arrays = inputs_of(meta, offset)
        ref = serial_ir.evaluate(ir, arrays)
        got = pw_vm.run(plan["params"]["program"], arrays)
        for key, value in ref.items():
            assert O.compare(got[key].reshape(value.shape), value, meta["rtol"], meta["atol"])["pass"]


def changed_a02(tmp_path):
    """a02 with the score scaled by sqrt(c) instead of 1/c: no longer the FP32 attention class."""
    dst = tmp_path / "a02_sqrt"
    shutil.copytree(golden("a02_attention_128"), dst)
    ir = next(dst.glob("*.ir.json"))
    text = ir.read_text()
    old = "Assign(name='v1', op=ElementwiseImpl('reciprocal'), args=('in0',)"
    assert old in text
    ir.write_text(text.replace(old, "Assign(name='v1', op=ElementwiseImpl('sqrt'), args=('in0',)"))
    return ir


def test_changed_attention_runs_as_serial_program(tmp_path):
    ir = changed_a02(tmp_path)
    plan = compile_file(ir)
    assert plan["op"] == "pointwise" and plan["params"]["serial"]
    meta = json.loads((ir.parent / "meta.json").read_text())
    arrays = inputs_of(meta, 1)
    ref = serial_ir.evaluate(ir, arrays)
    got = pw_vm.run(plan["params"]["program"], arrays)
    for key, value in ref.items():
        assert O.compare(got[key].reshape(value.shape), value, 1e-4, 1e-5)["pass"]


def test_serial_writes_must_cover_the_output(tmp_path):
    i, k = W.var("i"), W.var("k")
    ir = W.serial_package(tmp_path / "hole", "hole", {"x": ((8, 5), "f32")}, ("out", (9,), "f32"), [("i", 8)],
                          [W.loop("k", 5, [W.load("xv", "x", [i, k], "f32"), W.accum("s", "xv", "add")]),
                           W.write("out", [i], ["s"], "f32")])
    with pytest.raises(CompileError, match="cover"):
        compile_file(ir)


def test_values_defined_before_a_loop_survive_its_back_edge(tmp_path):
    """A value computed before the loop and read in its body is still intact on the
    last iteration, even after the body allocated many temporaries."""
    i, k = W.var("i"), W.var("k")
    body = [W.let("c", W.lit(1.5, "f32"), "f32"),
            W.loop("k", 64, [W.load("xv", "x", [i, k], "f32")] +
                   [W.assign(f"t{n}", "add", ["xv" if n == 0 else f"t{n - 1}", "xv"], "f32") for n in range(12)] +
                   [W.assign("u", "multiply", ["t11", "c"], "f32"), W.accum("s", "u", "add")]),
            W.write("out", [i], ["s"], "f32")]
    ir = W.serial_package(tmp_path / "live", "live", {"x": ((4, 64), "f32")}, ("out", (4,), "f32"), [("i", 4)], body)
    plan = compile_file(ir)
    meta = json.loads((tmp_path / "live" / "meta.json").read_text())
    arrays = inputs_of(meta)
    got = pw_vm.run(plan["params"]["program"], arrays)
    expect = (arrays["x"].astype(np.float64) * 13 * 1.5).sum(axis=1)
    np.testing.assert_allclose(got["out"], expect, rtol=1e-5)
