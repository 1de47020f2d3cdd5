"""The pointwise-program compiler (straight-line Tile bodies outside the fixed
classes), checked on CPU: the compiled register program, interpreted in
numpy (tests/pw_vm.py), against the IR oracle (oracle/pointwise_ir.py) and
the reference's golden vectors; rejection of bodies that are not pointwise
programs; the opcode table against the C header."""
import json
import re

import numpy as np
import pytest

import pw_packages as W
import pw_vm
from conftest import ROOT, golden, golden_ir, golden_meta
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.ir import CompileError
from lazy_compiler_b200.pointwise import OPCODES
from oracle import expressions as O
from oracle import pointwise_ir

ACTIVATION = sorted(p.name for p in golden("").iterdir()
                    if p.name.startswith("activation_") or p.name.startswith("floating_f32_"))


def inputs_of(meta, offset=0):
    return {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}


def test_opcodes_match_header():
    text = (ROOT / "include" / "lazyb200.h").read_text()
    enum = re.findall(r"LC_PW_([A-Z0-9_]+) = (\d+),", text)
    assert [(n, int(i)) for n, i in enum] == [(n, i) for i, n in enumerate(OPCODES)]


@pytest.mark.parametrize("name", ACTIVATION)
def test_activation_fixture_program_matches_golden(name):
    plan = compile_file(golden_ir(name))
    assert plan["op"] == "pointwise"
    meta = golden_meta(name)
    got = pw_vm.run(plan["params"]["program"], inputs_of(meta))
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            row = O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])
            assert row["pass"], row


@pytest.mark.parametrize("name", ACTIVATION)
def test_ir_oracle_matches_golden(name):
    meta = golden_meta(name)
    got = pointwise_ir.evaluate(golden_ir(name), inputs_of(meta))
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key], z[key], meta["rtol"], meta["atol"])["pass"]


@pytest.mark.parametrize("name", sorted(W.SYNTHETIC))
def test_synthetic_program_matches_ir_oracle(name, tmp_path):
    ir = W.SYNTHETIC[name](tmp_path / name)
    plan = compile_file(ir)
    assert plan["op"] == "pointwise", plan["op"]
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    for offset in (0, 3):
        arrays = inputs_of(meta, offset)
        ref = pointwise_ir.evaluate(ir, arrays)
        got = pw_vm.run(plan["params"]["program"], arrays)
        for key, value in ref.items():
            row = O.compare(got[key].reshape(value.shape), value, meta["rtol"], meta["atol"])
            assert row["pass"], (key, row)


def _simple(folder, body, out_shape=(64,), axes=(("i", 64),), inputs=None):
    return W.package(folder, "bad", inputs or {"x": ((64,), "f32")}, ("out", out_shape, "f32"), list(axes), body)


I = W.var("i")
REJECT = {
    "index_leaves_output": ([W.load("v", "x", [I], "f32"), W.write("out", [W.bin_("+", I, W.lit(1))], ["v"], "f32")],
                            "leaves the buffer"),
    "hole_in_output": ([W.load("v", "x", [I], "f32"), W.write("out", [I], ["v"], "f32")], "cover",
                       (65,)),
    "non_affine_index": ([W.load("v", "x", [W.bin_("*", I, I)], "f32"), W.write("out", [I], ["v"], "f32")],
                         "affine|leaves"),
    "unsupported_power": ([W.load("v", "x", [I], "f32"), W.assign("p", "power", ["v", "v"], "f32"),
                           W.write("out", [I], ["p"], "f32")], "power"),
    "write_to_input": ([W.load("v", "x", [I], "f32"), W.write("x", [I], ["v"], "f32")], "kernel.s outputs|write"),
}


@pytest.mark.parametrize("case", sorted(REJECT))
def test_rejected_bodies(case, tmp_path):
    body, match, *shape = REJECT[case]
    ir = _simple(tmp_path / case, body, out_shape=shape[0] if shape else (64,))
    with pytest.raises(CompileError, match=match):
        compile_file(ir)


def test_duplicate_writes_rejected(tmp_path):
    body = [W.load("v", "x", [I], "f32"), W.write("out", [I], ["v"], "f32"),
            W.write("out", [W.bin_("-", W.lit(63), I)], ["v"], "f32")]
    ir = W.package(tmp_path / "dup", "dup", {"x": ((64,), "f32")}, ("out", (128,), "f32"), [("i", 64)], body)
    with pytest.raises(CompileError, match="exactly once|cover"):
        compile_file(ir)


def test_large_tile_coverage_by_strides(tmp_path):
    """2^25 points: coverage is proved from the strides, not enumerated."""
    i, j = W.var("i"), W.var("j")
    body = [W.load("v", "x", [i, j], "f32"), W.assign("r", "abs", ["v"], "f32"), W.write("out", [i, j], ["r"], "f32")]
    ir = W.package(tmp_path / "big", "big", {"x": ((8192, 4096), "f32")}, ("out", (8192, 4096), "f32"),
                   [("i", 8192), ("j", 4096)], body)
    plan = compile_file(ir)
    assert plan["op"] == "pointwise" and plan["params"]["points"] == 1 << 25
    # the same tile writing every other row twice is rejected without enumeration
    body[-1] = W.write("out", [W.bin_("*", i, W.lit(1)), W.bin_("*", j, W.lit(1))], ["r"], "f32").replace(
        "Var(name='j')", "Var(name='j')").replace("left=Var(name='i'), right=Literal(value=1",
                                                  "left=Var(name='i'), right=Literal(value=2")
    ir = W.package(tmp_path / "big2", "big2", {"x": ((8192, 4096), "f32")}, ("out", (16384, 4096), "f32"),
                   [("i", 8192), ("j", 4096)], body)
    with pytest.raises(CompileError, match="cover"):
        compile_file(ir)
