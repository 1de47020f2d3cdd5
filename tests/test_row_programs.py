"""Row programs (reductions and fused row operations of any op mix), on CPU:
the compiled program, interpreted in numpy (tests/pw_vm.py), against the
row oracle (oracle/rowprog_ir.py) and the reference's golden vectors; the
checks that keep a body from being compiled as something it is not."""
import json

import numpy as np
import pytest

import pw_packages as W
import pw_vm
from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.ir import load_package, static_extent
from lazy_compiler_b200.recognize import _Eval
from lazy_compiler_b200.rowprog import compile_rowprog
from oracle import expressions as O
from oracle import rowprog_ir

REDUCTIONS = ["r01_array_sum", "r02_big_sum", "r03_mean", "r04_row_sum", "f01_rmsnorm", "f02_row_softmax",
              "f03_l2norm", "phase9_gelu_row_dot"]


def inputs_of(meta, offset=0):
    return {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}


def forced_plan(ir):
    pkg = load_package(ir)
    tile = pkg.body[0]
    ev = _Eval(pkg)
    ev.smem = set()
    for a in tile.axes:
        ev.axes[a.name] = static_extent(a.extent)
    ev.run(tile.body)
    return compile_rowprog(pkg, tile, ev).to_json()


@pytest.mark.parametrize("name", REDUCTIONS)
def test_row_oracle_matches_golden(name):
    meta = golden_meta(name)
    got = rowprog_ir.evaluate(golden_ir(name), inputs_of(meta))
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]


@pytest.mark.parametrize("name", REDUCTIONS)
def test_fixed_reductions_as_row_programs(name):
    """The fixed classes, forced through the row compiler, reproduce their golden vectors."""
    plan = forced_plan(golden_ir(name))
    meta = golden_meta(name)
    got = pw_vm.run_rows(plan["params"]["program"], plan["params"]["layout"], inputs_of(meta))
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]


@pytest.mark.parametrize("name", sorted(W.ROW_SYNTHETIC))
def test_synthetic_row_program_matches_oracle(name, tmp_path):
    ir = W.ROW_SYNTHETIC[name](tmp_path / name)
    plan = compile_file(ir)
    assert plan["op"] == "rowprog"
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    for offset in (0, 2):
        arrays = inputs_of(meta, offset)
        ref = rowprog_ir.evaluate(ir, arrays)
        got = pw_vm.run_rows(plan["params"]["program"], plan["params"]["layout"], arrays)
        for key, value in ref.items():
            assert O.compare(got[key].reshape(value.shape), value, meta["rtol"], meta["atol"])["pass"]


def test_combine_program_is_the_one_the_tile_states(tmp_path):
    """Accumulating by max but combining by add is run as written (the
    thread-by-thread merge of the oracle agrees), not taken for a row max."""
    ir = W.ROW_SYNTHETIC["row_max"](tmp_path / "m")
    text = ir.read_text()
    ir.write_text(text.replace("Assign(name='m', op=ElementwiseImpl('maximum')",
                               "Assign(name='m', op=ElementwiseImpl('add')"))
    plan = compile_file(ir)
    assert plan["op"] == "rowprog"
    meta = json.loads((tmp_path / "m" / "meta.json").read_text())
    arrays = inputs_of(meta)
    got = pw_vm.run_rows(plan["params"]["program"], plan["params"]["layout"], arrays)
    x = arrays["x"].astype(np.float64)
    # 128 threads each take the max of their columns; the merge adds the maxima
    per_thread = np.stack([x[:, t::128].max(axis=1) for t in range(128)], axis=1)
    np.testing.assert_allclose(got["out"], per_thread.sum(axis=1), rtol=1e-5, atol=1e-5)


def test_row_outputs_not_covered_run_as_written(tmp_path):
    """An output the rows do not cover is no row program; the block program
    writes what the IR writes and leaves the rest as the runner filled it."""
    ir = W.row_package(tmp_path / "hole", "hole", 8, 64, {"x": ((8, 64), "f32")}, ("out", (9,), "f32"),
                       [W.load("xv", "x", [W.var("a0"), W.var("a1")], "f32")], [("s", "add", "xv")],
                       final_writes=[W.write("out", [W.var("a0")], ["s"], "f32")])
    plan = compile_file(ir)
    assert plan["op"] == "blockprog"
    from oracle import staged_ir
    meta = json.loads((tmp_path / "hole" / "meta.json").read_text())
    arrays = inputs_of(meta, 0)
    ref = staged_ir.evaluate(ir, arrays)["out"]
    got = pw_vm.run_block(plan["params"]["program"], plan["params"]["layout"], arrays)["out"]
    assert np.isnan(ref[8]) and np.isnan(got[8])
    np.testing.assert_allclose(got[:8], ref[:8], rtol=1e-5)


@pytest.mark.parametrize("name", sorted(W.ROW_COUPLED))
def test_online_softmax_variants_run_as_row_programs(name, tmp_path):
    """Coupled online states (Accum through a base, merged by the Tile's own
    combine statements) are not the fixed softmax when the output changes:
    they run as row programs that match the row oracle."""
    ir = W.ROW_COUPLED[name](tmp_path / name)
    plan = compile_file(ir)
    assert plan["op"] == "rowprog"
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    arrays = inputs_of(meta, 1)
    ref = rowprog_ir.evaluate(ir, arrays)
    got = pw_vm.run_rows(plan["params"]["program"], plan["params"]["layout"], arrays)
    for key, value in ref.items():
        assert O.compare(got[key].reshape(value.shape), value, 1e-5, 1e-6)["pass"]


def test_f02_as_row_program_matches_golden():
    plan = forced_plan(golden_ir("f02_row_softmax"))
    meta = golden_meta("f02_row_softmax")
    got = pw_vm.run_rows(plan["params"]["program"], plan["params"]["layout"], inputs_of(meta))
    with np.load(golden("f02_row_softmax") / "expected.npz") as z:
        assert O.compare(got["softmax"].reshape(z["softmax"].shape), z["softmax"], meta["rtol"], meta["atol"])["pass"]
