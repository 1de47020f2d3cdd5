"""Recognition of the one-warp tensor-fragment programs (the reference's
tests/test_tensor_cores.py fixtures) by provenance interpretation, on CPU.

* every fixture's plan, evaluated by the oracle on the fixture's inputs,
  reproduces the fixture's expected output exactly;
* programs that compute something else — a swizzle applied on one side only,
  a missing barrier or cp.async wait, a stride that leaves the buffer, a guard
  that drops an element, a bias indexed by the row, a repack that swaps its
  halves, an atomic store into an output nobody zeroes — are rejected.
"""
import json
import shutil

import numpy as np
import pytest

from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.ir import CompileError
from oracle import expressions as O
import pw_vm

FIXTURES = sorted(p.name for p in golden("").iterdir() if p.name.startswith("tensor_"))


def test_fixture_list_is_complete():
    assert len(FIXTURES) == 17


@pytest.mark.parametrize("name", FIXTURES)
def test_plan_reproduces_fixture_output(name):
    plan = compile_file(golden_ir(name))
    meta = golden_meta(name)
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    got = O.evaluate(plan, arrays)
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            np.testing.assert_array_equal(got[key], z[key])


def mutated(tmp_path, name, old, new, meta_edit=None):
    dst = tmp_path / name
    shutil.copytree(golden(name), dst)
    ir = next(dst.glob("*.ir.json"))
    text = ir.read_text()
    assert old in text, old
    ir.write_text(text.replace(old, new))
    if meta_edit is not None:
        meta = json.loads((dst / "meta.json").read_text())
        meta_edit(meta)
        (dst / "meta.json").write_text(json.dumps(meta))
    return ir


def drop_zero_outputs(meta):
    meta["kernels"][0]["zero_outputs"] = []


MUTATIONS = {
    # the fill swizzles, the ldmatrix reads do not: odd rows read the other 8-column half
    "read_without_swizzle": ("tensor_shared_b32", "ldm=64, swizzle='B32', staged=True",
                             "ldm=64, swizzle='NONE', staged=True", None, "nothing wrote|contraction"),
    "missing_barrier": ("tensor_shared_f16", "Sync(barrier_id=0, count=None, warp=False), ", "", None,
                        "barrier"),
    "missing_cp_async_wait": ("tensor_cp_async_shared", "CpAsyncWait(group=0), ", "", None, "cp.async"),
    "b_stride_leaves_buffer": ("tensor_global_f16", "role='b', ldm=8,", "role='b', ldm=16,", None,
                               "outside"),
    "store_guard_drops_column": ("tensor_global_f16_ragged",
                                 "n_guard=(Literal(value=0, dtype='int'), Literal(value=7, dtype='int'))",
                                 "n_guard=(Literal(value=0, dtype='int'), Literal(value=6, dtype='int'))",
                                 None, "exactly once"),
    "atomic_without_zeroing": ("tensor_atomic_f32", "atomic=True", "atomic=True", drop_zero_outputs,
                               "zero_outputs"),
    "bias_by_row": ("tensor_fused_guarded_epilogue", "index=(Var(name='__N__'),)",
                    "index=(Var(name='__M__'),)", None, "output column"),
    "repack_swapped_halves": ("tensor_repack_f16", "srcs=('c0', 'c1')", "srcs=('c1', 'c0')", None,
                              "contraction"),
    "family_rows_not_advanced": ("tensor_family_live_index",
                                 "src_index=(BinaryExpr(op='*', left=Var(name='fi'), right=Literal(value=16, "
                                 "dtype='int')), Var(name='kk'))",
                                 "src_index=(Literal(value=0, dtype='int'), Var(name='kk'))", None,
                                 "row and column"),
}


STAGED = {"read_without_swizzle", "missing_barrier", "missing_cp_async_wait"}


@pytest.mark.parametrize("case", sorted(MUTATIONS))
def test_wrong_programs_are_not_misrecognised(case, tmp_path):
    """A changed program is never taken for the product it no longer computes.
    Programs that stage through shared memory are then rejected; the others
    run as lane programs that compute exactly what the changed IR says (the
    fragment oracle on the same IR)."""
    name, old, new, meta_edit, match = MUTATIONS[case]
    ir = mutated(tmp_path, name, old, new, meta_edit)
    if case in STAGED:
        with pytest.raises(CompileError, match=match):
            compile_file(ir)
        return
    from lazy_compiler_b200.recognize_frag import recognise_fragment_tile
    from lazy_compiler_b200.ir import load_package
    pkg = load_package(ir)
    with pytest.raises(CompileError, match=match):
        recognise_fragment_tile(pkg, pkg.body[0])
    pw_vm.assert_faithful(ir)


def test_second_store_of_paired_program_is_required(tmp_path):
    ir = next(golden("tensor_shared_paired").glob("*.ir.json"))
    text = ir.read_text()
    start = text.index(", RegStore(dst_buffer='out', dst_index=(Literal(value=0, dtype='int'), Literal(value=8")
    end = text.index("col_dim=1)", start) + len("col_dim=1)")
    dst = tmp_path / "tensor_shared_paired"
    shutil.copytree(golden("tensor_shared_paired"), dst)
    next(dst.glob("*.ir.json")).write_text(text[:start] + text[end:])
    with pytest.raises(CompileError, match="exactly once|shared memory"):
        compile_file(next(dst.glob("*.ir.json")))


FRAGMENT_ALGEBRA = sorted(p.name for p in golden("").iterdir()
                          if p.name.startswith("fragment_") and p.name != "fragment_attention_tile_f16")


@pytest.mark.parametrize("name", FRAGMENT_ALGEBRA)
def test_fragment_algebra_lane_program_matches_golden(name):
    """FragmentApply / FragmentRowReduce programs (examples/phase9/fragments) as lane programs."""
    plan = compile_file(golden_ir(name))
    assert plan["op"] == "pointwise" and plan["params"]["lanes"]
    meta = golden_meta(name)
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    got = pw_vm.run(plan["params"]["program"], arrays)
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            row = O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])
            assert row["pass"], row


@pytest.mark.parametrize("name", FRAGMENT_ALGEBRA + [f for f in FIXTURES if f not in (
    "tensor_cp_async_shared",) and not f.startswith("tensor_shared")])
def test_fragment_oracle_matches_golden(name):
    from oracle import fragment_ir
    meta = golden_meta(name)
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    got = fragment_ir.evaluate(golden_ir(name), arrays)
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]


@pytest.mark.parametrize("name", [f for f in FIXTURES if f != "tensor_cp_async_shared"
                                  and not f.startswith("tensor_shared")])
def test_tensor_fixtures_as_lane_programs(name):
    """The lane compiler also reproduces the tensor-core fixtures (gathers, MMA, repack, store variants)."""
    from lazy_compiler_b200.fragment_vm import compile_fragment_lanes
    from lazy_compiler_b200.ir import load_package
    pkg = load_package(golden_ir(name))
    plan = compile_fragment_lanes(pkg, pkg.body[0]).to_json()
    meta = golden_meta(name)
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    got = pw_vm.run(plan["params"]["program"], arrays)
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]
