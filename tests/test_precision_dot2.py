"""Compensated dot accumulation (Dot2) on the reference's exact-cancellation cases, on CPU.

The reference compiles an f32 dot accumulation as Dot2 whenever meta.json
states a tolerance (ptx_backend.py:571-593, policy :1860-1865) and pins it
with exact-integer identities (tests/test_precision.py:39-188).  The seven
cases are packaged by tests/golden/make_precision.py; here each is compiled
by this backend and its register program interpreted in numpy
(tests/pw_vm.py): the result must equal the exact integers bit for bit.
Without compensation five of them lose the identity, so a plain f32
accumulation fails this test.  The eligibility rule is also checked on the
reference's two negative cases (a dot read by a Select or by a nested loop
bound is not compensated) and on the golden packages it names.
"""
import json

import numpy as np
import pytest

import pw_vm
from conftest import GOLDEN
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.dot2 import compensated_states
from lazy_compiler_b200.ir import load_package, parse_body
from oracle import expressions as O

PRECISION = sorted(p.name for p in GOLDEN.glob("precision_*"))


def run_plan(plan, meta):
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    prog = plan["params"]["program"]
    if plan["op"] == "blockprog":
        return pw_vm.run_block(prog, plan["params"]["layout"], arrays)
    return pw_vm.run(prog, arrays)


def test_all_seven_cases_are_packaged():
    assert len(PRECISION) == 7


@pytest.mark.parametrize("name", PRECISION)
def test_precision_case_is_exact(name):
    folder = GOLDEN / name
    (ir,) = folder.glob("*.ir.json")
    meta = json.loads((folder / "meta.json").read_text())
    assert meta["rtol"] > 0 and meta["atol"] > 0      # the reference's default policy compensates
    plan = compile_file(ir)
    got = run_plan(plan, meta)
    with np.load(folder / "expected.npz") as z:
        want = z["out"]
    np.testing.assert_array_equal(got["out"].reshape(want.shape), want)


@pytest.mark.parametrize("name", PRECISION)
def test_ir_oracles_reproduce_the_known_answers(name):
    """The serial / staged IR oracles (their own Dot2 restatement, oracle/dot2_ir.py) are exact too."""
    from oracle import serial_ir, staged_ir
    folder = GOLDEN / name
    (ir,) = folder.glob("*.ir.json")
    meta = json.loads((folder / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    oracle = staged_ir if compile_file(ir)["op"] == "blockprog" else serial_ir
    got = oracle.evaluate(ir, arrays)
    with np.load(folder / "expected.npz") as z:
        want = z["out"]
    np.testing.assert_array_equal(got["out"].reshape(want.shape), want)


def test_zero_tolerance_turns_compensation_off(tmp_path):
    """With rtol = atol = 0 the reference does not compensate, and neither does this backend."""
    import shutil
    src = GOLDEN / "precision_dot_product_and_sum_residual"
    dst = tmp_path / src.name
    shutil.copytree(src, dst)
    meta = json.loads((dst / "meta.json").read_text())
    meta["rtol"] = meta["atol"] = 0
    (dst / "meta.json").write_text(json.dumps(meta))
    (ir,) = dst.glob("*.ir.json")
    pkg = load_package(ir)
    assert compensated_states(pkg.body, pkg) == set()
    got = run_plan(compile_file(ir), meta)["out"]
    assert not np.array_equal(got, [1, 1, 1, 1, 1, 2, 3, 4])   # plain f32 loses the identities


F32 = "DataType(name='f32', np=dtype('float32'), nbytes=4)"
DOT = (f"Load(names=('a',), input='x', index=(Var(name='i'), Var(name='k')), dtype={F32}), "
       f"Load(names=('b',), input='y', index=(Var(name='i'), Var(name='k')), dtype={F32}), "
       f"Assign(name='product', op=ElementwiseImpl('multiply'), args=('a', 'b'), dtype={F32}), "
       f"Accum(name='dot', value='product', op=ElementwiseImpl('add'), dtype={F32}, axes=('k',), base=None)")


def loop(extra=""):
    return parse_body(f"Loop(axis=Axis(name='k', extent=Dim(4), window=None), body=({DOT}{extra}), "
                      f"unroll=False, seed=True)")


def test_plain_dot_is_eligible():
    assert compensated_states((loop(),)) == {"dot"}


def test_dot_read_by_select_is_not_compensated():
    from lazy_compiler_b200.ir import Node
    branch = Node("SelectBranch", (("value", "dot"), ("select", Node("Literal", (("value", True), ("dtype", "int"))))))
    sel = Node("Select", (("name", "selected"), ("branches", (branch,))))
    base = loop()
    body = Node("Loop", tuple((k, v + (sel,)) if k == "body" else (k, v) for k, v in base.fields))
    assert "dot" not in compensated_states((body,))


def test_dot_read_by_nested_loop_bound_is_not_compensated():
    nested = (", StridedLoop(axis=Axis(name='j', extent=Dim(4), window=None), start=Literal(value=0, "
              "dtype='int'), step=Literal(value=1, dtype='int'), body=(), unroll=False, end=Var(name='dot'), "
              "seed=True)")
    assert "dot" not in compensated_states((loop(nested),))


def test_golden_packages_compensated_as_the_reference_does():
    """Tolerance-bearing packages whose dots the reference compensates."""
    want = {"a01_attention", "a02_attention_128", "f01_rmsnorm", "f03_l2norm", "m01_matmul_512",
            "m02_matmul_rect", "phase9_bias_gelu_gemm", "phase9_gelu_attention", "phase9_gelu_row_dot"}
    got = set()
    for folder in GOLDEN.iterdir():
        if folder.name.startswith("precision_"):
            continue
        (ir,) = folder.glob("*.ir.json")
        pkg = load_package(ir)
        if compensated_states(pkg.body, pkg):
            got.add(folder.name)
    assert got == want
