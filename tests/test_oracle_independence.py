"""The IR oracles pin every golden package by what its IR says, not by the recogniser's plan.

``tests/ir_oracles.ir_oracle`` picks an oracle from the IR structure alone.
Every golden package's IR, evaluated that way on the reference's seeded
inputs, must reproduce the reference's expected.npz within the package's
tolerance — so the IR oracles themselves are pinned to every golden vector.
And a plan forced into the wrong fixed class (its formula from
``oracle.expressions.evaluate``) must disagree with the IR oracle: the check
the GPU parity tests make against the IR oracle catches a misclassification.
"""
import json

import numpy as np
import pytest

from conftest import GOLDEN, golden_ir, golden_meta
from ir_oracles import ir_oracle, supported
from lazy_compiler_b200.compiler import compile_file
from oracle import expressions as O

ALL = sorted(p.name for p in GOLDEN.iterdir() if (p / "expected.npz").exists())
# the reference documents this package's FP16 erf-GELU mismatches as its own retained failure
KNOWN_REFERENCE_FAILURES = {"phase9_gelu_erf_half"}


def inputs(name, offset=0):
    meta = golden_meta(name)
    return {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}


@pytest.mark.parametrize("name", ALL)
def test_ir_oracle_reproduces_the_golden_vectors(name):
    if name in ("m01_matmul_512",):
        pytest.skip("the lockstep simulation of a 512^3 staged matmul is too slow for the CPU suite")
    if not supported(golden_ir(name)):
        pytest.skip("no IR oracle for staged or multi-warp fragment programs (golden vectors and the "
                    "reference PTX pin them)")
    meta = golden_meta(name)
    got = ir_oracle(golden_ir(name), inputs(name))
    with np.load(GOLDEN / name / "expected.npz") as z:
        for key in z.files:
            row = O.compare(np.asarray(got[key]).reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])
            if name in KNOWN_REFERENCE_FAILURES:
                continue
            assert row["pass"], (name, key, row)


WRONG = [("f01_rmsnorm", {"op": "l2norm_f32"}), ("f03_l2norm", {"op": "softmax_f32"}),
         ("r03_mean", {"op": "sum_f32"}), ("r04_row_sum", {"op": "l2norm_f32"}),
         ("p02_scale_shift", {"op": "relumul_f32", "bind": {"x": "x", "y": "x"}}),
         ("phase9_gelu_erf_tail", {"params": {"approximate": "tanh"}}),
         ("f02_row_softmax", {"op": "l2norm_f32"})]


@pytest.mark.parametrize("name,change", WRONG)
def test_a_plan_forced_into_the_wrong_class_fails_the_ir_check(name, change):
    plan = compile_file(golden_ir(name))
    arrays = inputs(name, 1)
    meta = golden_meta(name)
    right = O.evaluate(plan, arrays, ir=golden_ir(name))
    wrong = json.loads(json.dumps(plan))
    for key, value in change.items():
        if isinstance(value, dict):
            wrong[key] = {**wrong[key], **value}
        else:
            wrong[key] = value
    bad = O.evaluate(wrong, arrays, ir=golden_ir(name))
    ref = ir_oracle(golden_ir(name), arrays)
    for key, value in ref.items():
        ok = O.compare(np.asarray(right[key]).reshape(value.shape), value, meta["rtol"], meta["atol"])["pass"]
        wrong_value = np.asarray(bad[key])
        caught = wrong_value.size != value.size or \
            not O.compare(wrong_value.reshape(value.shape), value, meta["rtol"], meta["atol"])["pass"]
        assert ok and caught, (name, key, ok, caught)
