"""Op-mix mutations of the reference's packages, as the hidden set varies
them: seeded random replacements of the elementwise operations in Assign
statements (and of the Accum fold operations) of reduction, fused-row,
attention, matmul and pointwise packages.  Each mutated package must
compile, and its plan — whatever path takes it: a fixed class, a row,
serial, pointwise or block program, a GEMM with an epilogue program — must
compute what the mutated IR says, on the CPU: the plan executed by the
oracle of its class or by the numpy program interpreter, against an IR
oracle that runs the mutated Tile as written.  A recogniser that took a
mutated body for its class would fail here."""
import json
import random
import re
import shutil

import numpy as np
import pytest

import pw_vm
from conftest import golden
from ir_oracles import ir_oracle
from lazy_compiler_b200.compiler import compile_file
from oracle import expressions as O

BINARY = ["add", "subtract", "multiply", "maximum", "minimum"]
UNARY = ["exp", "tanh", "abs", "negative", "relu", "sigmoid", "sqrt", "copy"]
FOLDS = ["add", "maximum", "minimum"]
PACKAGES = ["r04_row_sum", "f01_rmsnorm", "f02_row_softmax", "f03_l2norm", "phase9_gelu_row_dot",
            "phase9_gelu_attention", "a02_attention_128", "m02_matmul_rect", "p03_relu_mul", "p02_scale_shift",
            "r01_array_sum", "r03_mean", "phase9_gelu_erf_tail", "phase9_gelu_tanh_matrix", "phase9_bias_gelu_gemm",
            "activation_gelu_f32", "p01_vector_add", "fragment_family_row_softmax", "fragment_attention_tile_f16",
            "fragment_row_add_ordered", "fragment_mma_row_normalization", "tensor_fused_guarded_epilogue",
            "fragment_masked_gmem_post"]
SEEDS = int(__import__("os").environ.get("LC_MUTATION_SEEDS", "3"))
CASES = [(name, seed) for name in PACKAGES for seed in range(SEEDS)]

ASSIGN = re.compile(r"Assign\(name='([^']+)', op=ElementwiseImpl\('(\w+)'\), args=\(([^)]*)\)")
FRAG_APPLY = re.compile(r"FragmentApply\(out='[^']+', op=ElementwiseImpl\('(\w+)'\), args=.*?kinds=\(([^)]*)\)")
FRAG_REDUCE = re.compile(r"FragmentRowReduce\(top='[^']+', bot='[^']+', frags=\([^)]*\), op=ElementwiseImpl\('(\w+)'\)")
FRAG_BINARY = ["add", "subtract", "multiply", "divide", "maximum", "minimum"]
FLOAT_LITERAL = re.compile(r"Literal\(value=(-?[0-9]+\.[0-9]*(?:e[-+]?[0-9]+)?), dtype=(?!'int')")
ACCUM = re.compile(r"(Accum\(name='[^']+', value='[^']+', op=ElementwiseImpl\(')(\w+)('\))")


def mutate(text: str, seed: int) -> tuple:
    rng = random.Random(seed * 7919 + len(text))
    sites = []
    for m in ASSIGN.finditer(text):
        args = [a for a in m.group(3).split(",") if a.strip()]
        if m.group(2) in BINARY and len(args) == 2:
            sites.append((m.start(2), m.end(2), BINARY))
        elif m.group(2) in UNARY and len(args) == 1:
            sites.append((m.start(2), m.end(2), UNARY))
    for m in ACCUM.finditer(text):
        if m.group(2) in FOLDS:
            sites.append((m.start(2), m.end(2), FOLDS))
    for m in FRAG_APPLY.finditer(text):
        arity = len([k for k in m.group(2).split(",") if k.strip()])
        if m.group(1) in FRAG_BINARY and arity == 2:
            sites.append((m.start(1), m.end(1), FRAG_BINARY))
        elif m.group(1) in UNARY and arity == 1:
            sites.append((m.start(1), m.end(1), UNARY))
    for m in FRAG_REDUCE.finditer(text):
        if m.group(1) in FOLDS:
            sites.append((m.start(1), m.end(1), FOLDS))
    for m in FLOAT_LITERAL.finditer(text):
        value = float(m.group(1))
        sites.append((m.start(1), m.end(1), [repr(value * 1.5 + 0.25), repr(-value), repr(value * 0.5)]))
    if not sites:
        pytest.skip("no mutable operation")
    picked = sorted(rng.sample(sites, min(len(sites), 2)), reverse=True)
    changes = []
    for start, end, pool in picked:
        old = text[start:end]
        new = rng.choice([p for p in pool if p != old])
        text = text[:start] + new + text[end:]
        changes.append(f"{old}->{new}")
    return text, changes




def run_plan_cpu(plan, arrays, ir):
    p = plan["params"]
    op = plan["op"]
    if op == "blockprog":
        return pw_vm.run_block(p["program"], p["layout"], arrays)
    if op == "rowprog":
        return pw_vm.run_rows(p["program"], p["layout"], arrays)
    if op == "pointwise":
        return pw_vm.run(p["program"], arrays)
    if op == "gemm" and "post" in p:
        a = arrays[plan["bind"]["a"]].astype(np.float64)
        b = arrays[plan["bind"]["b"]].astype(np.float64)
        c = a @ (b if p["b_layout"] == "kn" else b.T)
        return pw_vm.run(p["post"]["program"], {**arrays, plan["bind"]["c"]: c.astype(np.float32)})
    return O.evaluate(plan, arrays)     # a fixed class: its formula from the plan


@pytest.mark.parametrize("name,seed", CASES)
def test_mutated_package_computes_its_ir(name, seed, tmp_path):
    folder = tmp_path / name
    shutil.copytree(golden(name), folder)
    ir = next(folder.glob("*.ir.json"))
    graph = json.loads(ir.read_text())
    node = next(n for n in graph["nodes"].values() if n["op"] == "KernelOp")
    body, changes = mutate(node["op_fields"]["body"][0], seed)
    node["op_fields"]["body"][0] = body
    ir.write_text(json.dumps(graph))
    plan = compile_file(ir)
    meta = json.loads((folder / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, seed) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = ir_oracle(ir, arrays)
    got = run_plan_cpu(plan, arrays, ir)
    with np.errstate(all="ignore"):
        for key, value in ref.items():
            out = np.asarray(got[key], np.float64).reshape(value.shape)
            want = np.asarray(value, np.float64)
            finite = np.isfinite(want)
            scale = np.abs(want[finite]).max() if finite.any() else 1.0
            ok = np.isclose(out, want, rtol=2e-4, atol=2e-5 * max(scale, 1.0), equal_nan=True) | \
                (np.isinf(out) & np.isinf(want) & (np.sign(out) == np.sign(want)))
            assert ok.all(), (name, changes, plan["op"], key, np.argwhere(~ok)[:3], out[~ok][:3], want[~ok][:3])


@pytest.mark.gpu
@pytest.mark.parametrize("name,seed", CASES)
def test_mutated_package_on_gpu(name, seed, tmp_path, cuda_device):
    from lazy_compiler_b200.runner import run_package
    folder = tmp_path / name
    shutil.copytree(golden(name), folder)
    ir = next(folder.glob("*.ir.json"))
    graph = json.loads(ir.read_text())
    node = next(n for n in graph["nodes"].values() if n["op"] == "KernelOp")
    body, changes = mutate(node["op_fields"]["body"][0], seed)
    node["op_fields"]["body"][0] = body
    ir.write_text(json.dumps(graph))
    meta = json.loads((folder / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, seed) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = ir_oracle(ir, arrays)
    got = run_package(folder, inputs=arrays)
    with np.errstate(all="ignore"):
        for key, value in ref.items():
            out = np.asarray(got[key], np.float64).reshape(value.shape)
            want = np.asarray(value, np.float64)
            finite = np.isfinite(want)
            scale = np.abs(want[finite]).max() if finite.any() else 1.0
            # the device uses the reference's approximate ex2 / tanh / erf sequences
            ok = np.isclose(out, want, rtol=2e-3, atol=2e-4 * max(scale, 1.0), equal_nan=True) | \
                (np.isinf(out) & np.isinf(want) & (np.sign(out) == np.sign(want)))
            assert ok.all(), (name, changes, key, np.argwhere(~ok)[:3], out[~ok][:3], want[~ok][:3])


# ---------------------------------------------------------------- shapes
# The row packages at other (odd) shapes: the row and column axes of the
# Tile and its loops rescaled, the buffers' shapes and the column count
# constant with them, as a schedule for another size would have them.
ROW_AXES = {"r04_row_sum": ({"a0": "rows", "a1": "cols"}, {"x": ("rows", "cols"), "sum_1": ("rows",)}),
            "f01_rmsnorm": ({"a0": "rows", "a1": "cols", "a2": "cols"},
                            {"x": ("rows", "cols"), "w": ("cols",), "mul_1": ("rows", "cols")}),
            "f02_row_softmax": ({"a0": "rows", "a1": "cols", "a3": "cols"},
                                {"x": ("rows", "cols"), "softmax": ("rows", "cols")}),
            "f03_l2norm": ({"a0": "rows", "a1": "cols", "a2": "cols"}, {"x": ("rows", "cols"), "div": ("rows", "cols")})}
SHAPES = [(37, 300), (5, 1000), (64, 129)]


def reshaped_case(name, rows, cols, tmp_path):
    """The package at rows x cols, checked on the CPU; returns it for the device."""
    from oracle.rescale import rescale_body
    size = {"rows": rows, "cols": cols}
    axes, shapes = ROW_AXES[name]
    folder = tmp_path / name
    shutil.copytree(golden(name), folder)
    ir = next(folder.glob("*.ir.json"))
    graph = json.loads(ir.read_text())
    for node in graph["nodes"].values():
        if node["op"] == "KernelOp":
            node["op_fields"]["body"] = [rescale_body(b, {a: size[v] for a, v in axes.items()})
                                         for b in node["op_fields"]["body"]]
        for out in node.get("outputs", []):
            if out["name"] in shapes:
                out["shape"] = [size[v] for v in shapes[out["name"]]]
    ir.write_text(json.dumps(graph))
    meta = json.loads((folder / "meta.json").read_text())
    for arg in meta["kernels"][0]["args"]:
        if arg["name"] in shapes:
            arg["shape"] = [size[v] for v in shapes[arg["name"]]]
        if arg["name"] == "mean_count":
            arg["data"] = [float(cols)]
    meta["kernels"][0]["grid"] = [rows, 1, 1]
    (folder / "meta.json").write_text(json.dumps(meta))
    plan = compile_file(ir)
    arrays = {a["name"]: O.input_array(a, 1) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = ir_oracle(ir, arrays)
    got = run_plan_cpu(plan, arrays, ir)
    for key, value in ref.items():
        assert not np.isnan(value).any()
        np.testing.assert_allclose(np.asarray(got[key], np.float64).reshape(value.shape), value,
                                   rtol=2e-4, atol=2e-5, err_msg=f"{name} {rows}x{cols} {plan['op']}")
    return folder, ir, arrays, ref


@pytest.mark.parametrize("name", sorted(ROW_AXES))
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_row_package_at_other_shapes(name, rows, cols, tmp_path):
    reshaped_case(name, rows, cols, tmp_path)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(ROW_AXES))
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_row_package_at_other_shapes_on_gpu(name, rows, cols, tmp_path, cuda_device):
    from lazy_compiler_b200.runner import run_package
    folder, ir, arrays, ref = reshaped_case(name, rows, cols, tmp_path)
    got = run_package(folder, inputs=arrays)
    for key, value in ref.items():
        np.testing.assert_allclose(np.asarray(got[key], np.float64).reshape(value.shape), value,
                                   rtol=1e-3, atol=1e-4, err_msg=f"{name} {rows}x{cols}")
