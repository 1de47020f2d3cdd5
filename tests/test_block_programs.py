"""Block programs (any Tile body run statement for statement, one CTA per
block): the block oracle (oracle/staged_ir.py) against the reference's
golden vectors for the reductions, fused rows, attention and matmul
schedules; every such package compiled as a block program and run by the
numpy lockstep interpreter (tests/pw_vm.py) against the same vectors; the
host's checks on a program's branches, loops and barriers; and, with -m gpu,
the same programs through lc_blockprog."""
import ctypes

import numpy as np
import pytest

import pw_vm
from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200 import runtime
from lazy_compiler_b200.blockprog import compile_blockprog
from lazy_compiler_b200.ir import CompileError, load_package
from lazy_compiler_b200.pointwise import OP
from oracle import expressions as O
from oracle import staged_ir

BLOCK_PACKAGES = ["r01_array_sum", "r02_big_sum", "r03_mean", "r04_row_sum", "f01_rmsnorm", "f02_row_softmax",
                  "f03_l2norm", "phase9_gelu_row_dot", "phase9_gelu_attention", "phase9_bias_gelu_gemm",
                  "a02_attention_128", "m02_matmul_rect"]


def inputs_of(meta, offset=0):
    return {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}


def matches_golden(name, got):
    meta = golden_meta(name)
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            row = O.compare(np.asarray(got[key]).reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])
            assert row["pass"], (name, key, row)


@pytest.mark.parametrize("name", BLOCK_PACKAGES)
def test_block_oracle_matches_golden(name):
    matches_golden(name, staged_ir.evaluate(golden_ir(name), inputs_of(golden_meta(name))))


@pytest.mark.parametrize("name", BLOCK_PACKAGES)
def test_block_program_matches_golden(name):
    pkg = load_package(golden_ir(name))
    plan = compile_blockprog(pkg, pkg.body[0]).to_json()
    p = plan["params"]
    matches_golden(name, pw_vm.run_block(p["program"], p["layout"], inputs_of(golden_meta(name))))


def test_block_program_layout():
    pkg = load_package(golden_ir("f02_row_softmax"))
    plan = compile_blockprog(pkg, pkg.body[0]).to_json()
    lay = plan["params"]["layout"]
    assert lay["threads"] == 128 and lay["n_block_axes"] == 1 and len(lay["smem"]) == 2
    ops = {c[0] for c in plan["params"]["program"]["code"]}
    assert {OP["BAR"], OP["SHFL_XOR"], OP["SLB"], OP["SLE"], OP["LDS"], OP["STS"], OP["BRZ"]} <= ops


def test_barrier_in_a_condition_is_rejected():
    """A Sync inside a Cond is not reached by every thread: a compile error,
    never a program that could wait forever."""
    from pathlib import Path
    import pw_packages as W
    import tempfile
    with tempfile.TemporaryDirectory() as tmp:
        i = W.var("i")
        ir = W.package(Path(tmp) / "p", "cond_sync", {"x": ((256,), "f32")}, ("out", (256,), "f32"), [("i", 256)],
                       [W.load("xv", "x", [i], "f32"),
                        "Cond(cond=BinaryExpr(op='<', left=Var(name='i'), right=Literal(value=7, dtype='int')), "
                        "body=(Sync(barrier_id=0, count=None, warp=False),), else_body=())",
                        W.write("out", [i], ["xv"], "f32")])
        pkg = load_package(ir)
        tile = pkg.body[0]
        with pytest.raises(CompileError):
            compile_blockprog(pkg, tile)


def _program(code, n_regs=4, loops=()):
    return {"code": code, "consts": [0, 1, 5], "forms": [], "buffers": ["out"], "extents": [1, 32],
            "n_regs": n_regs, "sizes": [32], "loops": list(loops)}


@pytest.mark.parametrize("case", ["backward_branch", "bar_in_branch", "bar_in_thread_loop", "bad_smem"])
def test_host_rejects_unsafe_block_programs(case):
    """The library checks a block program before launching it: branches only
    forward, barriers outside branch regions and per-thread loops, shared
    arrays in range (no GPU needed: validation fails before any launch)."""
    BAR, BRZ, CONST, TID = OP["BAR"], OP["BRZ"], OP["CONST"], OP["TID"]
    if case == "backward_branch":
        code = [[CONST, 0, 0, 0, 0, 1], [BRZ, 0, 0, 0, 0, 0]]
        loops = ()
    elif case == "bar_in_branch":
        code = [[TID, 0, 0, 0, 0, 0], [BRZ, 0, 0, 0, 0, 3], [BAR, 0, 0, 0, 0, 0]]
        loops = ()
    elif case == "bar_in_thread_loop":
        # start from the thread index: the loop's range differs by thread
        code = [[TID, 0, 0, 0, 0, 0], [CONST, 1, 0, 0, 0, 1], [CONST, 2, 0, 0, 0, 2],
                [OP["SLB"], 0, 0, 2, 0, 0 | 5 << 4], [BAR, 0, 0, 0, 0, 0], [OP["SLE"], 0, 1, 2, 0, 0 | 3 << 4]]
        loops = (8,)
    else:
        code = [[CONST, 0, 0, 0, 0, 0], [OP["LDS"], 1, 0, 0, 0, 3]]
        loops = ()
    g = runtime.pw_program(_program(code, loops=loops))
    lay = runtime.bp_layout({"threads": 32, "n_block_axes": 1, "smem": [[0, 32]]})
    ptrs = (ctypes.c_void_p * runtime.PW_MAX_BUFFERS)(ctypes.c_void_p(16))
    lib = runtime.library()
    status = lib.lc_blockprog(ctypes.c_void_p(ctypes.addressof(g)), ctypes.c_void_p(ctypes.addressof(lay)),
                              ptrs, ctypes.c_void_p(0))
    assert status == -1  # LC_ERR_INVALID


@pytest.mark.gpu
@pytest.mark.parametrize("name", BLOCK_PACKAGES + ["m01_matmul_512", "a01_attention"])
def test_block_program_on_gpu(name, cuda_device):
    from test_gpu_lanes import run_plan
    pkg = load_package(golden_ir(name))
    plan = compile_blockprog(pkg, pkg.body[0]).to_json()
    meta = golden_meta(name)
    for offset in (0, 1):
        arrays = inputs_of(meta, offset)
        got = run_plan(plan, meta, arrays)
        if offset == 0:
            matches_golden(name, got)
        ref = staged_ir.evaluate(golden_ir(name), arrays)
        for key, value in ref.items():
            row = O.compare(got[key].reshape(value.shape), value, meta["rtol"], meta["atol"])
            assert row["pass"], (name, offset, key, row)


@pytest.mark.parametrize("name", sorted(__import__("pw_packages").BLOCK_SYNTHETIC))
def test_synthetic_block_program_matches_oracle(name, tmp_path):
    import json
    import pw_packages as W
    from lazy_compiler_b200.compiler import compile_file
    ir = W.BLOCK_SYNTHETIC[name](tmp_path / name)
    plan = compile_file(ir)
    assert plan["op"] == "blockprog"
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    for offset in (0, 2):
        arrays = inputs_of(meta, offset)
        ref = staged_ir.evaluate(ir, arrays)
        got = pw_vm.run_block(plan["params"]["program"], plan["params"]["layout"], arrays)
        for key, value in ref.items():
            assert not np.isnan(value).any()
            np.testing.assert_allclose(got[key].reshape(value.shape), value, rtol=1e-6, atol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(__import__("pw_packages").BLOCK_SYNTHETIC))
def test_synthetic_block_program_on_gpu(name, tmp_path, cuda_device):
    import json
    import pw_packages as W
    from lazy_compiler_b200.runner import run_package
    ir = W.BLOCK_SYNTHETIC[name](tmp_path / name)
    meta = json.loads((tmp_path / name / "meta.json").read_text())
    arrays = inputs_of(meta, 1)
    ref = staged_ir.evaluate(ir, arrays)
    got = run_package(ir.parent, inputs=arrays)
    for key, value in ref.items():
        np.testing.assert_allclose(np.asarray(got[key]).reshape(value.shape), value, rtol=1e-6, atol=1e-6)


def _nvrtc_available():
    try:
        from cuda.bindings import nvrtc  # noqa: F401
        return True
    except ImportError:
        return False


@pytest.mark.skipif(not _nvrtc_available(), reason="NVRTC is not installed")
@pytest.mark.parametrize("name", BLOCK_PACKAGES)
def test_native_translation_compiles(name):
    """Every golden package's block program, and its serial / pointwise plan,
    translates to CUDA C that NVRTC compiles for sm_100a (no GPU needed)."""
    from lazy_compiler_b200 import jit
    pkg = load_package(golden_ir(name))
    p = compile_blockprog(pkg, pkg.body[0]).to_json()["params"]
    cubin = jit.compile_cubin(jit.block_source(p["program"], p["layout"]))
    assert len(cubin) > 1000


@pytest.mark.skipif(not _nvrtc_available(), reason="NVRTC is not installed")
def test_native_translation_of_serial_and_pointwise_programs(tmp_path):
    import pw_packages as W
    from lazy_compiler_b200 import jit
    from lazy_compiler_b200.compiler import compile_file
    for name, build in list(W.SERIAL_SYNTHETIC.items()) + list(W.SYNTHETIC.items()):
        plan = compile_file(build(tmp_path / name))
        if plan["params"].get("lanes"):
            continue
        assert jit.point_cubin(plan["params"]["program"]) is not None, name


@pytest.mark.skipif(not _nvrtc_available(), reason="NVRTC is not installed")
@pytest.mark.parametrize("name", ["r04_row_sum", "f01_rmsnorm", "f02_row_softmax", "f03_l2norm",
                                  "phase9_gelu_row_dot"])
def test_native_translation_of_row_programs(name):
    from lazy_compiler_b200 import jit
    from lazy_compiler_b200.ir import static_extent
    from lazy_compiler_b200.recognize import _Eval
    from lazy_compiler_b200.rowprog import compile_rowprog
    pkg = load_package(golden_ir(name))
    tile = pkg.body[0]
    ev = _Eval(pkg)
    ev.smem = set()
    for axis in tile.axes:
        ev.axes[axis.name] = static_extent(axis.extent)
    ev.run(tile.body)
    p = compile_rowprog(pkg, tile, ev).to_json()["params"]
    assert jit.rows_cubin(p["program"], p["layout"]) is not None
