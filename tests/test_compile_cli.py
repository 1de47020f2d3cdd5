"""The drop-in CLI boundary: ``python compile.py kernel.ir.json`` (reference compile.py:8-19)."""
import json
import shutil
import subprocess
import sys

import pytest

from conftest import ROOT, golden, golden_ir
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.ir import CompileError, load_package, parse_body

CLI = [sys.executable, str(ROOT / "compile.py")]

EXPECTED = {
    "p00_scalar_add": ("add_f32", {"n": 128}),
    "p01_vector_add": ("add_f32", {"n": 1024}),
    "p02_scale_shift": ("axpb_f32", {"n": 4096}),
    "p03_relu_mul": ("relumul_f32", {"n": 2048}),
    "r01_array_sum": ("sum_f32", {"n": 1024}),
    "r02_big_sum": ("sum_f32", {"n": 65536}),
    "r03_mean": ("mean_f32", {"n": 32768}),
    "r04_row_sum": ("rowsum_f32", {"rows": 64, "cols": 512}),
    "f01_rmsnorm": ("rmsnorm_f32", {"rows": 64, "cols": 1024}),
    "f02_row_softmax": ("softmax_f32", {"rows": 64, "cols": 256}),
    "f03_l2norm": ("l2norm_f32", {"rows": 64, "cols": 512}),
    "phase9_gelu_erf_tail": ("gelu", {"n": 4099, "approximate": "none"}),
    "phase9_gelu_tanh_matrix": ("gelu", {"n": 2603, "approximate": "tanh"}),
    "phase9_gelu_erf_half": ("gelu", {"n": 1813, "approximate": "none"}),
    "phase9_gelu_tanh_half": ("gelu", {"n": 1031, "approximate": "tanh"}),
    "phase9_half_gelu_gemm": ("gemm", {"m": 17, "n": 21, "k": 33, "b_layout": "kn", "epilogue": "gelu_tanh"}),
    "generated_tensor": ("gemm", {"m": 11, "n": 19, "k": 7, "b_layout": "kn", "epilogue": "none"}),
    # FP32 contraction classes: staged (cp.async, split-K), serial and block-cooperative schedules
    # (every one states a tolerance, so the reference compensates its dot products: Dot2)
    "m01_matmul_512": ("gemm", {"m": 512, "n": 512, "k": 512, "b_layout": "kn", "epilogue": "none",
                                "compensated": True}),
    "m02_matmul_rect": ("gemm", {"m": 128, "n": 64, "k": 256, "b_layout": "kn", "epilogue": "none",
                                 "compensated": True}),
    "phase9_bias_gelu_gemm": ("gemm", {"m": 33, "n": 47, "k": 65, "b_layout": "kn", "epilogue": "gelu_erf",
                                       "compensated": True}),
    "a01_attention": ("attention_f32", {"bh": 1, "s_q": 64, "s_kv": 64, "d": 64, "dv": 64,
                                        "scale_mode": "mul_recip", "epilogue": "none", "compensated": True}),
    "a02_attention_128": ("attention_f32", {"bh": 1, "s_q": 128, "s_kv": 128, "d": 32, "dv": 32,
                                            "scale_mode": "mul_recip", "epilogue": "none", "compensated": True}),
    "phase9_gelu_attention": ("attention_f32", {"bh": 1, "s_q": 11, "s_kv": 37, "d": 17, "dv": 13,
                                                "scale_mode": "mul", "epilogue": "gelu_erf",
                                                "compensated": True}),
    "phase9_gelu_row_dot": ("rowdot_f32", {"rows": 19, "cols": 131, "activation": "gelu_erf"}),
    "fragment_attention_tile_f16": ("attention_tile_f16q", {"bh": 1, "s_q": 16, "s_kv": 16, "d": 16,
                                                            "dv": 8}),
    # one-warp m16n8k16 fragment programs (tests/test_tensor_cores.py fixtures)
    **{name: ("gemm_mixed", {"m": m, "n": n, "k": k, "b_layout": lay, "epilogue": epi, "transpose": tr,
                             "accumulate": acc})
       for name, (m, n, k, lay, epi, tr, acc) in {
           "tensor_atomic_f32": (16, 8, 16, "kn", "none", False, True),
           "tensor_cp_async_shared": (16, 8, 16, "kn", "none", False, False),
           "tensor_family_live_index": (32, 8, 16, "kn", "none", False, False),
           "tensor_fused_guarded_epilogue": (11, 7, 19, "kn", "relu", False, False),
           "tensor_global_bf16": (16, 8, 16, "kn", "none", False, False),
           "tensor_global_bf16_trans_ragged": (9, 7, 17, "nk", "none", False, False),
           "tensor_global_f16": (16, 8, 16, "kn", "none", False, False),
           "tensor_global_f16_ragged": (11, 7, 19, "kn", "none", False, False),
           "tensor_shared_b128": (16, 8, 16, "kn", "none", False, False),
           "tensor_shared_b32": (16, 8, 16, "kn", "none", False, False),
           "tensor_shared_b64": (16, 8, 16, "kn", "none", False, False),
           "tensor_shared_bf16_trans": (16, 8, 16, "nk", "none", False, False),
           "tensor_shared_f16": (16, 8, 16, "kn", "none", False, False),
           "tensor_shared_paired": (16, 16, 16, "kn", "none", False, False),
           "tensor_shared_paired_trans": (16, 16, 16, "nk", "none", False, False),
           "tensor_transposed_output": (16, 8, 16, "kn", "none", True, False),
       }.items()},
    "tensor_repack_f16": ("gemm_chain", {"m": 16, "k": 16, "n1": 16, "n2": 8, "y_layout": "kn",
                                         "z_layout": "kn"}),
    # GELU regression packages (examples/phase9/gelu): several typed results per element
    **{f"activation_gelu{t}_{k}": ("pointwise", {"out": "out", "points": 37 if k == "special" else 273})
       for t in ("", "_tanh") for k in ("f32", "f16", "bf16", "special")},
    "floating_f32_mod": ("pointwise", {"out": "out", "points": 528}),
    "floating_f32_remainder": ("pointwise", {"out": "out", "points": 528}),
    # fragment algebra (examples/phase9/fragments) as lane programs
    **{name: ("pointwise", {"points": 32, "lanes": True}) for name in (
        "fragment_family_row_softmax", "fragment_masked_gmem_post", "fragment_mma_row_normalization",
        "fragment_row_add_ordered", "fragment_row_maximum_ordered", "fragment_row_minimum_ordered",
        "fragment_row_multiply_ordered")},
}


@pytest.mark.parametrize("name", sorted(EXPECTED))
def test_cli_prints_plan(name):
    result = subprocess.run(CLI + [str(golden_ir(name))], capture_output=True, text=True, cwd=ROOT)
    assert result.returncode == 0, result.stderr
    plan = json.loads(result.stdout)
    op, params = EXPECTED[name]
    assert plan["op"] == op
    if op == "pointwise":   # the register program itself is checked in test_pointwise_programs.py
        assert {k: plan["params"][k] for k in params} == params
    else:
        assert plan["params"] == params
    assert plan["format"] == "lazyb200-plan/1"
    meta = json.loads((golden(name) / "meta.json").read_text())
    assert plan["arg_order"] == meta["kernels"][0]["arg_order"]
    assert plan["entry"] == meta["kernels"][0]["entry"]
    assert set(plan["bind"].values()) <= set(plan["arg_order"])


def test_cli_usage_exit_2():
    result = subprocess.run(CLI, capture_output=True, text=True, cwd=ROOT)
    assert result.returncode == 2 and result.stdout == ""
    assert "usage" in result.stderr


def test_cli_missing_file_exit_1(tmp_path):
    result = subprocess.run(CLI + [str(tmp_path / "nope.ir.json")], capture_output=True, text=True, cwd=ROOT)
    assert result.returncode == 1 and result.stdout == ""
    assert result.stderr.startswith("compile.py: ")


def test_cli_rejects_unsupported_classes_without_output(tmp_path):
    import pw_packages as W
    i = W.var("i")
    ir = W.package(tmp_path / "pow", "pow", {"x": ((64,), "f32")}, ("out", (64,), "f32"), [("i", 64)],
                   [W.load("v", "x", [i], "f32"), W.assign("p", "power", ["v", "v"], "f32"),
                    W.write("out", [i], ["p"], "f32")])
    result = subprocess.run(CLI + [str(ir)], capture_output=True, text=True, cwd=ROOT)
    assert result.returncode == 1
    assert result.stdout == ""
    assert result.stderr.startswith("compile.py: ")


def _copy(name, tmp_path):
    dst = tmp_path / name
    shutil.copytree(golden(name), dst)
    return dst, next(dst.glob("*.ir.json"))


def test_meta_entry_must_match_kernel_name(tmp_path):
    folder, ir = _copy("p01_vector_add", tmp_path)
    meta = json.loads((folder / "meta.json").read_text())
    meta["kernels"][0]["entry"] = "k_other"
    (folder / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(CompileError, match="no unique kernel entry"):
        compile_file(ir)


def test_arg_order_must_match_node_arguments(tmp_path):
    folder, ir = _copy("p01_vector_add", tmp_path)
    meta = json.loads((folder / "meta.json").read_text())
    meta["kernels"][0]["arg_order"] = meta["kernels"][0]["arg_order"][:-1]
    (folder / "meta.json").write_text(json.dumps(meta))
    with pytest.raises(CompileError, match="arg_order"):
        compile_file(ir)


def test_arg_order_permutation_is_honoured(tmp_path):
    folder, ir = _copy("p03_relu_mul", tmp_path)
    meta = json.loads((folder / "meta.json").read_text())
    meta["kernels"][0]["arg_order"] = list(reversed(meta["kernels"][0]["arg_order"]))
    (folder / "meta.json").write_text(json.dumps(meta))
    plan = compile_file(ir)
    assert plan["arg_order"] == meta["kernels"][0]["arg_order"]
    assert plan["bind"] == {"x": "x", "y": "y", "out": "mul"}


def test_unknown_constructor_is_rejected():
    with pytest.raises(CompileError, match="unsupported IR constructor"):
        parse_body("Tile(axes=(), body=(Evil(x=1),))")
    with pytest.raises(CompileError, match="plain name"):
        parse_body("__import__('os').system('true')")
    with pytest.raises(CompileError, match="unsupported IR syntax"):
        parse_body("[x for x in ()]")
    with pytest.raises(CompileError):
        parse_body("Tile(axes=(), body=(Load(names=('a',), input=x.y),))")


def test_corrupt_ir_is_a_compile_error(tmp_path):
    folder, ir = _copy("r01_array_sum", tmp_path)
    ir.write_text(ir.read_text()[:200])
    with pytest.raises(CompileError, match="invalid JSON"):
        compile_file(ir)


def test_modified_semantics_are_not_misrecognised(tmp_path):
    """A pointwise body whose op changes (add -> subtract) is not run as add: it
    compiles to a register program that subtracts."""
    import numpy as np
    import pw_vm
    folder, ir = _copy("p01_vector_add", tmp_path)
    ir.write_text(ir.read_text().replace("ElementwiseImpl('add')", "ElementwiseImpl('subtract')"))
    plan = compile_file(ir)
    assert plan["op"] == "pointwise"
    x0, x1 = (np.random.default_rng(s).standard_normal(1024).astype(np.float32) for s in (0, 1))
    out = pw_vm.run(plan["params"]["program"], {"x0": x0, "x1": x1})
    np.testing.assert_array_equal(out[plan["params"]["out"]], x0 - x1)


def test_gelu_constant_values_are_checked(tmp_path):
    """A GELU-shaped body with a wrong constant is not run as GELU: it compiles
    to a register program of the formula as written."""
    import numpy as np
    import pw_vm
    from oracle import expressions as O
    from oracle import pointwise_ir
    folder, ir = _copy("phase9_gelu_erf_tail", tmp_path)
    meta = json.loads((folder / "meta.json").read_text())
    for arg in meta["kernels"][0]["args"]:
        if arg["name"] == "gelu_half":
            arg["data"] = [0.25]
    (folder / "meta.json").write_text(json.dumps(meta))
    plan = compile_file(ir)
    assert plan["op"] == "pointwise"
    arrays = {a["name"]: O.input_array(a) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = pointwise_ir.evaluate(ir, arrays)
    got = pw_vm.run(plan["params"]["program"], arrays)
    for key, value in ref.items():
        assert O.compare(got[key].reshape(value.shape), value, 1e-5, 2e-6)["pass"]
        half = O.gelu(arrays["x"], "none", "f32") * np.float32(0.5)   # 0.25 x (1 + erf) = GELU / 2
        assert O.compare(got[key].reshape(value.shape), half.reshape(value.shape), 1e-5, 2e-6)["pass"]


def test_package_loader_reads_buffers():
    pkg = load_package(golden_ir("f01_rmsnorm"))
    assert pkg.entry == "k_mean_cbd1de"
    assert pkg.buffers["x"].shape == (64, 1024)
    assert pkg.buffers["mean_count"].role == "constant"
    assert pkg.rtol == 1e-3


def test_f32_plans_bind_bias_and_dtypes():
    plan = compile_file(golden_ir("phase9_bias_gelu_gemm"))
    assert plan["bind"] == {"a": "a", "b": "b", "bias": "bias", "c": "gelu"}
    assert plan["dtypes"] == {"ab": "f32", "c": "f32"}
    plan = compile_file(golden_ir("m02_matmul_rect"))
    assert plan["zero_outputs"] == ["matmul"]


def _mutate(name, tmp_path, old, new, count=None):
    folder, ir = _copy(name, tmp_path)
    text = ir.read_text()
    assert old in text
    ir.write_text(text.replace(old, new) if count is None else text.replace(old, new, count))
    return folder, ir


def test_staged_gemm_with_wrong_prefetch_distance_is_not_a_gemm(tmp_path):
    """Prefetching 64 instead of 128 columns ahead pairs stale shared-memory
    tiles: not a GEMM, so it runs as the block program it is."""
    _, ir = _mutate("m01_matmul_512", tmp_path, "Literal(value=128, dtype='int')",
                    "Literal(value=64, dtype='int')")
    plan = compile_file(ir)
    assert plan["op"] == "blockprog"


def test_split_k_without_zeroed_output_is_not_the_split_k_gemm(tmp_path):
    """Atomic partial sums into an output nobody zeroes are not the split-K
    GEMM (which relies on the zeroing); the block program adds into whatever
    the output holds, as the reference's kernel would."""
    folder, ir = _copy("m02_matmul_rect", tmp_path)
    meta = json.loads((folder / "meta.json").read_text())
    meta["kernels"][0]["zero_outputs"] = []
    (folder / "meta.json").write_text(json.dumps(meta))
    assert compile_file(ir)["op"] == "blockprog"


def test_attention_with_transposed_keys_is_not_attention(tmp_path):
    """kt indexed (key, dim) instead of (dim, key) leaves kt's bounds: no
    attention class or per-point program takes it (their indices are proved
    in range); the block program's loads are clamped into the buffer."""
    _, ir = _mutate("a02_attention_128", tmp_path, "input='kt', index=(Var(name='a2'), Var(name='a1'))",
                    "input='kt', index=(Var(name='a1'), Var(name='a2'))")
    assert compile_file(ir)["op"] == "blockprog"


def test_attention_with_min_instead_of_max_is_not_attention(tmp_path):
    """A running minimum in the online softmax is not the attention class; the
    block program runs the body as written (checked against the block oracle)."""
    import numpy as np
    import pw_vm
    from oracle import expressions as O
    from oracle import staged_ir
    folder, ir = _mutate("phase9_gelu_attention", tmp_path, "ElementwiseImpl('maximum')",
                         "ElementwiseImpl('minimum')")
    plan = compile_file(ir)
    assert plan["op"] == "blockprog"
    meta = json.loads((folder / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = staged_ir.evaluate(ir, arrays)
    got = pw_vm.run_block(plan["params"]["program"], plan["params"]["layout"], arrays)
    for key, value in ref.items():
        np.testing.assert_allclose(got[key].reshape(value.shape), value, rtol=1e-4, atol=1e-5, equal_nan=True)


def test_gemm_bias_on_the_wrong_axis_is_not_a_bias_gemm(tmp_path):
    """A bias indexed by the row is not the bias-GEMM class: the body runs as
    the row program it is (the row oracle on the same IR)."""
    import numpy as np
    import pw_vm
    from oracle import expressions as O
    from oracle import rowprog_ir
    folder, ir = _mutate("phase9_bias_gelu_gemm", tmp_path, "input='bias', index=(Var(name='a1'),)",
                         "input='bias', index=(Var(name='a0'),)")
    plan = compile_file(ir)
    assert plan["op"] == "rowprog"
    meta = json.loads((folder / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = rowprog_ir.evaluate(ir, arrays)
    got = pw_vm.run_rows(plan["params"]["program"], plan["params"]["layout"], arrays)
    for key, value in ref.items():
        assert O.compare(got[key].reshape(value.shape), value, 1e-4, 1e-5)["pass"]


def test_row_dot_with_changed_gelu_constant_is_not_gelu(tmp_path):
    """With a changed constant the body is no GELU row dot: it runs as the row
    program it is (the row oracle on the same IR)."""
    import numpy as np
    import pw_vm
    from oracle import expressions as O
    from oracle import rowprog_ir
    folder, ir = _copy("phase9_gelu_row_dot", tmp_path)
    meta = json.loads((folder / "meta.json").read_text())
    for arg in meta["kernels"][0]["args"]:
        if arg["name"] == "gelu_inv_sqrt2":
            arg["data"] = [0.5]
    (folder / "meta.json").write_text(json.dumps(meta))
    plan = compile_file(ir)
    assert plan["op"] == "rowprog"
    arrays = {a["name"]: O.input_array(a) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = rowprog_ir.evaluate(ir, arrays)
    got = pw_vm.run_rows(plan["params"]["program"], plan["params"]["layout"], arrays)
    for key, value in ref.items():
        assert O.compare(got[key].reshape(value.shape), value, 1e-4, 1e-5)["pass"]


def test_fragment_attention_without_exp_is_not_attention(tmp_path):
    """Without the exp the tile is no softmax: it runs as its own lane program."""
    import pw_vm
    _, ir = _mutate("fragment_attention_tile_f16", tmp_path, "post=(ElementwiseImpl('exp'),)", "post=()")
    pw_vm.assert_faithful(ir)


def test_fragment_attention_with_row_min_is_not_attention(tmp_path):
    import pw_vm
    _, ir = _mutate("fragment_attention_tile_f16", tmp_path,
                    "FragmentRowReduce(top='pivot0', bot='pivot1', frags=('scores[0]', 'scores[1]'), "
                    "op=ElementwiseImpl('maximum')",
                    "FragmentRowReduce(top='pivot0', bot='pivot1', frags=('scores[0]', 'scores[1]'), "
                    "op=ElementwiseImpl('minimum')")
    pw_vm.assert_faithful(ir, rtol=2e-3, atol=2e-3)
