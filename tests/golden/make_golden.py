"""Copies the reference's hot-path golden packages into tests/golden/packages.

Run in a container where the reference checkout exists:
    python tests/golden/make_golden.py /path/to/Lazy-Compiler

For every package listed in PACKAGES it copies the IR (``*.ir.json``), the
launch contract (``meta.json``) and the golden outputs (``expected.npz``) —
data files only, never source — and records the source path and SHA-256 of
each file in ``manifest.json``.  The GPU box has no reference checkout; the
tests read these copies.
"""
import hashlib
import json
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PACKAGES = [
    # public problems (problems/PROVENANCE.md)
    "problems/p00_scalar_add", "problems/p01_vector_add", "problems/p02_scale_shift",
    "problems/p03_relu_mul", "problems/r01_array_sum", "problems/r02_big_sum",
    "problems/r03_mean", "problems/r04_row_sum", "problems/f01_rmsnorm",
    "problems/f02_row_softmax", "problems/f03_l2norm", "problems/m01_matmul_512",
    "problems/m02_matmul_rect", "problems/a01_attention", "problems/a02_attention_128",
    # Emmy-generated GELU / tensor packages
    "examples/phase9/generated/phase9_gelu_erf_tail",
    "examples/phase9/generated/phase9_gelu_tanh_matrix",
    "examples/phase9/generated/phase9_gelu_erf_half",
    "examples/phase9/generated/phase9_gelu_tanh_half",
    "examples/phase9/generated/phase9_half_gelu_gemm",
    "examples/phase9/generated/phase9_bias_gelu_gemm",
    "examples/phase9/generated/phase9_gelu_attention",
    "examples/phase9/generated/phase9_gelu_row_dot",
    "examples/generated_tensor",
    # typed GELU fixtures (tests/test_gelu.py)
    "examples/phase9/gelu/activation_gelu_f32", "examples/phase9/gelu/activation_gelu_f16",
    "examples/phase9/gelu/activation_gelu_bf16", "examples/phase9/gelu/activation_gelu_tanh_f32",
    "examples/phase9/gelu/activation_gelu_tanh_f16", "examples/phase9/gelu/activation_gelu_tanh_bf16",
    "examples/phase9/gelu/activation_gelu_special", "examples/phase9/gelu/activation_gelu_tanh_special",
    # fragment attention tile (tests/test_fragment_rows.py)
    "examples/phase9/fragments/fragment_attention_tile_f16",
    # pointwise floor remainder of f32 bit patterns (phase8 remainder packages)
    "examples/phase8/remainder/floating_f32_mod", "examples/phase8/remainder/floating_f32_remainder",
    # fragment algebra: FragmentApply operand kinds, ordered row folds, MMA + row normalisation
    *[f"examples/phase9/fragments/{name}" for name in (
        "fragment_family_row_softmax", "fragment_masked_gmem_post", "fragment_mma_row_normalization",
        "fragment_row_add_ordered", "fragment_row_maximum_ordered", "fragment_row_minimum_ordered",
        "fragment_row_multiply_ordered")],
    # tensor-core lowering fixtures (tests/test_tensor_cores.py)
    *[f"examples/tensor/packages/{name}" for name in (
        "tensor_atomic_f32", "tensor_cp_async_shared", "tensor_family_live_index",
        "tensor_fused_guarded_epilogue", "tensor_global_bf16", "tensor_global_bf16_trans_ragged",
        "tensor_global_f16", "tensor_global_f16_ragged", "tensor_repack_f16", "tensor_shared_b128",
        "tensor_shared_b32", "tensor_shared_b64", "tensor_shared_bf16_trans", "tensor_shared_f16",
        "tensor_shared_paired", "tensor_shared_paired_trans", "tensor_transposed_output")],
]


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def main(reference: Path) -> None:
    out = HERE / "packages"
    manifest = {}
    for rel in PACKAGES:
        src = reference / rel
        dst = out / src.name
        dst.mkdir(parents=True, exist_ok=True)
        files = sorted(src.glob("*.ir.json")) + [src / "meta.json", src / "expected.npz"]
        manifest[src.name] = {"source": rel, "files": {}}
        for f in files:
            shutil.copyfile(f, dst / f.name)
            manifest[src.name]["files"][f.name] = sha256(f)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(f"{len(manifest)} packages -> {out}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py REFERENCE_CHECKOUT")
    main(Path(sys.argv[1]))
