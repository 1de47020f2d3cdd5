"""Runs the reference's own compiler and keeps its PTX — TEST INFRASTRUCTURE ONLY.

    python oracle/ref_ptx.py REFERENCE_CHECKOUT

The reference (Lazy-Compiler) compiles an IR package to PTX with
``ptx_backend.compile_file`` (ptx_backend.py:1821-1876); it needs Emmy 0.3.11,
which is absent here, so ``oracle/emmy_shim`` stands in for the Emmy modules
it imports.  This script

1. imports the checkout's ``ptx_backend`` unchanged with the shim on the path;
2. compiles every IR of PACKAGES exactly as the reference CLI would
   (``compile_file(path)`` with its defaults);
3. checks the SHA-256 of each PTX text against every hash the reference
   recorded for that IR (``artifacts/validation/phase9/tensor/compatibility.json``
   ``current_ptx_sha256`` and ``artifacts/validation/phase9/checkout/verification.json``
   ``expected_ptx_sha256``; LF and CRLF forms), which pins the shim;
4. writes the PTX to ``oracle/_ref/ptx/<package>.ptx`` (not committed; it
   travels to the GPU box with the snapshot) and ``oracle/_ref/manifest.json``.

The PTX is only hashed here and, on the GPU, JIT-loaded and launched
(``tests/test_gpu_reference_ptx.py``); it is never parsed or edited.
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"

PACKAGES = [
    "problems/p00_scalar_add", "problems/p01_vector_add", "problems/p02_scale_shift",
    "problems/p03_relu_mul", "problems/r01_array_sum", "problems/r02_big_sum",
    "problems/r03_mean", "problems/r04_row_sum", "problems/f01_rmsnorm",
    "problems/f02_row_softmax", "problems/f03_l2norm", "problems/m01_matmul_512",
    "problems/m02_matmul_rect", "problems/a01_attention", "problems/a02_attention_128",
    "examples/phase9/generated/phase9_gelu_erf_tail",
    "examples/phase9/generated/phase9_gelu_tanh_matrix",
    "examples/phase9/generated/phase9_gelu_erf_half",
    "examples/phase9/generated/phase9_gelu_tanh_half",
    "examples/phase9/generated/phase9_half_gelu_gemm",
    "examples/phase9/generated/phase9_bias_gelu_gemm",
    "examples/phase9/generated/phase9_gelu_attention",
    "examples/phase9/generated/phase9_gelu_row_dot",
    "examples/generated_tensor",
    "examples/phase9/gelu/activation_gelu_f32", "examples/phase9/gelu/activation_gelu_f16",
    "examples/phase9/gelu/activation_gelu_bf16", "examples/phase9/gelu/activation_gelu_tanh_f32",
    "examples/phase9/gelu/activation_gelu_tanh_f16", "examples/phase9/gelu/activation_gelu_tanh_bf16",
    "examples/phase9/gelu/activation_gelu_special", "examples/phase9/gelu/activation_gelu_tanh_special",
    "examples/phase9/fragments/fragment_attention_tile_f16",
]


# This repository's own packages of the reference's Dot2 known-answer cases
# (tests/golden/make_precision.py), compiled by the reference the same way.
LOCAL_PACKAGES = ["precision_dot_product_and_sum_residual", "precision_dot_seed_false_slabs",
                  "precision_dot_nested_reset", "precision_dot_shuffle_snapshot",
                  "precision_dot_half_inputs_float_state", "precision_dot_standalone_initial_update",
                  "precision_dot_followed_by_explicit_base"]


def sha(text: str) -> str:
    return hashlib.sha256(text.encode("ascii")).hexdigest()


def recorded_hashes(reference: Path) -> dict:
    """IR path (relative) -> set of PTX SHA-256 values the reference recorded."""
    out: dict[str, set] = {}
    compat = reference / "artifacts/validation/phase9/tensor/compatibility.json"
    if compat.exists():
        for row in json.loads(compat.read_text())["rows"]:
            out.setdefault(row["path"], set()).add(row["current_ptx_sha256"])
    verify = reference / "artifacts/validation/phase9/checkout/verification.json"
    if verify.exists():
        for row in json.loads(verify.read_text())["fresh_cli_checks"]:
            out.setdefault(row["ir"], set()).add(row["expected_ptx_sha256"])
    return out


def main(reference: Path) -> int:
    sys.path.insert(0, str(HERE / "emmy_shim"))
    sys.path.insert(0, str(reference))
    import ptx_backend  # the reference compiler, unchanged

    recorded = recorded_hashes(reference)
    (OUT / "ptx").mkdir(parents=True, exist_ok=True)
    manifest = {}
    failures = 0
    golden = HERE.parent / "tests" / "golden" / "packages"
    for rel in PACKAGES + [f"local:{name}" for name in LOCAL_PACKAGES]:
        folder = golden / rel[6:] if rel.startswith("local:") else reference / rel
        (ir,) = sorted(folder.glob("*.ir.json"))
        name = folder.name
        row = {"source": f"{rel}/{ir.name}"}
        try:
            ptx = ptx_backend.compile_file(ir)
        except Exception as exc:  # a package the reference itself rejects
            row["error"] = f"{type(exc).__name__}: {exc}"
            manifest[name] = row
            print(f"{name}: reference compile error: {row['error']}")
            continue
        lf, crlf = sha(ptx), sha(ptx.replace("\n", "\r\n"))
        want = recorded.get(f"{rel}/{ir.name}", set())
        row.update(sha256=lf, sha256_crlf=crlf, bytes=len(ptx), recorded=sorted(want),
                   identical=bool(want) and (lf in want or crlf in want),
                   meta=json.loads((folder / "meta.json").read_text()))
        if want and not row["identical"]:
            failures += 1
        (OUT / "ptx" / f"{name}.ptx").write_text(ptx)
        manifest[name] = row
        status = "IDENTICAL" if row["identical"] else ("no record" if not want else "DIFFERENT")
        print(f"{name}: {status}")
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    checked = sum(1 for r in manifest.values() if r.get("recorded"))
    same = sum(1 for r in manifest.values() if r.get("identical"))
    print(f"{same}/{checked} recorded hashes reproduced; {len(manifest)} packages written")
    return 1 if failures else 0


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python oracle/ref_ptx.py REFERENCE_CHECKOUT")
    sys.exit(main(Path(sys.argv[1]).resolve()))
