"""Rescaled copies of the reference's public IR packages at the BASELINE sizes — TEST INFRASTRUCTURE.

    python oracle/rescale.py REFERENCE_CHECKOUT

Emmy (absent here) would schedule new IR for new shapes; instead each public
package is copied with only its extents changed — the Tile / loop axis
extents in the KernelOp body, the tensor shapes of the graph and meta.json,
the meta grid (same block size, so the same per-thread schedule), and the
count constants that depend on the size.  The rescaled packages go to
``oracle/_ref/rescaled/<name>/`` and the reference's own compiler (unchanged,
through ``oracle/emmy_shim``) emits their PTX to
``oracle/_ref/ptx_rescaled/<name>.ptx``; ``manifest_rescaled.json`` records
hashes and meta.  These are labelled "rescaled" wherever they are used.
"""
from __future__ import annotations

import hashlib
import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
N28, N24 = 1 << 28, 1 << 24
ROWS, COLS = 16384, 4096
GEMM = 8192
SLICE, HEAD, KEYS = 512, 128, 4096

# name: (source package, {axis name: new extent}, {buffer: new shape}, grid x, {constant: value}
#        [, {integer literal of the index arithmetic: new value} [, {exact text: replacement}
#          [, {"block": threads per CTA, "dtypes": {buffer: storage type of its graph tensor and Loads}}]]])
PLAN = {
    "r02_big_sum": ("problems/r02_big_sum", {"a0": N24}, {"x": [N24]}, 1, {}),
    "r03_mean": ("problems/r03_mean", {"a0": N24}, {"x": [N24]}, 1, {"mean_keepdim_count": float(N24)}),
    "p01_vector_add": ("problems/p01_vector_add", {"a0": N28 // 2}, {"x0": [N28], "x1": [N28], "add": [N28]},
                       N28 // 2 // 256, {}),
    "p02_scale_shift": ("problems/p02_scale_shift", {"a0": N28 // 4}, {"x": [N28], "add": [N28]},
                        N28 // 4 // 256, {"mul_c1": 1.5, "add_c1": -0.25}),
    "p03_relu_mul": ("problems/p03_relu_mul", {"a0": N28 // 4}, {"x": [N28], "y": [N28], "mul": [N28]},
                     N28 // 4 // 256, {}),
    "phase9_gelu_erf_tail": ("examples/phase9/generated/phase9_gelu_erf_tail", {"a0": N28},
                             {"x": [N28], "gelu": [N28]}, N28 // 256, {}),
    "phase9_gelu_tanh_matrix": ("examples/phase9/generated/phase9_gelu_tanh_matrix", {"a0": N28},
                                {"x": [N28 // COLS, COLS], "gelu": [N28 // COLS, COLS]}, N28 // 256, {},
                                {137: COLS}),
    # the reference's mma.sync GEMM (m16n8k16 fragments, 16 warps of 128 x 32, tanh-GELU
    # epilogue, f16 out): the odd extents 17 / 21 / 33 occur only as the M and N guards,
    # the K extent and zero-fill bound and the leading dimensions, so they all become 8192;
    # the block axes a0_b / a1_b count 1024-row / 64-column blocks
    "phase9_half_gelu_gemm": ("examples/phase9/generated/phase9_half_gelu_gemm",
                              {"a0_b": GEMM // 1024, "a0": GEMM, "a1_b": GEMM // 64, "a1": GEMM, "a2": GEMM},
                              {"a": [GEMM, GEMM], "b": [GEMM, GEMM], "gelu": [GEMM, GEMM]},
                              (GEMM // 1024) * (GEMM // 64), {}, {17: GEMM, 21: GEMM, 33: GEMM},
                              {"ldm=33,": f"ldm={GEMM},", "ldm=21,": f"ldm={GEMM},"}),
    # the reference's scalar FP32 attention (a02: one CTA per query row, a thread per value
    # column, each thread recomputing every score) at the SDPA head size D = 128 over 4096
    # keys, with f16 loads of Q, Kt and V (f32 arithmetic), on a slice of 512 query rows of
    # one head; the only other literal, 32, is the always-zero a5_b block index's stride
    "a02_attention_f16_slice": ("problems/a02_attention_128",
                                {"a0_b": SLICE, "a0": SLICE, "a5": HEAD, "a5_u": HEAD, "a1": KEYS, "a2": HEAD},
                                {"q": [SLICE, HEAD], "kt": [HEAD, KEYS], "v": [KEYS, HEAD], "matmul_1": [SLICE, HEAD]},
                                SLICE, {"div_c1": float(np.float32(HEAD ** 0.5))}, {32: HEAD},
                                {"block_threads=32,": f"block_threads={HEAD},"},
                                {"block": HEAD, "dtypes": {"q": "f16", "kt": "f16", "v": "f16"}}),
    "r04_row_sum": ("problems/r04_row_sum", {"a0": ROWS, "a1": COLS}, {"x": [ROWS, COLS], "sum_1": [ROWS]},
                    ROWS, {}),
    "f01_rmsnorm": ("problems/f01_rmsnorm", {"a0": ROWS, "a1": COLS, "a2": COLS},
                    {"x": [ROWS, COLS], "w": [COLS], "mul_1": [ROWS, COLS]}, ROWS,
                    {"mean_count": float(COLS), "add_c1": 1e-6}),
    "f02_row_softmax": ("problems/f02_row_softmax", {"a0": ROWS, "a1": COLS, "a3": COLS},
                        {"x": [ROWS, COLS], "softmax": [ROWS, COLS]}, ROWS, {}),
    "f03_l2norm": ("problems/f03_l2norm", {"a0": ROWS, "a1": COLS, "a2": COLS},
                   {"x": [ROWS, COLS], "div": [ROWS, COLS]}, ROWS, {}),
}


def rescale_body(text: str, axes: dict) -> str:
    for axis, extent in axes.items():
        text, count = re.subn(rf"Axis\(name='{axis}', extent=Dim\(\d+\)", f"Axis(name='{axis}', extent=Dim({extent})", text)
        if count == 0:
            raise ValueError(f"axis {axis} not found")
    return text


def rescale_literals(text: str, literals: dict) -> str:
    for old, new in literals.items():
        text, count = re.subn(rf"Literal\(value={old}, dtype='int'\)", f"Literal(value={new}, dtype='int')", text)
        if count == 0:
            raise ValueError(f"integer literal {old} not found")
    return text


_DTYPE = {"f32": "DataType(name='f32', np=dtype('float32'), nbytes=4)",
          "f16": "DataType(name='f16', np=dtype('float16'), nbytes=2)"}


def retype_loads(text: str, dtypes: dict) -> str:
    """Give every Load of the named buffers the new storage type (its last field)."""
    for buf, dt in dtypes.items():
        at, count = 0, 0
        while True:
            i = text.find(f"input='{buf}', index=", at)
            if i < 0:
                break
            j = text.index("dtype=DataType(", i)
            end = text.index(")", text.index("nbytes=", j)) + 1
            text = text[:j] + "dtype=" + _DTYPE[dt] + text[end:]
            at, count = j + 1, count + 1
        if count == 0:
            raise ValueError(f"no Load of {buf}")
    return text


def rescale_texts(text: str, texts: dict) -> str:
    for old, new in texts.items():
        if old not in text:
            raise ValueError(f"{old!r} not found")
        text = text.replace(old, new)
    return text


def make(reference: Path, name: str) -> Path:
    src_rel, axes, shapes, grid_x, constants, *rest = PLAN[name]
    literals = rest[0] if rest else {}
    texts = rest[1] if len(rest) > 1 else {}
    options = rest[2] if len(rest) > 2 else {}
    dtypes = options.get("dtypes", {})
    src = reference / src_rel
    (ir_path,) = sorted(src.glob("*.ir.json"))
    graph = json.loads(ir_path.read_text())
    for node in graph["nodes"].values():
        if node["op"] == "KernelOp":
            node["op_fields"]["body"] = [retype_loads(rescale_texts(rescale_literals(rescale_body(b, axes), literals),
                                                                    texts), dtypes)
                                         for b in node["op_fields"]["body"]]
        for out in node.get("outputs", []):
            if out["name"] in shapes:
                out["shape"] = shapes[out["name"]]
            if out["name"] in dtypes:
                out["dtype"] = dtypes[out["name"]]
        if node["op"] == "ConstantOp" and node["op_fields"].get("name") in constants:
            node["op_fields"]["value"] = constants[node["op_fields"]["name"]]
    meta = json.loads((src / "meta.json").read_text())
    meta["id"] = f"{meta['id']}_rescaled"
    for kernel in meta["kernels"]:
        kernel["grid"] = [grid_x, 1, 1]
        if "block" in options:
            kernel["block"] = [options["block"], 1, 1]
        for arg in kernel["args"]:
            if arg["name"] in shapes:
                arg["shape"] = shapes[arg["name"]]
            if arg["name"] in constants:
                arg["data"] = [constants[arg["name"]]]
            if arg["name"] in dtypes:
                arg["dtype"] = dtypes[arg["name"]]
    dst = OUT / "rescaled" / name
    dst.mkdir(parents=True, exist_ok=True)
    (dst / ir_path.name).write_text(json.dumps(graph))
    (dst / "meta.json").write_text(json.dumps(meta, indent=1))
    return dst / ir_path.name


def main(reference: Path) -> int:
    sys.path.insert(0, str(HERE / "emmy_shim"))
    sys.path.insert(0, str(reference))
    import ptx_backend  # the reference compiler, unchanged

    (OUT / "ptx_rescaled").mkdir(parents=True, exist_ok=True)
    manifest = {}
    for name in PLAN:
        ir = make(reference, name)
        ptx = ptx_backend.compile_file(ir)
        (OUT / "ptx_rescaled" / f"{name}.ptx").write_text(ptx)
        manifest[name] = {"package": str(ir.parent.relative_to(HERE.parent)),
                          "sha256": hashlib.sha256(ptx.encode("ascii")).hexdigest(),
                          "meta": json.loads((ir.parent / "meta.json").read_text())}
        print(f"{name}: rescaled and compiled by the reference")
    (OUT / "manifest_rescaled.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python oracle/rescale.py REFERENCE_CHECKOUT")
    sys.exit(main(Path(sys.argv[1]).resolve()))
