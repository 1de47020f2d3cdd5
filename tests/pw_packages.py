"""Builders of small pointwise IR packages (kernel.ir.json + meta.json) —
test infrastructure for the pointwise-program compiler.

Statements are written as IR ``repr`` text, the form the reference's
packages carry, with helpers for the common node spellings.
"""
import json
from pathlib import Path

_NP = {"f32": ("float32", 4), "f16": ("float16", 2), "bf16": ("uint16", 2), "i32": ("int32", 4)}


def dt(name):
    np_name, size = _NP[name]
    return f"DataType(name='{name}', np=dtype('{np_name}'), nbytes={size})"


def var(name):
    return f"Var(name='{name}')"


def lit(value, kind="int"):
    if kind == "int":
        return f"Literal(value={value}, dtype='int')"
    return f"Literal(value={value!r}, dtype={dt(kind)})"


def bin_(op, a, b):
    return f"BinaryExpr(op='{op}', left={a}, right={b})"


def load(name, buf, index, kind):
    return f"Load(names=('{name}',), input='{buf}', index=({', '.join(index)},), dtype={dt(kind)})"


def assign(name, op, args, kind=None):
    d = dt(kind) if kind else "None"
    return f"Assign(name='{name}', op=ElementwiseImpl('{op}'), args=({', '.join(repr(a) for a in args)},), dtype={d})"


def let(name, value, kind=None):
    d = dt(kind) if kind else "None"
    return f"Let(name='{name}', value={value}, dtype={d})"


def write(out, index, values, kind):
    return (f"Write(output='{out}', index=({', '.join(index)},), values=({', '.join(repr(v) for v in values)},), "
            f"value_dtype={dt(kind)}, atomic=False, swizzle='NONE')")


def package(folder: Path, name: str, inputs: dict, output: tuple, axes: list, body: list, rtol=1e-5,
            atol=1e-6, data: dict | None = None) -> Path:
    """Write a one-kernel package; inputs {name: (shape, dtype)}, output (name, shape, dtype)."""
    folder.mkdir(parents=True, exist_ok=True)
    out_name, out_shape, out_dtype = output
    axes_repr = ", ".join(f"Axis(name='{a}', extent=Dim({e}), window=None)" for a, e in axes)
    tile = (f"Tile(axes=({axes_repr},), body=({', '.join(body)},), block_threads=None, aux_threads=0, "
            f"raster_axes=None, raster_group=None, raster_orient='m')")
    entry = f"k_{name}"
    nodes = {n: {"op": "InputOp", "op_fields": {}, "inputs": [],
                 "outputs": [{"name": n, "shape": list(s), "dtype": d}]} for n, (s, d) in inputs.items()}
    nodes[out_name] = {"op": "KernelOp", "op_fields": {"body": [tile], "name": entry, "zero_delegated": [],
                                                       "serial": []},
                       "inputs": list(inputs), "outputs": [{"name": out_name, "shape": list(out_shape),
                                                            "dtype": out_dtype}]}
    graph = {"inputs": list(inputs), "outputs": [out_name], "nodes": nodes}
    ir = folder / f"{entry}.ir.json"
    ir.write_text(json.dumps(graph))
    args = []
    for i, (n, (s, d)) in enumerate(inputs.items()):
        a = {"name": n, "dtype": d, "shape": list(s), "seed": i}
        if data and n in data:
            a["data"] = list(data[n])
        args.append(a)
    args.append({"name": out_name, "dtype": out_dtype, "shape": list(out_shape), "output": True})
    meta = {"id": name, "rtol": rtol, "atol": atol, "graph_inputs": list(inputs), "graph_outputs": [out_name],
            "kernels": [{"node": out_name, "entry": entry, "arg_order": list(inputs) + [out_name],
                         "grid": [1, 1, 1], "block": [256, 1, 1], "smem_bytes": 0, "zero_outputs": [],
                         "args": args, "final": True}]}
    (folder / "meta.json").write_text(json.dumps(meta))
    return ir


# ---------------------------------------------------------------- synthetic programs
# name -> (builder(folder) -> ir path, tolerance): op mixes beyond the fixed classes

def _bias_rows(folder):
    i, j = var("i"), var("j")
    return package(folder, "bias_rows", {"x": ((64, 48), "f32"), "w": ((48,), "f32"), "b": ((48,), "f32")},
                   ("out", (64, 48), "f32"), [("i", 64), ("j", 48)],
                   [load("xv", "x", [i, j], "f32"), load("wv", "w", [j], "f32"), load("bv", "b", [j], "f32"),
                    assign("p", "multiply", ["xv", "wv"], "f32"), assign("s", "add", ["p", "bv"], "f32"),
                    assign("y", "sigmoid", ["s"], "f32"), write("out", [i, j], ["y"], "f32")])


def _half_io(folder):
    i = var("i")
    return package(folder, "half_io", {"x": ((1000,), "f16"), "y": ((1000,), "f16")}, ("out", (1000,), "f16"),
                   [("i", 1000)],
                   [load("xv", "x", [i], "f16"), load("yv", "y", [i], "f16"),
                    assign("sx", "silu", ["xv"], "f16"), let("half", lit(0.5, "f16"), "f16"),
                    assign("hy", "multiply", ["yv", "half"], "f16"), assign("d", "subtract", ["sx", "hy"], "f16"),
                    write("out", [i], ["d"], "f16")], rtol=2e-3, atol=2e-3)


def _bf16_mix(folder):
    i = var("i")
    return package(folder, "bf16_mix", {"x": ((777,), "bf16")}, ("out", (777,), "f32"), [("i", 777)],
                   [load("xv", "x", [i], "bf16"), assign("t", "tanh", ["xv"], "bf16"),
                    let("k", lit(0.1, "f32"), "f32"), let("xf", var("xv"), "f32"),
                    assign("sc", "multiply", ["xf", "k"], "f32"), assign("e", "exp", ["sc"], "f32"),
                    let("tf", var("t"), "f32"), assign("r", "add", ["tf", "e"], "f32"),
                    write("out", [i], ["r"], "f32")], rtol=1e-2, atol=1e-2)


def _int_select(folder):
    i = var("i")
    return package(folder, "int_select", {"n": ((256,), "i32"), "x": ((256,), "f32")}, ("out", (256,), "f32"),
                   [("i", 256)],
                   [load("nv", "n", [i], "i32"), load("xv", "x", [i], "f32"),
                    let("three", lit(3), None), assign("m", "remainder", ["nv", "three"], None),
                    let("zero", lit(0), None), assign("c", "equal", ["m", "zero"], "i32"),
                    assign("ax", "abs", ["xv"], "f32"), assign("sq", "sqrt", ["ax"], "f32"),
                    assign("ng", "negative", ["xv"], "f32"), assign("r", "where", ["c", "sq", "ng"], "f32"),
                    write("out", [i], ["r"], "f32")],
                   data={"n": [(-1) ** k * (k * 7919 % 1000) for k in range(256)]})


def _compare_flags(folder):
    i = var("i")
    rows = 300
    body = [load("xv", "x", [i], "f32"), load("yv", "y", [i], "f32"), let("zero", lit(0.0, "f32"), "f32"),
            assign("pos", "greater", ["xv", "zero"], "i32"), assign("eq", "equal", ["xv", "yv"], "i32"),
            assign("nan", "not_equal", ["xv", "xv"], "i32"), assign("any", "logical_or", ["pos", "nan"], "i32")]
    body += [write("out", [bin_("+", bin_("*", i, lit(4)), lit(c))], [v], "i32")
             for c, v in enumerate(("pos", "eq", "nan", "any"))]
    data_x = [float("nan") if k % 17 == 0 else (k % 7) - 3.0 for k in range(rows)]
    data_y = [(k % 5) - 2.0 for k in range(rows)]
    return package(folder, "compare_flags", {"x": ((rows,), "f32"), "y": ((rows,), "f32")},
                   ("out", (rows * 4,), "i32"), [("i", rows)], body, rtol=0, atol=0,
                   data={"x": data_x, "y": data_y})


def _erf_log(folder):
    i = var("i")
    return package(folder, "erf_log", {"x": ((4099,), "f32"), "y": ((4099,), "f32")}, ("out", (4099,), "f32"),
                   [("i", 4099)],
                   [load("xv", "x", [i], "f32"), load("yv", "y", [i], "f32"), assign("e", "erf", ["xv"], "f32"),
                    assign("x2", "square", ["xv"], "f32"), let("one", lit(1.0, "f32"), "f32"),
                    assign("q", "add", ["x2", "one"], "f32"), assign("l", "log", ["q"], "f32"),
                    assign("rs", "rsqrt", ["q"], "f32"), let("three", lit(3.0, "f32"), "f32"),
                    assign("t3", "multiply", ["xv", "three"], "f32"), assign("fl", "floor", ["t3"], "f32"),
                    assign("mx", "maximum", ["xv", "yv"], "f32"), assign("s1", "add", ["e", "l"], "f32"),
                    assign("s2", "add", ["s1", "rs"], "f32"), assign("s3", "add", ["s2", "fl"], "f32"),
                    assign("s4", "add", ["s3", "mx"], "f32"), write("out", [i], ["s4"], "f32")],
                   rtol=1e-5, atol=2e-6)


def _vector_rows(folder):
    i = var("i")
    idx = bin_("*", i, lit(4))
    return package(folder, "vector_rows", {"x": ((128,), "f32")}, ("out", (128,), "f32"), [("i", 32)],
                   [f"Load(names=('a', 'b', 'c', 'd'), input='x', index=({idx},), dtype={dt('f32')})"] +
                   [assign(f"r{k}", "relu", [v], "f32") for k, v in enumerate("abcd")] +
                   [write("out", [idx], ["r0", "r1", "r2", "r3"], "f32")], rtol=0, atol=0)


def _transposed(folder):
    i, j = var("i"), var("j")
    return package(folder, "transposed", {"x": ((40, 24), "f32")}, ("out", (24, 40), "f32"), [("i", 40), ("j", 24)],
                   [load("xv", "x", [i, j], "f32"), let("two", lit(2.0, "f32"), "f32"),
                    assign("y", "multiply", ["xv", "two"], "f32"), write("out", [j, i], ["y"], "f32")],
                   rtol=0, atol=0)


SYNTHETIC = {"bias_rows": _bias_rows, "half_io": _half_io, "bf16_mix": _bf16_mix, "int_select": _int_select,
             "compare_flags": _compare_flags, "erf_log": _erf_log, "vector_rows": _vector_rows,
             "transposed": _transposed}


def chain_package(folder: Path, n: int = 4096) -> Path:
    """Two kernels chained through an intermediate: t = 2 x, then out = t + y."""
    folder.mkdir(parents=True, exist_ok=True)
    i = var("i")
    first = [load("xv", "x", [i], "f32"), let("two", lit(2.0, "f32"), "f32"),
             assign("tv", "multiply", ["xv", "two"], "f32"), write("t", [i], ["tv"], "f32")]
    second = [load("tv", "t", [i], "f32"), load("yv", "y", [i], "f32"),
              assign("ov", "add", ["tv", "yv"], "f32"), write("out", [i], ["ov"], "f32")]
    kernels = []
    for entry, ins, out, body in (("k_first", ["x"], "t", first), ("k_second", ["t", "y"], "out", second)):
        tile = (f"Tile(axes=(Axis(name='i', extent=Dim({n}), window=None),), body=({', '.join(body)},), "
                "block_threads=None, aux_threads=0, raster_axes=None, raster_group=None, raster_orient='m')")
        nodes = {name: {"op": "InputOp", "op_fields": {}, "inputs": [],
                        "outputs": [{"name": name, "shape": [n], "dtype": "f32"}]} for name in ins}
        nodes[out] = {"op": "KernelOp", "op_fields": {"body": [tile], "name": entry, "zero_delegated": [],
                                                      "serial": []},
                      "inputs": ins, "outputs": [{"name": out, "shape": [n], "dtype": "f32"}]}
        (folder / f"{entry}.ir.json").write_text(json.dumps({"inputs": ins, "outputs": [out], "nodes": nodes}))
        args = []
        for name in ins:
            if name == "t":
                args.append({"name": "t", "dtype": "f32", "shape": [n], "intermediate": True})
            else:
                args.append({"name": name, "dtype": "f32", "shape": [n], "seed": 0 if name == "x" else 1})
        args.append({"name": out, "dtype": "f32", "shape": [n], "output": True})
        kernels.append({"node": out, "entry": entry, "arg_order": ins + [out], "grid": [1, 1, 1],
                        "block": [256, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args,
                        "final": out == "out"})
    meta = {"id": "chain", "rtol": 0, "atol": 0, "graph_inputs": ["x", "y"], "graph_outputs": ["out"],
            "kernels": kernels}
    (folder / "meta.json").write_text(json.dumps(meta))
    return folder


# ---------------------------------------------------------------- reduction / fused row programs

def row_package(folder: Path, name: str, rows: int, cols: int, inputs: dict, output: tuple, pass1: list,
                accs: list, final: list = (), final_writes: list = (), pass2: list = (), block: int = 128,
                rtol=1e-5, atol=1e-6) -> Path:
    """A Tile [a0 rows, a1_co block] with the reference's reduction schedule:
    pass 1 strides the block over the row (body + Accum of each (acc, op, value)),
    a warp butterfly and a shared-memory tree combine each accumulator, then an
    optional second pass (loop variable a2) and per-row statements guarded to
    thread 0."""
    row, co = var("a0"), var("a1_co")
    f32 = dt("f32")
    loop1 = list(pass1) + [f"Accum(name='{a}', value='{v}', op=ElementwiseImpl('{o}'), dtype={f32}, axes=('a1',), base=None)"
                          for a, o, v in accs]
    states = tuple(a for a, _, _ in accs)
    combine = ", ".join(f"Assign(name='{a}', op=ElementwiseImpl('{o}'), args=('{a}', '{a}__o'), dtype=None)"
                        for a, o, _ in accs)
    st = ", ".join(repr(a) for a in states) + ","
    stb = ", ".join(repr(a + "__o") for a in states) + ","
    warps = block // 32
    body = [f"StridedLoop(axis=Axis(name='a1', extent=Dim({cols}), window=None), start={co}, step={lit(block)}, "
            f"body=({', '.join(loop1)},), unroll=False, end=None, seed=True)",
            f"WarpShuffle(state=({st}), state_b=({stb}), combine_states=({combine},), length=32, dtype={f32})"]
    for a in states:
        body.append(f"Smem(name='{a}_smem', extents=({warps},), dtype='float', align=0)")
    body.append(f"Cond(cond=BinaryExpr(op='==', left=Var(name='lane'), right={lit(0)}), body=(" +
                ", ".join(f"Write(output='{a}_smem', index=(Var(name='warp'),), values=('{a}',), value_dtype={f32}, "
                          "atomic=False, swizzle='NONE')" for a in states) + ",), else_body=())")
    body.append("Sync(barrier_id=0, count=None, warp=False)")
    smem = ", ".join(repr(a + "_smem") for a in states) + ","
    body.append(f"TreeHalve(bufs=({smem}), state=({st}), state_b=({stb}), combine_states=({combine},), "
                f"length={warps}, tid_var='warp', dtype={f32}, barrier_id=0, barrier_count=None, inner=None)")
    if pass2:
        body.append(f"StridedLoop(axis=Axis(name='a2', extent=Dim({cols}), window=None), start={co}, "
                    f"step={lit(block)}, body=({', '.join(pass2)},), unroll=False, end=None, seed=True)")
    if final or final_writes:
        body.append(f"Cond(cond=BinaryExpr(op='==', left={co}, right={lit(0)}), body=(" +
                    ", ".join(list(final) + list(final_writes)) + ",), else_body=())")
    folder.mkdir(parents=True, exist_ok=True)
    tile = (f"Tile(axes=(Axis(name='a0', extent=Dim({rows}), window=None), Axis(name='a1_co', extent=Dim({block}), "
            f"window=None)), body=({', '.join(body)},), block_threads={block}, aux_threads=0, raster_axes=None, "
            "raster_group=None, raster_orient='m')")
    out_name, out_shape, out_dtype = output
    entry = f"k_{name}"
    nodes = {n: {"op": "InputOp", "op_fields": {}, "inputs": [], "outputs": [{"name": n, "shape": list(s), "dtype": d}]}
             for n, (s, d) in inputs.items()}
    nodes[out_name] = {"op": "KernelOp", "op_fields": {"body": [tile], "name": entry, "zero_delegated": [],
                                                       "serial": []},
                       "inputs": list(inputs), "outputs": [{"name": out_name, "shape": list(out_shape),
                                                            "dtype": out_dtype}]}
    (folder / f"{entry}.ir.json").write_text(json.dumps({"inputs": list(inputs), "outputs": [out_name], "nodes": nodes}))
    args = [{"name": n, "dtype": d, "shape": list(s), "seed": i} for i, (n, (s, d)) in enumerate(inputs.items())]
    args.append({"name": out_name, "dtype": out_dtype, "shape": list(out_shape), "output": True})
    meta = {"id": name, "rtol": rtol, "atol": atol, "graph_inputs": list(inputs), "graph_outputs": [out_name],
            "kernels": [{"node": out_name, "entry": entry, "arg_order": list(inputs) + [out_name], "grid": [rows, 1, 1],
                         "block": [block, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args, "final": True}]}
    (folder / "meta.json").write_text(json.dumps(meta))
    return folder / f"{entry}.ir.json"


def _x(cols):
    return load("xv", "x", [var("a0"), var("a1")], "f32")


def _row_max(folder):
    return row_package(folder, "row_max", 37, 300, {"x": ((37, 300), "f32")}, ("out", (37,), "f32"),
                       [_x(300)], [("m", "maximum", "xv")], final_writes=[write("out", [var("a0")], ["m"], "f32")])


def _row_min_abs(folder):
    return row_package(folder, "row_min_abs", 16, 1000, {"x": ((16, 1000), "f32")}, ("out", (16,), "f32"),
                       [_x(1000), assign("ax", "abs", ["xv"], "f32")], [("m", "minimum", "ax")],
                       final_writes=[write("out", [var("a0")], ["m"], "f32")])


def _variance(folder):
    cols = 777
    return row_package(folder, "variance", 24, cols, {"x": ((24, cols), "f32")}, ("out", (24,), "f32"),
                       [_x(cols), assign("sq", "multiply", ["xv", "xv"], "f32")],
                       [("s1", "add", "xv"), ("s2", "add", "sq")],
                       final=[let("inv", lit(1.0 / cols, "f32"), "f32"), assign("mean", "multiply", ["s1", "inv"], "f32"),
                              assign("msq", "multiply", ["s2", "inv"], "f32"),
                              assign("m2", "multiply", ["mean", "mean"], "f32"),
                              assign("var", "subtract", ["msq", "m2"], "f32")],
                       final_writes=[write("out", [var("a0")], ["var"], "f32")], rtol=1e-4, atol=1e-5)


def _log_sum_exp(folder):
    """Row max, then a second pass is a write; here the sum of exp(x - 0) and its log."""
    cols = 512
    return row_package(folder, "log_sum_exp", 20, cols, {"x": ((20, cols), "f32")}, ("out", (20,), "f32"),
                       [_x(cols), assign("e", "exp", ["xv"], "f32")], [("s", "add", "e")],
                       final=[assign("l", "log", ["s"], "f32")],
                       final_writes=[write("out", [var("a0")], ["l"], "f32")], rtol=1e-5, atol=1e-5)


def _center_rows(folder):
    """Two passes: the row mean, then every element minus it, scaled by w[col]."""
    cols = 640
    a0, a2 = var("a0"), var("a2")
    return row_package(folder, "center_rows", 33, cols, {"x": ((33, cols), "f32"), "w": ((cols,), "f32")},
                       ("out", (33, cols), "f32"), [_x(cols)], [("s", "add", "xv")],
                       pass2=[load("x2", "x", [a0, a2], "f32"), load("wv", "w", [a2], "f32"),
                              let("inv", lit(1.0 / cols, "f32"), "f32"), assign("mean", "multiply", ["s", "inv"], "f32"),
                              assign("d", "subtract", ["x2", "mean"], "f32"), assign("o", "multiply", ["d", "wv"], "f32"),
                              write("out", [a0, a2], ["o"], "f32")], rtol=1e-5, atol=1e-5)


def _half_row_sum(folder):
    """f16 storage: the row sum of x (f16) written as f16."""
    cols = 256
    return row_package(folder, "half_row_sum", 40, cols, {"x": ((40, cols), "f16")}, ("out", (40,), "f16"),
                       [load("xv", "x", [var("a0"), var("a1")], "f16")], [("s", "add", "xv")],
                       final_writes=[write("out", [var("a0")], ["s"], "f16")], rtol=2e-3, atol=2e-3)


ROW_SYNTHETIC = {"row_max": _row_max, "row_min_abs": _row_min_abs, "variance": _variance,
                 "log_sum_exp": _log_sum_exp, "center_rows": _center_rows, "half_row_sum": _half_row_sum}


# ---------------------------------------------------------------- online-softmax variants (coupled states)

def _from_f02(folder: Path, name: str, edits: list) -> Path:
    """A copy of the f02 online-softmax package with textual edits of its IR."""
    import shutil
    src = Path(__file__).resolve().parent / "golden" / "packages" / "f02_row_softmax"
    shutil.copytree(src, folder)
    ir = next(folder.glob("*.ir.json"))
    text = ir.read_text()
    for old, new in edits:
        assert old in text, old
        text = text.replace(old, new)
    ir.write_text(text)
    meta = json.loads((folder / "meta.json").read_text())
    meta["id"] = name
    meta["rtol"], meta["atol"] = 1e-5, 1e-6
    (folder / "meta.json").write_text(json.dumps(meta))
    return ir


def _log_softmax(folder):
    """log softmax: x - max - log(sum exp(x - max)) from the same coupled states."""
    return _from_f02(folder, "log_softmax", [
        ("Assign(name='v4', op=ElementwiseImpl('exp'), args=('v3',)",
         "Assign(name='v4', op=ElementwiseImpl('log'), args=('acc1',)"),
        ("Assign(name='v5', op=ElementwiseImpl('multiply'), args=('v2', 'v4')",
         "Assign(name='v5', op=ElementwiseImpl('subtract'), args=('v3', 'v4')")])


def _softmax_times_x(folder):
    """softmax(x) * x (an attention-like reweighting of the row by itself)."""
    return _from_f02(folder, "softmax_times_x", [
        ("Assign(name='v5', op=ElementwiseImpl('multiply'), args=('v2', 'v4')",
         "Assign(name='v6', op=ElementwiseImpl('multiply'), args=('v2', 'v4'), dtype=None), "
         "Assign(name='v5', op=ElementwiseImpl('multiply'), args=('v6', 'in2')")])


ROW_COUPLED = {"log_softmax": _log_softmax, "softmax_times_x": _softmax_times_x}


# ---------------------------------------------------------------- serial programs (per-point runtime loops)

def serial_package(folder: Path, name: str, inputs: dict, output: tuple, axes: list, body: list, rtol=1e-5,
                   atol=1e-6) -> Path:
    return package(folder, name, inputs, output, axes, body, rtol=rtol, atol=atol)


def loop(name, extent, body, seed=True):
    return (f"Loop(axis=Axis(name='{name}', extent=Dim({extent}), window=None), body=({', '.join(body)},), "
            f"unroll=False, seed={seed})")


def accum(name, value, op, base=None):
    b = repr(base) if base else "None"
    return f"Accum(name='{name}', value='{value}', op=ElementwiseImpl('{op}'), dtype={dt('f32')}, axes=(), base={b})"


def _serial_matmul_relu(folder):
    i, j, k = var("i"), var("j"), var("k")
    return serial_package(folder, "serial_matmul_relu", {"a": ((24, 40), "f32"), "b": ((40, 17), "f32"),
                                                         "bias": ((17,), "f32")},
                          ("out", (24, 17), "f32"), [("i", 24), ("j", 17)],
                          [loop("k", 40, [load("av", "a", [i, k], "f32"), load("bv", "b", [k, j], "f32"),
                                          assign("p", "multiply", ["av", "bv"], "f32"), accum("acc", "p", "add")]),
                           load("cv", "bias", [j], "f32"), assign("s", "add", ["acc", "cv"], "f32"),
                           assign("r", "relu", ["s"], "f32"), write("out", [i, j], ["r"], "f32")])


def _serial_row_max_argmax_value(folder):
    """Per point: the max over k of |x[i, k] * w[k]| (a serial max reduction)."""
    i, k = var("i"), var("k")
    return serial_package(folder, "serial_max_abs", {"x": ((50, 70), "f32"), "w": ((70,), "f32")},
                          ("out", (50,), "f32"), [("i", 50)],
                          [loop("k", 70, [load("xv", "x", [i, k], "f32"), load("wv", "w", [k], "f32"),
                                          assign("p", "multiply", ["xv", "wv"], "f32"),
                                          assign("q", "abs", ["p"], "f32"), accum("m", "q", "maximum")]),
                           write("out", [i], ["m"], "f32")])


def _serial_nested(folder):
    """Nested loops: out[i] = sum_k exp(sum_d q[i, d] * kt[d, k] / 4)."""
    i, k, d = var("i"), var("k"), var("d")
    return serial_package(folder, "serial_nested", {"q": ((12, 8), "f32"), "kt": ((8, 20), "f32")},
                          ("out", (12,), "f32"), [("i", 12)],
                          [let("quarter", lit(0.25, "f32"), "f32"),
                           loop("k", 20, [loop("d", 8, [load("qv", "q", [i, d], "f32"), load("kv", "kt", [d, k], "f32"),
                                                        assign("p", "multiply", ["qv", "kv"], "f32"),
                                                        accum("dot", "p", "add")]),
                                          assign("s", "multiply", ["dot", "quarter"], "f32"),
                                          assign("e", "exp", ["s"], "f32"), accum("tot", "e", "add")]),
                           write("out", [i], ["tot"], "f32")], rtol=1e-5, atol=1e-6)


def _serial_lower_matmul(folder):
    # out[i, j] = sum over k <= i of a[i, k] * b[k, j]: the loop counter and a tile
    # coordinate as values (a causal-style mask)
    i, j, k = var("i"), var("j"), var("k")
    body = [loop("k", 24, [load("av", "a", [i, k], "f32"), load("bv", "b", [k, j], "f32"),
                           assign("pv", "multiply", ["av", "bv"]),
                           let("keep", "TernaryExpr(cond=BinaryExpr(op='<=', left=Var(name='k'), "
                               "right=Var(name='i')), if_true=Var(name='pv'), if_false=" + lit(0.0, "f32") + ")"),
                           accum("acc", "keep", "add")]),
            write("out", [i, j], ["acc"], "f32")]
    return serial_package(folder, "serial_lower_matmul", {"a": ((20, 24), "f32"), "b": ((24, 12), "f32")},
                          ("out", (20, 12), "f32"), [("i", 20), ("j", 12)], body)


def _pointwise_lower_mask(folder):
    # out[i, j] = x[i, j] where j <= i, else -x[i, j] * (i - j): coordinates as values
    i, j = var("i"), var("j")
    return package(folder, "pointwise_lower_mask", {"x": ((32, 48), "f32")}, ("out", (32, 48), "f32"),
                   [("i", 32), ("j", 48)],
                   [load("xv", "x", [i, j], "f32"),
                    let("d", "CastExpr(expr=BinaryExpr(op='-', left=Var(name='i'), right=Var(name='j')), "
                        "dtype='float')", "f32"),
                    assign("nx", "multiply", ["xv", "d"]), assign("mx", "negative", ["nx"]),
                    let("v", "TernaryExpr(cond=BinaryExpr(op='<=', left=Var(name='j'), right=Var(name='i')), "
                        "if_true=Var(name='xv'), if_false=Var(name='mx'))", "f32"),
                    write("out", [i, j], ["v"], "f32")])


SYNTHETIC["pointwise_lower_mask"] = _pointwise_lower_mask

SERIAL_SYNTHETIC = {"serial_lower_matmul": _serial_lower_matmul, "serial_matmul_relu": _serial_matmul_relu, "serial_max_abs": _serial_row_max_argmax_value,
                    "serial_nested": _serial_nested}


# ---------------------------------------------------------------- op-mix variants of the reference's packages
# (package, textual edits of its IR, plan op, oracle module name): bodies a fixed class no longer
# matches, which must run as the general program they are.

VARIANTS = {
    "bias_gemm_tanh_gate": ("phase9_bias_gelu_gemm", [("ElementwiseImpl('erf')", "ElementwiseImpl('tanh')")],
                            "rowprog", "rowprog_ir"),
    "bias_gemm_relu": ("phase9_bias_gelu_gemm",
                       [("Assign(name='v6', op=ElementwiseImpl('multiply'), args=('v4', 'v5')",
                         "Assign(name='v6', op=ElementwiseImpl('relu'), args=('v1',)")], "rowprog", "rowprog_ir"),
    "attention_sqrt_scale": ("a01_attention", [("ElementwiseImpl('reciprocal')", "ElementwiseImpl('sqrt')")],
                             "pointwise", "serial_ir"),
    "attention_128_negated_scale": ("a02_attention_128",
                                    [("Assign(name='v1', op=ElementwiseImpl('reciprocal'), args=('in0',)",
                                      "Assign(name='v1', op=ElementwiseImpl('negative'), args=('in0',)")],
                                    "pointwise", "serial_ir"),
    "gelu_attention_tanh_score": ("phase9_gelu_attention",
                                  [("Assign(name='v1', op=ElementwiseImpl('multiply'), args=('acc0', 'in3')",
                                    "Assign(name='v1', op=ElementwiseImpl('tanh'), args=('acc0',)")],
                                  "blockprog", "staged_ir"),
    "split_k_relu_a": ("m02_matmul_rect",
                       [("Assign(name='acc0__v__c0_0', op=ElementwiseImpl('multiply'), args=('in1__c0_0', 'in0__c0_0')",
                         "Assign(name='r0', op=ElementwiseImpl('relu'), args=('in0__c0_0',), dtype=None), "
                         "Assign(name='acc0__v__c0_0', op=ElementwiseImpl('multiply'), args=('in1__c0_0', 'r0')"),
                        ("Assign(name='acc0__v__c1_0', op=ElementwiseImpl('multiply'), args=('in1__c0_0', 'in0__c1_0')",
                         "Assign(name='r1', op=ElementwiseImpl('relu'), args=('in0__c1_0',), dtype=None), "
                         "Assign(name='acc0__v__c1_0', op=ElementwiseImpl('multiply'), args=('in1__c0_0', 'r1')")],
                       "blockprog", "staged_ir"),
    "row_sum_of_abs": ("r04_row_sum",
                       [("Accum(name='acc0', value='in0'", "Assign(name='ax', op=ElementwiseImpl("
                         "'abs'), args=('in0',), dtype=None), Accum(name='acc0', value='ax'")],
                       "rowprog", "rowprog_ir"),
}


def variant(folder: Path, name: str) -> Path:
    import shutil
    src, edits, _, _ = VARIANTS[name]
    shutil.copytree(Path(__file__).resolve().parent / "golden" / "packages" / src, folder)
    ir = next(folder.glob("*.ir.json"))
    text = ir.read_text()
    for old, new in edits:
        assert old in text, old
        text = text.replace(old, new)
    ir.write_text(text)
    return ir


# ---------------------------------------------------------------- staged matmul epilogues
# m01 (the staged cp.async matmul) with an expression of each accumulator
# written instead of the accumulator; ``epilogue(acc_name, tag)`` returns the
# statements and the name to write.  ``extra`` adds inputs {name: (shape, seed)}.

def staged_epilogue(folder: Path, epilogue, extra: dict | None = None) -> Path:
    import re
    import shutil
    shutil.copytree(Path(__file__).resolve().parent / "golden" / "packages" / "m01_matmul_512", folder)
    ir = next(folder.glob("*.ir.json"))
    graph = json.loads(ir.read_text())
    node = graph["nodes"]["matmul"]
    body = node["op_fields"]["body"][0]
    pieces, pos, count = [], 0, 0
    for m in re.finditer(r"Write\(output='matmul', index=\((.*?)\), values=\(([^)]*)\)", body):
        row, col = _split_top(m.group(1))
        names = [n.strip().strip("'") for n in m.group(2).split(",") if n.strip()]
        stmts, new = [], []
        for lane, name in enumerate(names):
            s, out = epilogue(name, f"e{count}", row, bin_("+", col, lit(lane)))
            count += 1
            stmts += s
            new.append(out)
        pieces.append(body[pos:m.start()])
        pieces.append(", ".join(stmts) + ", ")
        values = ", ".join(f"'{n}'" for n in new) + ("," if len(new) == 1 else "")
        pieces.append(body[m.start():m.start(2)] + values)
        pos = m.end(2)
    pieces.append(body[pos:])
    node["op_fields"]["body"][0] = "".join(pieces)
    meta = json.loads((folder / "meta.json").read_text())
    kernel = meta["kernels"][0]
    for name, (shape, seed) in (extra or {}).items():
        graph["inputs"].append(name)
        graph["nodes"][name] = {"op": "InputOp", "op_fields": {}, "inputs": [],
                                "outputs": [{"name": name, "shape": list(shape), "dtype": "f32"}]}
        node["inputs"].append(name)
        meta["graph_inputs"].append(name)
        kernel["arg_order"].insert(len(kernel["arg_order"]) - 1, name)
        kernel["args"].insert(len(kernel["args"]) - 1, {"name": name, "dtype": "f32", "shape": list(shape),
                                                         "seed": seed})
    ir.write_text(json.dumps(graph))
    (folder / "meta.json").write_text(json.dumps(meta))
    return ir


def _split_top(text: str) -> list:
    """Top-level comma-separated parts of an IR tuple's text."""
    parts, depth, start = [], 0, 0
    for i, ch in enumerate(text):
        if ch == "(":
            depth += 1
        elif ch == ")":
            depth -= 1
        elif ch == "," and depth == 0:
            parts.append(text[start:i].strip())
            start = i + 1
    parts.append(text[start:].strip())
    return [p for p in parts if p]


def _staged_tanh(folder):
    return staged_epilogue(folder, lambda acc, t, row, col: ([assign(t, "tanh", [acc])], t))


def _staged_scaled_silu(folder):
    # v = 0.25 * acc; v * sigmoid(v)
    def epi(acc, t, row, col):
        return ([let(f"{t}c", lit(0.25, "f32"), "f32"), assign(f"{t}v", "multiply", [acc, f"{t}c"]),
                 assign(f"{t}g", "sigmoid", [f"{t}v"]), assign(t, "multiply", [f"{t}v", f"{t}g"])], t)
    return staged_epilogue(folder, epi)


def _staged_bias_residual(folder):
    # relu(acc + bias[col]) + 0.5 * res[row, col]: the loads sit at the write position
    def epi(acc, t, row, col):
        return ([f"Load(names=('{t}b',), input='bias', index=({col},), dtype=None)",
                 f"Load(names=('{t}r',), input='res', index=({row}, {col}), dtype=None)",
                 assign(f"{t}s", "add", [acc, f"{t}b"]), assign(f"{t}a", "relu", [f"{t}s"]),
                 let(f"{t}h", lit(0.5, "f32"), "f32"), assign(f"{t}q", "multiply", [f"{t}r", f"{t}h"]),
                 assign(t, "add", [f"{t}a", f"{t}q"])], t)
    return staged_epilogue(folder, epi, {"bias": ((512,), 2), "res": ((512, 512), 3)})


STAGED_EPILOGUES = {"staged_tanh": _staged_tanh, "staged_scaled_silu": _staged_scaled_silu,
                    "staged_bias_residual": _staged_bias_residual}


# ---------------------------------------------------------------- block programs
def block_package(folder: Path, name: str, inputs: dict, output: tuple, axes: list, body: list, threads: int,
                  rtol=1e-5, atol=1e-6) -> Path:
    """``package`` with the Tile's trailing axes a block of ``threads`` threads."""
    ir = package(folder, name, inputs, output, axes, body, rtol, atol)
    ir.write_text(ir.read_text().replace("block_threads=None", f"block_threads={threads}"))
    meta = json.loads((folder / "meta.json").read_text())
    meta["kernels"][0]["block"] = [threads, 1, 1]
    (folder / "meta.json").write_text(json.dumps(meta))
    return ir


def _captured_end_rows(folder):
    # out[r, t] = sum of x[r, c] over c = t, t + 16, ... below r * 10 + 20 (a per-row captured end)
    r, t = var("r"), var("t")
    end = bin_("+", bin_("*", r, lit(10)), lit(20))
    body = [f"Init(name='acc', identity=0.0, dtype={dt('f32')})",
            f"StridedLoop(axis=Axis(name='c', extent=Dim(64), window=None), start={t}, step={lit(16)}, "
            f"body=({load('xv', 'x', [r, var('c')], 'f32')}, {accum('acc', 'xv', 'add')}), unroll=False, "
            f"end={end}, seed=False)",
            write("out", [r, t], ["acc"], "f32")]
    return block_package(folder, "captured_end_rows", {"x": ((4, 64), "f32")}, ("out", (4, 16), "f32"),
                         [("r", 4), ("t", 16)], body, 16)


def _shared_transpose(folder):
    # each block stages a 16 x 16 tile in shared memory, syncs, and writes it transposed
    b, t = var("b"), var("t")
    row, col = bin_("/", t, lit(16)), bin_("%", t, lit(16))
    body = ["Smem(name='tile', extents=(16, 16), dtype='float', align=0)",
            load("xv", "x", [b, row, col], "f32"),
            f"Write(output='tile', index=({row}, {col}), values=('xv',), value_dtype={dt('f32')}, atomic=False, "
            "swizzle='NONE')",
            "Sync(barrier_id=0, count=None, warp=False)",
            f"Load(names=('tv',), input='tile', index=({col}, {row}), dtype=None)",
            write("out", [b, row, col], ["tv"], "f32")]
    return block_package(folder, "shared_transpose", {"x": ((3, 16, 16), "f32")}, ("out", (3, 16, 16), "f32"),
                         [("b", 3), ("t", 256)], body, 256)


BLOCK_SYNTHETIC = {"captured_end_rows": _captured_end_rows, "shared_transpose": _shared_transpose}
