"""Writes the compensated-dot (Dot2) known-answer packages — TEST INFRASTRUCTURE.

    python tests/golden/make_precision.py

The reference pins its compensated dot accumulation (Ogita, Rump and Oishi
2005, Algorithm 5.3; ptx_backend.py:571-593, enabled by meta rtol/atol > 0 at
ptx_backend.py:1860-1865) with exact-integer identities in
tests/test_precision.py:39-188 (``precision_cases``): separately rounded f32
products and sums lose them, Dot2 keeps them.  This script restates those
seven cases as IR packages in the reference's package format (graph JSON
with KernelOp bodies as the IR ``repr``, a meta.json, an expected.npz), built
by this script's own writers — no Emmy — and writes them to
``tests/golden/packages/precision_*``:

1. dot_product_and_sum_residual: 4097^2 - 4096*4098 == 1 (product residual)
   and 1e8 + n - 1e8 == n (addition residual), one dot per row;
2. dot_seed_false_slabs: the correction survives unseeded drain loops;
3. dot_nested_reset: an inner dot re-seeded per outer iteration, summed;
4. dot_shuffle_snapshot: a snapshot of the dot, then an 8-lane butterfly;
5. dot_half_inputs_float_state: f16 loads feeding an f32 product and state;
6. dot_standalone_initial_update: a plain update before the unseeded dot;
7. dot_followed_by_explicit_base: a later update with an explicit base.

Meta rtol = 1e-5, atol = 1e-6 (the reference's case defaults), so the
reference CLI's default policy compiles Dot2 in; the expected values are the
exact integers (the tests compare them exactly).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "packages"

DT = {"f32": "DataType(name='f32', np=dtype('float32'), nbytes=4)",
      "f16": "DataType(name='f16', np=dtype('float16'), nbytes=2)"}


def axis(name, n):
    return f"Axis(name='{name}', extent=Dim({n}), window=None)"


def var(name):
    return f"Var(name='{name}')"


def lit(v):
    return f"Literal(value={v!r}, dtype='{'int' if isinstance(v, int) else 'float'}')"


def binop(op, left, right):
    return f"BinaryExpr(op='{op}', left={left}, right={right})"


def tup(items):
    items = list(items)
    return "(" + ", ".join(items) + ("," if len(items) == 1 else "") + ")"


def names(items):
    return tup(repr(i) for i in items)


def load(name, buf, index, dt="f32"):
    return f"Load(names=('{name}',), input='{buf}', index={tup(index)}, dtype={DT[dt]})"


def assign(name, op, args, dt="f32"):
    return f"Assign(name='{name}', op=ElementwiseImpl('{op}'), args={names(args)}, dtype={DT[dt]})"


def accum(name, value, op, axes, base=None, dt="f32"):
    return (f"Accum(name='{name}', value='{value}', op=ElementwiseImpl('{op}'), dtype={DT[dt]}, "
            f"axes={names(axes)}, base={base!r})")


def init(name, identity, dt="f32"):
    return f"Init(name='{name}', identity={identity!r}, dtype={DT[dt]})"


def let(name, value, dt="f32"):
    return f"Let(name='{name}', value={value}, dtype={DT[dt]})"


def loop(ax, body, unroll=True, seed=True):
    return f"Loop(axis={ax}, body={tup(body)}, unroll={unroll}, seed={seed})"


def write(index, values, dt="f32"):
    return (f"Write(output='out', index={tup(index)}, values={names(values)}, value_dtype={DT[dt]}, "
            f"atomic=False, swizzle='NONE')")


def shuffle(state, other, combine, length, dt="f32"):
    return (f"WarpShuffle(state={names(state)}, state_b={names(other)}, combine_states={tup(combine)}, "
            f"length={length}, dtype={DT[dt]})")


def tile(ax, body):
    return (f"Tile(axes=({ax},), body={tup(body)}, block_threads=None, aux_threads=0, raster_axes=None, "
            f"raster_group=None, raster_orient='m')")


def dot_body(index, a_dt="f32"):
    return (load("a", "x", index, a_dt), load("b", "y", index, a_dt),
            assign("product", "multiply", ("a", "b")), accum("dot", "product", "add", ("k",)))


def package(name, body, x, y, expected, in_dt="f32"):
    entry = f"k_precision_{name}"
    out_shape = list(np.shape(expected))
    graph = {"inputs": ["x", "y"], "outputs": ["out"], "nodes": {
        "x": {"op": "InputOp", "op_fields": {}, "inputs": [],
              "outputs": [{"name": "x", "shape": list(x.shape), "dtype": in_dt}]},
        "y": {"op": "InputOp", "op_fields": {}, "inputs": [],
              "outputs": [{"name": "y", "shape": list(y.shape), "dtype": in_dt}]},
        "out": {"op": "KernelOp", "op_fields": {"body": [tile(axis("i", 8), body)], "name": entry,
                                                "zero_delegated": [], "serial": []},
                "inputs": ["x", "y"], "outputs": [{"name": "out", "shape": out_shape, "dtype": "f32"}]}}}
    args = [{"name": "x", "dtype": in_dt, "shape": list(x.shape), "data": x.ravel().tolist()},
            {"name": "y", "dtype": in_dt, "shape": list(y.shape), "data": y.ravel().tolist()},
            {"name": "out", "dtype": "f32", "shape": out_shape, "output": True}]
    meta = {"id": f"precision_{name}", "graph_inputs": ["x", "y"], "graph_outputs": ["out"],
            "rtol": 1e-5, "atol": 1e-6,
            "kernels": [{"node": "out", "entry": entry, "arg_order": ["x", "y", "out"], "grid": [1, 1, 1],
                         "block": [8, 1, 1], "smem_bytes": 0, "zero_outputs": [], "args": args, "final": True}]}
    folder = OUT / f"precision_{name}"
    folder.mkdir(parents=True, exist_ok=True)
    (folder / f"{entry}.ir.json").write_text(json.dumps(graph, indent=1) + "\n")
    (folder / "meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    np.savez(folder / "expected.npz", out=np.asarray(expected, np.float32))
    return folder


def cases():
    i, j, k = var("i"), var("j"), var("k")
    # 1. product residual (rows 0-3) and addition residual (rows 4-7)
    x = np.tile(np.asarray([4097, -4096, 0, 0], np.float32), (8, 1))
    y = np.tile(np.asarray([4097, 4098, 1, 1], np.float32), (8, 1))
    x[4:] = [[1e8, n, -1e8, 0] for n in range(1, 5)]
    y[4:] = 1
    yield ("dot_product_and_sum_residual",
           (loop(axis("k", 4), dot_body((i, k))), write((i,), ("dot",))),
           x, y, np.asarray([1, 1, 1, 1, 1, 2, 3, 4], np.float32), "f32")
    # 2. the correction of the first slab survives an unseeded second slab
    x = np.asarray([[1e8, n, -1e8, 0] for n in range(1, 9)], np.float32)
    y = np.ones_like(x)
    offset = binop("+", binop("*", j, lit(2)), k)
    yield ("dot_seed_false_slabs",
           (init("dot", 0.0), loop(axis("j", 2), (loop(axis("k", 2), dot_body((i, offset)), seed=False),),
                                   unroll=False), write((i,), ("dot",))),
           x, y, np.arange(1, 9, dtype=np.float32), "f32")
    # 3. an inner dot seeded again on every outer iteration
    x = np.asarray([[[1e8, n, -1e8], [1e8, 2 * n, -1e8]] for n in range(1, 9)], np.float32)
    y = np.ones_like(x)
    yield ("dot_nested_reset",
           (loop(axis("j", 2), (loop(axis("k", 3), dot_body((i, j, k))), accum("total", "dot", "add", ("j",))),
                 unroll=False), write((i,), ("total",))),
           x, y, 3 * np.arange(1, 9, dtype=np.float32), "f32")
    # 4. a snapshot of the dot, then a butterfly over 8 lanes
    x = np.asarray([[1e8, n, -1e8] for n in range(1, 9)], np.float32)
    y = np.ones_like(x)
    yield ("dot_shuffle_snapshot",
           (loop(axis("k", 3), dot_body((i, k))), let("before", var("dot")),
            shuffle(("dot",), ("other",), (assign("dot", "add", ("dot", "other")),), 8),
            write((i, lit(0)), ("before", "dot"))),
           x, y, np.column_stack((np.arange(1, 9), np.full(8, 36))).astype(np.float32), "f32")
    # 5. f16 inputs feeding an f32 product and state
    x = np.asarray([[2048, n, -2048] for n in range(1, 9)], np.float32)
    y = np.ones_like(x)
    yield ("dot_half_inputs_float_state",
           (loop(axis("k", 3), dot_body((i, k), "f16")), write((i,), ("dot",))),
           x.astype(np.float16), y.astype(np.float16), np.arange(1, 9, dtype=np.float32), "f16")
    # 6. a plain update before the unseeded dot
    x = np.asarray([[1e8, n, -1e8] for n in range(1, 9)], np.float32)
    y = np.ones_like(x)
    yield ("dot_standalone_initial_update",
           (init("dot", 0.0), let("initial", lit(5.0)), accum("dot", "initial", "add", ()),
            loop(axis("k", 3), dot_body((i, k)), seed=False), write((i,), ("dot",))),
           x, y, np.arange(6, 14, dtype=np.float32), "f32")
    # 7. a later update with an explicit base consumes, then replaces, the dot
    yield ("dot_followed_by_explicit_base",
           (loop(axis("k", 3), dot_body((i, k))), let("half", lit(0.5)), let("one", lit(1.0)),
            let("two", lit(2.0)), assign("scaled", "multiply", ("dot", "half")),
            assign("product", "multiply", ("one", "two")),
            accum("dot", "product", "add", (), base="scaled"), write((i,), ("dot",))),
           x, y, np.arange(1, 9, dtype=np.float32) / 2 + 2, "f32")


PACKAGES = [f"precision_{c[0]}" for c in cases()]


def main() -> None:
    for name, body, x, y, expected, dt in cases():
        print(package(name, body, x, y, expected, dt))


if __name__ == "__main__":
    main()
