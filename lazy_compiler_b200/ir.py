"""Loader for Emmy 0.3.11 scheduled Kernel IR packages (``*.ir.json`` + ``meta.json``).

The reference loads the IR with Emmy's ``Graph.from_dict`` (ptx_backend.py:1839)
and then walks Emmy dataclasses.  Emmy is a third-party package
(``emmy-ml==0.3.11``, requirements.txt:1) and is not vendored, so this module
reads the same JSON without it.  A KernelOp body is a Python ``repr`` string of
Emmy constructors.  It is parsed with :func:`ast.parse` and evaluated by a
closed whitelist of constructor names: nothing in the file is executed, and a
name outside the whitelist is a :class:`CompileError` (the reference raises
its ``CompileError`` for unsupported statements before printing anything,
ptx_backend.py:57-58, 1371-1372).

The package contract follows ptx_backend.py:1821-1876 ``compile_file``: one
KernelOp per graph (:1840-1844), and the ``meta.json`` kernel entry whose
``entry`` equals the KernelOp name (:1853-1859).
"""

from __future__ import annotations

import ast
import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any


class CompileError(ValueError):
    """An unsupported or inconsistent IR package, diagnosed before any output."""


# Constructor names that may appear in a KernelOp body, with the positional
# field names of the few that are written positionally in Emmy's repr.
_POSITIONAL = {
    "Dim": ("value",),
    "ElementwiseImpl": ("name",),
    "dtype": ("name",),
}
WHITELIST = frozenset({
    "Accum", "Assign", "Axis", "BinaryExpr", "Builtin", "CastExpr", "Cond",
    "CpAsyncCommit", "CpAsyncCopy", "CpAsyncWait", "DataType", "Dim",
    "ElementwiseImpl", "FlatIndex", "FragLayout", "FragmentApply",
    "FragmentRepack", "FragmentRowReduce", "FuncCallExpr", "Init", "Lambda",
    "LdmatrixLoad", "Let", "Literal", "Load", "Loop", "MbarrierArrive",
    "MbarrierArriveExpectTx", "MbarrierInit", "MbarrierWait", "MmaSyncPtx",
    "RegFragment", "RegStore", "Select", "Smem", "StridedLoop", "Sync",
    "TernaryExpr", "Tile", "TmaDescriptor", "TmaLoad", "TreeHalve", "Var",
    "WarpShuffle", "Window", "Write", "dtype",
})


@dataclass(frozen=True)
class Node:
    """One constructor application from the IR ``repr``: ``kind(**fields)``."""

    kind: str
    fields: tuple

    def __getattr__(self, name: str) -> Any:
        for key, value in object.__getattribute__(self, "fields"):
            if key == name:
                return value
        raise AttributeError(f"{object.__getattribute__(self, 'kind')} has no field {name!r}")

    def get(self, name: str, default: Any = None) -> Any:
        for key, value in self.fields:
            if key == name:
                return value
        return default

    def __repr__(self) -> str:  # compact, for diagnostics only
        inner = ", ".join(f"{k}={v!r}" for k, v in self.fields)
        return f"{self.kind}({inner})"


def _evaluate(tree: ast.AST) -> Any:
    if isinstance(tree, ast.Constant):
        return tree.value
    if isinstance(tree, ast.Tuple):
        return tuple(_evaluate(item) for item in tree.elts)
    if isinstance(tree, ast.List):
        return tuple(_evaluate(item) for item in tree.elts)
    if isinstance(tree, ast.UnaryOp) and isinstance(tree.op, ast.USub):
        value = _evaluate(tree.operand)
        if not isinstance(value, (int, float)):
            raise CompileError("negation of a non-number in IR")
        return -value
    if isinstance(tree, ast.Name) and tree.id in ("inf", "nan"):
        return float(tree.id)
    if isinstance(tree, ast.Call):
        if not isinstance(tree.func, ast.Name):
            raise CompileError("IR constructor must be a plain name")
        name = tree.func.id
        if name not in WHITELIST:
            raise CompileError(f"unsupported IR constructor {name}")
        positional = _POSITIONAL.get(name, ())
        if len(tree.args) > len(positional):
            raise CompileError(f"{name}: unexpected positional arguments")
        fields = [(positional[i], _evaluate(arg)) for i, arg in enumerate(tree.args)]
        for keyword in tree.keywords:
            if keyword.arg is None:
                raise CompileError(f"{name}: ** arguments are not IR")
            fields.append((keyword.arg, _evaluate(keyword.value)))
        return Node(name, tuple(fields))
    raise CompileError(f"unsupported IR syntax {type(tree).__name__}")


def parse_body(text: str) -> Node:
    """Parse one KernelOp body statement (a ``repr`` string) into :class:`Node`s."""
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as exc:
        raise CompileError(f"malformed IR body: {exc.msg}") from exc
    return _evaluate(tree.body)


def dtype_name(value: Any) -> str | None:
    """Short dtype name (``f32``, ``f16``, ``bf16`` ...) of a DataType or string."""
    if value is None:
        return None
    if isinstance(value, Node) and value.kind == "DataType":
        return value.name
    if isinstance(value, str):
        return {"float": "f32", "__half": "f16", "half": "f16", "__nv_bfloat16": "bf16",
                "double": "f64", "int": "i32"}.get(value, value)
    raise CompileError(f"not a dtype: {value!r}")


def static_extent(extent: Any) -> int:
    """Integer value of an ``Axis.extent`` (``Dim(n)``), as ``Dim.as_static`` gives it."""
    if isinstance(extent, Node) and extent.kind == "Dim" and isinstance(extent.value, int):
        return extent.value
    if isinstance(extent, int):
        return extent
    raise CompileError(f"dynamic extent {extent!r} is not supported")


@dataclass
class Buffer:
    name: str
    shape: tuple
    dtype: str
    role: str  # "input", "constant", "output"
    constant: Any = None


@dataclass
class KernelPackage:
    """A loaded IR package: the single KernelOp, its buffers and its meta entry."""

    path: Path
    entry: str
    body: tuple
    buffers: dict
    graph_inputs: list
    graph_outputs: list
    meta: dict
    kernel_meta: dict
    arg_order: list
    zero_delegated: list = field(default_factory=list)

    @property
    def rtol(self) -> float:
        return float(self.meta.get("rtol", 0.0))

    @property
    def atol(self) -> float:
        return float(self.meta.get("atol", 0.0))


def load_package(path: str | Path, meta_path: str | Path | None = None) -> KernelPackage:
    """Load ``kernel.ir.json`` and the neighbouring ``meta.json``.

    Mirrors ptx_backend.py:1821-1876: exactly one KernelOp, the meta kernel
    entry matched by name, and ``arg_order`` equal to the node's inputs and
    outputs (ptx_backend.py:1759-1764).
    """
    path = Path(path)
    try:
        graph = json.loads(path.read_text())
    except json.JSONDecodeError as exc:
        raise CompileError(f"{path.name}: invalid JSON: {exc.msg}") from exc
    nodes = graph.get("nodes")
    if not isinstance(nodes, dict):
        raise CompileError(f"{path.name}: graph has no nodes")
    kernels = [(name, node) for name, node in nodes.items() if node.get("op") == "KernelOp"]
    if len(kernels) != 1:
        raise CompileError(f"{path.name}: expected exactly one KernelOp, found {len(kernels)}")
    node_name, kernel = kernels[0]
    fields = kernel.get("op_fields", {})
    entry = fields.get("name")
    if not entry:
        raise CompileError("KernelOp has no name")
    bodies = fields.get("body") or []
    body = tuple(parse_body(text) for text in bodies)
    if fields.get("serial"):
        raise CompileError("serial axes are not supported")

    buffers: dict[str, Buffer] = {}
    for name, node in nodes.items():
        op = node.get("op")
        for out in node.get("outputs", []):
            shape = tuple(out.get("shape") or ())
            role = {"InputOp": "input", "ConstantOp": "constant", "KernelOp": "output"}.get(op)
            if role is None:
                raise CompileError(f"unsupported graph node op {op}")
            constant = node.get("op_fields", {}).get("value") if op == "ConstantOp" else None
            buffers[out["name"]] = Buffer(out["name"], shape, out.get("dtype", "f32"), role, constant)

    meta_path = Path(meta_path) if meta_path else path.with_name("meta.json")
    try:
        meta = json.loads(meta_path.read_text())
    except OSError as exc:
        raise CompileError(f"meta.json not found next to {path.name}") from exc
    matches = [k for k in meta.get("kernels", []) if k.get("entry") == entry]
    if len(matches) != 1:
        raise CompileError(f"meta.json has no unique kernel entry {entry}")
    kernel_meta = matches[0]
    arg_order = list(kernel_meta.get("arg_order", []))
    expected = set(kernel.get("inputs", [])) | {o["name"] for o in kernel.get("outputs", [])}
    if set(arg_order) != expected or len(arg_order) != len(expected):
        raise CompileError(f"meta arg_order {arg_order} does not match kernel arguments {sorted(expected)}")
    by_name = {a["name"]: a for a in kernel_meta.get("args", [])}
    for name in arg_order:
        if name not in buffers:
            raise CompileError(f"argument {name} has no buffer in the graph")
        if name in by_name and "dtype" in by_name[name]:
            buffers[name].dtype = by_name[name]["dtype"]
    return KernelPackage(
        path=path, entry=entry, body=body, buffers=buffers,
        graph_inputs=list(meta.get("graph_inputs", graph.get("inputs", []))),
        graph_outputs=list(meta.get("graph_outputs", graph.get("outputs", []))),
        meta=meta, kernel_meta=kernel_meta, arg_order=arg_order,
        zero_delegated=list(fields.get("zero_delegated", [])),
    )
