"""Graph.from_dict: the IR package JSON with KernelOp bodies parsed from their repr.

Bodies are parsed with ``ast`` and evaluated against a closed table of node
classes; nothing in the file is executed.
"""
from __future__ import annotations

import ast

import numpy as np

from . import dtype as _dtype
from .ir import elementwise, expr
from .ir.kernel import ir as kernel
from .ir.pure import lam
from .ir.stmt import blocks, leaves

_CLASSES = {}
for _module in (expr, kernel, blocks, leaves, lam, elementwise, _dtype):
    for _name in dir(_module):
        _obj = getattr(_module, _name)
        if isinstance(_obj, type) and _obj.__module__ == _module.__name__:
            _CLASSES[_name] = _obj


def _evaluate(tree):
    if isinstance(tree, ast.Constant):
        return tree.value
    if isinstance(tree, (ast.Tuple, ast.List)):
        return tuple(_evaluate(e) for e in tree.elts)
    if isinstance(tree, ast.UnaryOp) and isinstance(tree.op, ast.USub):
        return -_evaluate(tree.operand)
    if isinstance(tree, ast.Name) and tree.id in ("inf", "nan"):
        return float(tree.id)
    if isinstance(tree, ast.Call) and isinstance(tree.func, ast.Name):
        name = tree.func.id
        args = [_evaluate(a) for a in tree.args]
        kwargs = {k.arg: _evaluate(k.value) for k in tree.keywords}
        if name == "dtype":
            return np.dtype(*args)
        cls = _CLASSES.get(name)
        if cls is None:
            raise ValueError(f"unknown IR constructor {name}")
        return cls(*args, **kwargs)
    raise ValueError(f"unsupported IR syntax {type(tree).__name__}")


def parse(text: str):
    return _evaluate(ast.parse(text, mode="eval").body)


class TensorSpec:
    def __init__(self, name, shape, dtype):
        self.name, self.shape, self.dtype = name, tuple(shape or ()), dtype


class InputOp:
    pass


class ConstantOp:
    def __init__(self, **fields):
        self.__dict__.update(fields)


class GraphNode:
    def __init__(self, name, op, inputs, outputs):
        self.name, self.op, self.inputs, self.outputs = name, op, list(inputs), list(outputs)


class Graph:
    def __init__(self, nodes, inputs, outputs):
        self.nodes, self.inputs, self.outputs = nodes, inputs, outputs

    @classmethod
    def from_dict(cls, data):
        nodes = {}
        for name, node in data["nodes"].items():
            kind = node["op"]
            fields = node.get("op_fields", {})
            if kind == "KernelOp":
                body = tuple(parse(b) for b in fields.get("body", []))
                op = kernel.KernelOp(body=body, name=fields["name"],
                                     zero_delegated=tuple(fields.get("zero_delegated", ())),
                                     serial=tuple(fields.get("serial", ())))
            elif kind == "InputOp":
                op = InputOp()
            elif kind == "ConstantOp":
                op = ConstantOp(**fields)
            else:
                raise ValueError(f"unknown graph node {kind}")
            outputs = [TensorSpec(o["name"], o.get("shape"), o.get("dtype", "f32"))
                       for o in node.get("outputs", [])]
            nodes[name] = GraphNode(name, op, node.get("inputs", []), outputs)
        return cls(nodes, data.get("inputs", []), data.get("outputs", []))
