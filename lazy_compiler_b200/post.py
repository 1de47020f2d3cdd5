"""Epilogue programs: any f32 function of a GEMM's accumulator, run after the
GEMM as one pointwise register program over the (row, column) points of C.

The reference's staged scalar matmul (ptx_backend.py:1496-1554 Loop / Accum,
:1597-1631 Write) stores an expression of each accumulator: the accumulator
itself for a plain product, or ``f(acc, bias[col], x[row, col], scalars)``
when the frontend fuses elementwise operations into the matmul kernel.  The
GEMM kernels take the accumulator and a bias / GELU epilogue; any other
expression is applied here instead: the GEMM writes the accumulators to C,
then this program reads C[row, col] back, evaluates the expression with the
reference's scalar rules (the same lowering as pointwise programs) and
stores the result over it.  Each point reads and writes only its own
element, so running it in place is exact.

The expression arrives from the recogniser's symbolic evaluation with the
accumulator replaced by ``("acc",)`` and every load index component named
``"row"`` / ``"col"`` (plus an offset) or a constant.
"""
from __future__ import annotations

import math

from .ir import CompileError, KernelPackage
from .pointwise import MAX_CODE, PointwiseCompiler, Program, Val, _STORAGE, vm_type

ROW, COL = "#row", "#col"


class EpilogueCompiler(PointwiseCompiler):
    """Compiles a normalised epilogue expression over the points of C."""

    def __init__(self, pkg: KernelPackage, out: str, m: int, n: int):
        self.setup(pkg, [ROW, COL], (m, n))
        self.out = out

    def affine(self, e) -> dict:
        if isinstance(e, dict):
            return e
        return super().affine(e)

    def index(self, component) -> dict:
        if isinstance(component, int):
            return {1: component}
        axis, offset = component
        return {ROW if axis == "row" else COL: 1, 1: offset}

    def load(self, buffer: str, index: tuple) -> Val:
        buf = self.pkg.buffers.get(buffer)
        if buf is None:
            raise CompileError(f"epilogue reads unknown buffer {buffer}")
        dt = vm_type(buf.dtype)
        if dt not in _STORAGE:
            raise CompileError(f"epilogue cannot read {buf.dtype}")
        f = self.form(buffer, tuple(self.index(c) for c in index) or ({1: 0},), 0)
        return self.emit("LD_" + _STORAGE[dt], dt, aux=f)

    def value(self, e) -> Val:
        kind = e[0]
        if kind == "acc":
            return self.acc
        if kind == "lit":
            return self.literal(float(e[1]), "f32")
        if kind == "s":
            return self.load(e[1], ())
        if kind == "ld":
            return self.load(e[1], e[2])
        if kind == "cast":
            return self.convert(self.value(e[2]), e[1])
        if kind == "op":
            args = [self.value(a) for a in e[2:]]
            return self.operation(e[1], args, self.assign_type(e[1], args))
        raise CompileError(f"unsupported epilogue term {kind}")

    def compile_epilogue(self, expr) -> Program:
        here = self.form(self.out, ({ROW: 1}, {COL: 1}), 0)
        self.acc = self.emit("LD_F32", "f32", aux=here)
        result = self.convert(self.value(expr), "f32")
        self.emit("ST_F32", None, result, aux=here)
        code, nregs = self.allocate()
        if len(code) > MAX_CODE:
            raise CompileError("epilogue program too long")
        consts = [0] * len(self.consts)
        for word, i in self.consts.items():
            consts[i] = word
        return Program(code, consts, self.forms, list(self.slots), self.extents, nregs,
                       [math.prod(self.pkg.buffers[b].shape or (1,)) for b in self.slots])


def compile_epilogue(pkg: KernelPackage, expr, out: str, m: int, n: int) -> dict:
    """``params["post"]`` of a plan: the program and its buffer binding."""
    prog = EpilogueCompiler(pkg, out, m, n).compile_epilogue(expr)
    return {"program": prog.to_json(), "bind": {f"buf{i}": name for i, name in enumerate(prog.buffers)},
            "points": m * n}
