"""Expression nodes: each reports the variable names it reads (free_vars)."""
from __future__ import annotations

from .base import IRNode


class Expr(IRNode):
    def free_vars(self) -> set:
        out = set()
        for k in self._fields:
            out |= _vars(getattr(self, k))
        return out


def _vars(value) -> set:
    if isinstance(value, Expr):
        return value.free_vars()
    if isinstance(value, tuple):
        out = set()
        for v in value:
            out |= _vars(v)
        return out
    return set()


class Var(Expr):
    _positional = ("name",)

    def free_vars(self):
        return {self.name}


class Literal(Expr):
    _positional = ("value", "dtype")

    def free_vars(self):
        return set()


class Builtin(Expr):
    _positional = ("name",)

    def free_vars(self):
        return set()


class BinaryExpr(Expr):
    _positional = ("op", "left", "right")


class CastExpr(Expr):
    pass


class FlatIndex(Expr):
    pass


class FuncCallExpr(Expr):
    _positional = ("name", "args")


class TernaryExpr(Expr):
    _positional = ("cond", "if_true", "if_false")
