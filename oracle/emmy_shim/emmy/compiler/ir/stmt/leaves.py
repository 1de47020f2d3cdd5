"""Leaf statements: what each defines and which names and expressions it reads."""
from __future__ import annotations

from ..base import IRNode, expressions, names


class Load(IRNode):
    def defines(self):
        return tuple(self.names)

    def exprs(self):
        return expressions(self.index)


class Write(IRNode):
    def deps(self):
        return names(self.values)

    def exprs(self):
        return expressions(self.index)


class Assign(IRNode):
    def defines(self):
        return (self.name,)

    def deps(self):
        return names(self.args)


class Let(IRNode):
    def defines(self):
        return (self.name,)

    def deps(self):
        return names(self.value)

    def exprs(self):
        return expressions(self.value)


class Init(IRNode):
    def defines(self):
        return (self.name,)


class Accum(IRNode):
    _defaults = {"base": None}

    def defines(self):
        return (self.name,)

    def deps(self):
        return names(self.value) + names(self.base)


class Select(IRNode):
    def defines(self):
        return (self.name,)

    def deps(self):
        return tuple(n for b in getattr(self, "branches", ()) for n in names(getattr(b, "value", None)))

    def exprs(self):
        return tuple(e for b in getattr(self, "branches", ()) for e in expressions(getattr(b, "select", None)))
