"""Block statements: conditionals and loops."""
from __future__ import annotations

from ..base import IRNode, expressions


class Cond(IRNode):
    _defaults = {"else_body": ()}

    def exprs(self):
        return expressions(self.cond)


class Loop(IRNode):
    pass


class StridedLoop(IRNode):
    _defaults = {"end": None}

    def exprs(self):
        return expressions((self.start, self.step, self.end))
