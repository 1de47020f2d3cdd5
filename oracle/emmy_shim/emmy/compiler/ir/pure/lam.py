from __future__ import annotations

from ..base import IRNode


class Lambda(IRNode):
    pass
