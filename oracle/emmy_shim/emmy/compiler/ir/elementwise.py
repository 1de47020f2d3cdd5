"""Elementwise operation implementations: the name and the fold identity.

The max/min fold identities are the finite -1e30 / 1e30 that Emmy's own
generated CUDA seeds them with (problems/f02_row_softmax/*.ref.cu).
"""
from __future__ import annotations


from .base import IRNode

_IDENTITY = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "prod": 1.0,
             "maximum": -1e30, "fmax": -1e30, "minimum": 1e30, "fmin": 1e30}


class ElementwiseImpl(IRNode):
    _positional = ("name",)

    @property
    def identity(self):
        return _IDENTITY.get(self.name)
