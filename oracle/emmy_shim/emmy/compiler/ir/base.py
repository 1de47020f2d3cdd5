"""Generic IR node: keyword fields from the IR repr, value equality, queries."""
from __future__ import annotations


def _freeze(v):
    if isinstance(v, list):
        return tuple(_freeze(x) for x in v)
    if isinstance(v, tuple):
        return tuple(_freeze(x) for x in v)
    return v


class IRNode:
    _positional: tuple = ()
    _defaults: dict = {}

    def __init__(self, *args, **kwargs):
        if len(args) > len(self._positional):
            raise TypeError(f"{type(self).__name__}: too many positional arguments")
        fields = dict(self._defaults)
        fields.update(zip(self._positional, args))
        fields.update(kwargs)
        for k, v in fields.items():
            object.__setattr__(self, k, _freeze(v))
        object.__setattr__(self, "_fields", tuple(fields))

    def _key(self):
        return (type(self).__name__,) + tuple((k, getattr(self, k)) for k in self._fields)

    def __eq__(self, other):
        return isinstance(other, IRNode) and self._key() == other._key()

    def __hash__(self):
        try:
            return hash(self._key())
        except TypeError:
            return id(self)

    def __repr__(self):
        inner = ", ".join(f"{k}={getattr(self, k)!r}" for k in self._fields)
        return f"{type(self).__name__}({inner})"

    # statement queries -------------------------------------------------
    def defines(self):
        return ()

    def deps(self):
        return ()

    def exprs(self):
        return ()


def names(value) -> tuple:
    """Names a field refers to: a string, or strings inside tuples."""
    if value is None:
        return ()
    if isinstance(value, str):
        return (value,)
    if isinstance(value, tuple):
        out = ()
        for v in value:
            out += names(v)
        return out
    return ()


def expressions(value) -> tuple:
    """Expression objects inside a field (tuples flattened)."""
    from .expr import Expr
    if isinstance(value, Expr):
        return (value,)
    if isinstance(value, tuple):
        out = ()
        for v in value:
            out += expressions(v)
        return out
    return ()
