"""Which accumulators get compensated (Dot2) accumulation, and how a read sees them.

The reference compiles an f32 dot product accumulation as Dot2 (Ogita, Rump
and Oishi 2005, "Accurate Sum and Dot Product", Algorithm 5.3: TwoProduct by
FMA plus TwoSum, the errors summed in a separate correction;
ptx_backend.py:571-593 ``compensated_dot``) whenever the package's meta.json
has rtol > 0 or atol > 0 (ptx_backend.py:1860-1865, the CLI's default).  An
accumulator qualifies (ptx_backend.py:337-374 ``independent_dots``) when, in
some Loop or StridedLoop body,

* it is updated by an ``Accum`` with no explicit base, operation add / sum,
  directly after the ``Assign`` multiply that defines its value, both f32;
* and nothing in that loop (nested statements included) reads it other than
  its own updates.

Any other ``Accum`` of it in such a loop disqualifies it.  The state is then
a pair (high, low): the adjacent product updates both; a read anywhere yields
``high + (low if high is finite else 0)`` (ptx_backend.py:539-552 ``lookup``);
any other write (a seed, a plain update, a shuffle merge) sets high and
clears low (ptx_backend.py:554-569).  This module finds the qualifying names;
the program compilers emit the arithmetic.
"""
from __future__ import annotations

from .ir import KernelPackage, Node, dtype_name

LOOPS = ("Loop", "StridedLoop")


def enabled(pkg: KernelPackage) -> bool:
    """The reference CLI's policy: compensate when the package states any tolerance."""
    return pkg.rtol > 0 or pkg.atol > 0


def walk(body):
    """Statements of a body, depth first, descending into loops, tiles and conditionals."""
    for s in body:
        if not isinstance(s, Node):
            continue
        yield s
        if s.kind in LOOPS + ("Tile",):
            yield from walk(s.body)
        elif s.kind == "Cond":
            yield from walk(s.body)
            yield from walk(s.get("else_body") or ())


def expr_vars(e) -> set:
    """Names of the Var nodes inside an expression tree."""
    out: set = set()
    stack = [e]
    while stack:
        x = stack.pop()
        if isinstance(x, Node):
            if x.kind == "Var":
                out.add(x.name)
            else:
                stack.extend(v for _, v in x.fields)
        elif isinstance(x, tuple):
            stack.extend(x)
    return out


def _names(value) -> set:
    if value is None:
        return set()
    if isinstance(value, str):
        return {value}
    if isinstance(value, tuple):
        return {v for v in value if isinstance(v, str)}
    return set()


def reads(s: Node) -> set:
    """Names a statement reads: its operands and the free variables of its expressions."""
    k = s.kind
    if k == "Accum":
        return _names(s.value) | _names(s.get("base"))
    if k == "Assign":
        return _names(s.args) | expr_vars(tuple(a for a in s.args if isinstance(a, Node)))
    if k == "Let":
        return _names(s.value) | expr_vars(s.value)
    if k == "Load":
        return expr_vars(s.index)
    if k == "Write":
        return _names(s.values) | expr_vars(s.index)
    if k == "Select":
        out: set = set()
        for br in s.branches:
            out |= _names(br.get("value")) | expr_vars(br.get("select"))
        return out
    if k == "StridedLoop":
        return expr_vars((s.get("start"), s.get("step"), s.get("end")))
    if k == "Cond":
        return expr_vars(s.cond)
    if k in ("WarpShuffle", "TreeHalve"):
        return _names(s.state)
    # any other statement: every Var in its fields except nested bodies
    return expr_vars(tuple(v for key, v in s.fields if key not in ("body", "else_body")))


def _op(s: Node) -> str:
    return s.op.name if isinstance(s.op, Node) else str(s.op)


def adjacent_dot(previous, s: Node) -> bool:
    """``s`` is an Accum add of the f32 product the immediately preceding Assign defines."""
    return (isinstance(previous, Node) and previous.kind == "Assign" and _op(previous) == "multiply"
            and s.kind == "Accum" and s.value == previous.name and s.get("base") is None
            and _op(s) in ("add", "sum")
            and dtype_name(previous.get("dtype")) == dtype_name(s.get("dtype")) == "f32")


def compensated_states(body, pkg: KernelPackage | None = None) -> set:
    """Accumulator names the reference would compensate in this kernel body."""
    if pkg is not None and not enabled(pkg):
        return set()
    eligible: set = set()
    rejected: set = set()
    for loop in walk(body):
        if loop.kind not in LOOPS:
            continue
        inner = [s for s in loop.body if isinstance(s, Node)]
        states = {s.name for s in inner if s.kind == "Accum"}
        for i, s in enumerate(inner):
            if s.kind != "Accum":
                continue
            (eligible if adjacent_dot(inner[i - 1] if i else None, s) else rejected).add(s.name)
        for s in walk(inner):
            rejected |= states & reads(s)
    return eligible - rejected
