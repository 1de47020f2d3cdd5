"""Compensated dot accumulation (Dot2) for the IR oracles — TEST INFRASTRUCTURE ONLY.

A restatement, for the numpy oracles, of the reference's compensated dot
accumulation (Ogita, Rump and Oishi 2005, "Accurate Sum and Dot Product",
Algorithm 5.3; ptx_backend.py:571-593 ``compensated_dot``) and of the rule
that selects it (ptx_backend.py:337-374 ``independent_dots``; enabled when
meta.json states rtol > 0 or atol > 0, :1860-1865).  It shares no code with
the product's compilers.

* ``compensated(body, pkg)``: the accumulator names the reference compensates —
  an ``Accum`` add / sum with no base directly after the f32 ``Assign``
  multiply that defines its value, inside a Loop / StridedLoop where nothing
  else reads it;
* ``step(hi, lo, a, b)``: one Dot2 update on float32 arrays — the product
  rounded to f32, its exact rounding residual (a*b - p is exact in float64
  and rounded once, which is what an FMA returns), TwoSum of hi and the
  product, both errors summed into lo;
* ``value(hi, lo)``: hi + lo while hi is finite, else hi (ptx_backend.py:539-552).
"""
from __future__ import annotations

import numpy as np


def _name(x) -> str:
    return x.name if hasattr(x, "name") else str(x)


def _walk(body):
    for s in body:
        if not hasattr(s, "kind"):
            continue
        yield s
        if s.kind in ("Loop", "StridedLoop", "Tile"):
            yield from _walk(s.body)
        elif s.kind == "Cond":
            yield from _walk(s.body)
            yield from _walk(s.get("else_body") or ())


def _vars(e, out: set) -> set:
    if hasattr(e, "kind"):
        if e.kind == "Var":
            out.add(e.name)
        else:
            for _, v in e.fields:
                _vars(v, out)
    elif isinstance(e, tuple):
        for v in e:
            _vars(v, out)
    return out


def _strings(v) -> set:
    if isinstance(v, str):
        return {v}
    if isinstance(v, tuple):
        return {x for x in v if isinstance(x, str)}
    return set()


def _reads(s) -> set:
    k = s.kind
    if k == "Accum":
        return _strings(s.value) | _strings(s.get("base"))
    if k in ("WarpShuffle", "TreeHalve"):
        return _strings(s.state)
    if k == "Select":
        out: set = set()
        for br in s.branches:
            out |= _strings(br.get("value")) | _vars(br.get("select"), set())
        return out
    out = set()
    for key, v in s.fields:
        if key in ("body", "else_body", "axis", "dtype", "value_dtype", "op", "name", "names", "output",
                   "input"):
            continue
        out |= _strings(v) if key in ("args", "values", "value") else set()
        _vars(v, out)
    return out


def _dtype(x) -> str | None:
    if x is None:
        return None
    return x.name if hasattr(x, "name") else str(x)


def adjacent(previous, s) -> bool:
    return (previous is not None and previous.kind == "Assign" and _name(previous.op) == "multiply"
            and s.kind == "Accum" and s.value == previous.name and s.get("base") is None
            and _name(s.op) in ("add", "sum")
            and _dtype(previous.get("dtype")) == _dtype(s.get("dtype")) == "f32")


def compensated(body, pkg=None) -> set:
    if pkg is not None and not (float(pkg.meta.get("rtol", 0)) > 0 or float(pkg.meta.get("atol", 0)) > 0):
        return set()
    eligible, rejected = set(), set()
    for loop in _walk(body):
        if loop.kind not in ("Loop", "StridedLoop"):
            continue
        inner = [s for s in loop.body if hasattr(s, "kind")]
        states = {s.name for s in inner if s.kind == "Accum"}
        for i, s in enumerate(inner):
            if s.kind == "Accum":
                (eligible if adjacent(inner[i - 1] if i else None, s) else rejected).add(s.name)
        for s in _walk(inner):
            rejected |= states & _reads(s)
    return eligible - rejected


def step(hi, lo, a, b):
    """(hi, lo) after hi + lo += a * b, float32 arrays, every operation rounded as the reference's."""
    f32 = np.float32
    a, b = np.asarray(a, f32), np.asarray(b, f32)
    hi, lo = np.asarray(hi, f32), np.asarray(lo, f32)
    with np.errstate(all="ignore"):
        p = a * b
        residual = (a.astype(np.float64) * b.astype(np.float64) - p.astype(np.float64)).astype(f32)
        total = hi + p
        delta = total - hi
        error = (hi - (total - delta)) + (p - delta)
        return total, lo + (error + residual)


def value(hi, lo):
    hi, lo = np.asarray(hi, np.float32), np.asarray(lo, np.float32)
    with np.errstate(all="ignore"):
        return hi + np.where(np.isfinite(hi), lo, np.float32(0))
