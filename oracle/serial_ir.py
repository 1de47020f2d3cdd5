"""CPU oracle of per-point bodies with runtime loops — TEST INFRASTRUCTURE ONLY.

Evaluates a Tile whose every point runs Loop nests with Accum statements
(the reference's serial schedule, ptx_backend.py:1496-1554) over all points
at once with numpy: each loop runs its iterations in order with the loop
variable a constant of that iteration, an accumulator starts at its
operation's identity on entry to a seeding loop (or at its Init) and is
updated as op(base or accumulator, value) in statement order.  Scalar rules
and accurate float64 transcendentals come from oracle/pointwise_ir.py.  When
the package states a tolerance, the dot accumulators the reference
compensates are Dot2 pairs (oracle/dot2_ir.py): the adjacent product update
is a Dot2 step, every read sees hi + lo, every other write clears lo.
"""
from __future__ import annotations

import numpy as np

from oracle import dot2_ir
from oracle.pointwise_ir import PointwiseOracle, V, conv

# Fold identities as Emmy seeds them: max / min start at the finite -1e30 / 1e30
# (an empty lane's state then combines without inf - inf).
_IDENTITY = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "prod": 1.0, "maximum": -1e30, "max": -1e30,
             "minimum": 1e30, "min": 1e30, "fmax": -1e30, "fmin": 1e30}


class SerialOracle(PointwiseOracle):
    def set_state(self, name, hi, lo=None) -> None:
        """An accumulator's new value; a compensated one keeps (hi, lo) and is read as their value."""
        comp = self.__dict__.setdefault("comp", dot2_ir.compensated(self.pkg.body, self.pkg))
        if name in comp:
            n = len(np.asarray(hi.a if isinstance(hi, V) else hi).ravel())
            hi_a = np.asarray(hi.a if isinstance(hi, V) else hi, np.float32)
            lo_a = np.zeros(n, np.float32) if lo is None else lo
            self.__dict__.setdefault("dot2", {})[name] = (hi_a, lo_a)
            self.env[name] = V(dot2_ir.value(hi_a, lo_a), "f32")
        else:
            self.env[name] = hi if isinstance(hi, V) else V(np.asarray(hi, np.float32), "f32")

    def run_serial(self, body) -> dict:
        n = len(next(iter(self.coord.values())))
        previous = None
        for s in body:
            prev, previous = previous, s
            k = s.kind
            if k in ("Loop", "StridedLoop"):
                extent = int(s.axis.extent.value)
                if s.get("seed", True):
                    for inner in s.body:
                        if inner.kind == "Accum":
                            opname = inner.op.name if hasattr(inner.op, "name") else str(inner.op)
                            self.set_state(inner.name, V(np.full(n, _IDENTITY[opname], np.float32), "f32"))
                saved = dict(self.env)
                for v in range(extent):
                    self.coord[s.axis.name] = np.full(n, v, np.int64)
                    self.run_serial(s.body)
                # names bound in the loop go out of scope; accumulators keep their values
                kept = {a: self.env[a] for a in _accumulators(s.body) if a in self.env}
                self.env = {**saved, **kept}
                self.coord.pop(s.axis.name, None)
                continue
            elif k == "Accum" and s.name in self.__dict__.get("dot2", {}) and dot2_ir.adjacent(prev, s):
                hi, lo = self.dot2[s.name]
                a, b = (conv(self.env[x] if isinstance(x, str) else self.expr(x), "f32").a for x in prev.args)
                self.set_state(s.name, *dot2_ir.step(hi, lo, a, b))
            elif k == "Accum":
                opname = s.op.name if hasattr(s.op, "name") else str(s.op)
                base = self.env[s.base] if s.get("base") else self.env[s.name]
                value = self.env[s.value] if isinstance(s.value, str) else self.expr(s.value)
                self.set_state(s.name, conv(self.op(opname, [conv(base, "f32"), conv(value, "f32")], "f32"), "f32"))
            elif k == "Init":
                self.set_state(s.name, V(np.full(n, float(s.identity), np.float32), "f32"))
            else:
                self.run([s])
        return {k: v.reshape(tuple(self.pkg.buffers[k].shape) or (1,)) for k, v in self.out.items()}


def _accumulators(body) -> set:
    names = set()
    for s in body:
        if s.kind == "Accum":
            names.add(s.name)
        elif s.kind in ("Loop", "StridedLoop"):
            names |= _accumulators(s.body)
    return names


def evaluate(ir_path, arrays: dict) -> dict:
    """Outputs of the serial package at ``ir_path`` on named input arrays."""
    from lazy_compiler_b200.ir import load_package
    pkg = load_package(ir_path)
    (tile,) = pkg.body
    return SerialOracle(pkg, tile, arrays).run_serial(tile.body)
