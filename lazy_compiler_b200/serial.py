"""Serial programs: per-point bodies with runtime loops.

The reference's schedules give some matmul and attention-like IR (the
scalar a02 attention, small contractions) the serial form: every tile point
is one output element, and its thread runs Loop nests with Accum statements
in registers (ptx_backend.py:1496-1554: an s32 induction variable, the
accumulators seeded with their identity on loop entry, ``base`` giving the
coupled online-softmax updates) before a Write.  This module compiles such a
body, when no recogniser takes it, to a register program for
csrc/pointwise.cu:

* the tile axes are the point space; each loop is a runtime loop
  (LOOPB / LOOPE) whose counter is an extra coordinate that loads and
  stores may be affine in;
* an accumulator lives in a fixed register, set to its identity where the
  IR seeds it (a seeded loop's entry, or an Init) and updated in statement
  order as ``op(base or accumulator, value)``;
* values computed before a loop and read inside it stay live for the whole
  loop (the register allocator extends them across the back edge);
* every output element must be written exactly once over the tile points
  and the loop iterations that enclose the write;
* when the package states a tolerance, the dot accumulators the reference
  compensates (``dot2.compensated_states``) carry a second fixed register
  with the Dot2 correction: the product statement's update is TwoProduct by
  FMA plus TwoSum (ptx_backend.py:571-593), every read adds the correction
  while the high part is finite (:539-552), and every other write clears it
  (:554-569).

Loops with a per-thread start, a captured end or a non-unit step, and
conditional statements, are not taken here.
"""
from __future__ import annotations

import math

import numpy as np

from .dot2 import adjacent_dot, compensated_states
from .ir import CompileError, KernelPackage, Node, static_extent
from .pointwise import MAX_AXES, MAX_CODE, MAX_CONST, OP, PointwiseCompiler, Program, Val, vm_type

# Fold identities as Emmy seeds them: max / min start at the finite -1e30 / 1e30
# (an empty lane's state then combines without inf - inf).
IDENTITY = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "prod": 1.0, "maximum": -1e30, "max": -1e30,
            "minimum": 1e30, "min": 1e30, "fmax": -1e30, "fmin": 1e30}


class SerialCompiler(PointwiseCompiler):
    """Lowers a per-point body with runtime loops (see the module docstring)."""

    def __init__(self, pkg: KernelPackage, tile: Node):
        super().__init__(pkg, tile)
        self.tile_axes = len(self.axes)
        self.loop_extents: list = []
        self.loop_ranges: list = []     # (LOOPB pc, LOOPE pc)
        self.loop_stack: list = []      # (depth, extent) of the enclosing loops
        self.accs: dict = {}            # accumulator -> fixed register id
        self.n_fixed = 0
        self.store_loops: list = []     # (buffer, form, enclosing loop slots)
        self.active: dict = {}          # loop variable -> its coordinate in the innermost enclosing loop
        self.compensated = compensated_states(tuple(tile.body), pkg)
        self.lows: dict = {}            # compensated accumulator -> fixed register of its correction
        self.previous = None            # the statement before the current one in its body

    def affine(self, e) -> dict:
        if isinstance(e, Node) and e.kind == "Var" and e.name in self.active:
            return {self.active[e.name]: 1}
        if isinstance(e, Node) and e.kind == "Var" and e.name not in self.axes[:self.tile_axes]:
            raise CompileError(f"index variable {e.name!r} is not a tile axis or an enclosing loop")
        return super().affine(e)

    def expr(self, e) -> Val:
        if isinstance(e, Node) and e.kind == "Var" and e.name in self.active and e.name not in self.env:
            # an enclosing loop's counter as a value (s32)
            return self.emit("COORD", "s32", aux=self.axes.index(self.active[e.name]))
        if isinstance(e, Node) and e.kind == "Var" and e.name not in self.env and \
                e.name not in self.axes[:self.tile_axes]:
            raise CompileError(f"{e.name!r} is not a tile axis, an enclosing loop or a value")
        return super().expr(e)

    # ------------------------------------------------------------ statements
    def statement(self, s: Node) -> None:
        k = s.kind
        if k in ("Loop", "StridedLoop"):
            self.loop(s)
        elif k == "Accum":
            self.accum(s)
        elif k == "Init":
            reg = self.acc_register(s.name)
            self.put(reg, self.literal(float(s.identity), vm_type(s.get("dtype") or "f32")))
            self.clear_low(s.name)
        elif k == "Write":
            before = len(self.writes)
            super().statement(s)
            for buffer, form in self.writes[before:]:
                self.store_loops.append((buffer, form, tuple(self.loop_stack)))
        elif k in ("Load", "Let", "Assign", "Select"):
            super().statement(s)
        else:
            raise CompileError(f"{k} is not part of a serial program")

    def acc_register(self, name: str) -> int:
        if name not in self.accs:
            self.accs[name] = -1 - self.n_fixed
            self.n_fixed += 1
        reg = self.accs[name]
        self.env[name] = Val(reg, "f32")
        return reg

    def put(self, reg: int, v: Val) -> None:
        self.code.append((OP["MOV"], reg, self.convert(v, "f32").reg, 0, 0, 0, 1, True))

    # ------------------------------------------------------------ compensated (Dot2) states
    def low_register(self, name: str) -> int:
        if name not in self.lows:
            self.lows[name] = -1 - self.n_fixed
            self.n_fixed += 1
        return self.lows[name]

    def clear_low(self, name: str) -> None:
        if name in self.compensated:
            self.put(self.low_register(name), self.literal(0.0, "f32"))

    def lookup(self, name: str) -> Val:
        v = super().lookup(name)
        if name in self.compensated and name in self.accs and v.reg == self.accs[name]:
            # high + correction while high is finite (a non-finite high stays as it is)
            low = Val(self.low_register(name), "f32")
            finite = self.compare("lt", self.emit("FABS", "f32", v), self.literal(float("inf"), "f32"))
            return self.emit("FADD", "f32", v, self.select(finite, low, self.literal(0.0, "f32"), "f32"))
        return v

    def compensated_dot(self, s: Node, product: Node) -> None:
        """Dot2 step: TwoProduct residual by FMA, TwoSum of high and the product, correction sum."""
        hi = Val(self.acc_register(s.name), "f32")
        lo = Val(self.low_register(s.name), "f32")
        p = self.convert(self.lookup(product.name), "f32")
        a, b = (self.convert(self.lookup(n) if isinstance(n, str) else self.expr(n), "f32") for n in product.args)
        residual = self.fma(a, b, self.emit("FNEG", "f32", p))
        total = self.emit("FADD", "f32", hi, p)
        delta = self.emit("FSUB", "f32", total, hi)
        error = self.emit("FADD", "f32", self.emit("FSUB", "f32", hi, self.emit("FSUB", "f32", total, delta)),
                          self.emit("FSUB", "f32", p, delta))
        self.put(lo.reg, self.emit("FADD", "f32", lo, self.emit("FADD", "f32", error, residual)))
        self.put(hi.reg, total)
        self.env[s.name] = hi

    def accum(self, s: Node) -> None:
        op = s.op.name if isinstance(s.op, Node) else str(s.op)
        dt = vm_type(s.get("dtype") or "f32")
        if dt != "f32":
            raise CompileError("serial accumulators are f32")
        if s.name in self.compensated and adjacent_dot(self.previous, s):
            self.compensated_dot(s, self.previous)
            return
        reg = self.acc_register(s.name)
        base = self.lookup(s.base) if s.get("base") else self.lookup(s.name)
        value = self.lookup(s.value) if isinstance(s.value, str) else self.expr(s.value)
        new = self.operation(op, [self.convert(base, "f32"), self.convert(value, "f32")], "f32")
        self.put(reg, new)
        self.clear_low(s.name)
        self.env[s.name] = Val(reg, "f32")

    def loop(self, s: Node) -> None:
        if s.kind == "StridedLoop":
            start, step = s.get("start"), s.get("step")
            if s.get("end") is not None or not _is_int(start, 0) or not _is_int(step, 1):
                raise CompileError("serial loops count from 0 in steps of 1 over their extent")
        extent = static_extent(s.axis.extent)
        depth = len(self.loop_stack)       # loops at one depth are never active together
        if self.tile_axes + depth + 1 > MAX_AXES:
            raise CompileError("loops nested too deep for a serial program")
        internal = f"#{depth}"
        if depth == len(self.loop_extents):
            self.loop_extents.append(extent)
            self.axes.append(internal)
            self.extents = tuple(self.extents) + (extent,)
        else:
            self.loop_extents[depth] = max(self.loop_extents[depth], extent)
            self.extents = tuple(self.extents[:self.tile_axes + depth]) + (extent,) + \
                tuple(self.extents[self.tile_axes + depth + 1:])
        outer_binding = self.active.get(s.axis.name)
        self.active[s.axis.name] = internal
        if s.get("seed", True):
            for inner in s.body:
                if isinstance(inner, Node) and inner.kind == "Accum":
                    op = inner.op.name if isinstance(inner.op, Node) else str(inner.op)
                    if op not in IDENTITY:
                        raise CompileError(f"no identity for accumulator operation {op}")
                    self.put(self.acc_register(inner.name), self.literal(IDENTITY[op], "f32"))
                    self.clear_low(inner.name)
        self.__dict__["_memo"] = {}
        count = self.literal(extent, "s32")
        begin = len(self.code)
        self.code.append(None)
        self.loop_stack.append((depth, extent))
        saved = dict(self.env)
        previous = None
        for inner in s.body:
            self.previous = previous
            self.statement(inner)
            previous = inner
        # names bound inside the loop go out of scope; accumulators stay visible
        self.env = {**saved, **{n: Val(r, "f32") for n, r in self.accs.items()}}
        self.loop_stack.pop()
        if outer_binding is None:
            self.active.pop(s.axis.name, None)
        else:
            self.active[s.axis.name] = outer_binding
        self.__dict__["_memo"] = {}
        end = len(self.code)
        self.code.append(None)
        self.code[begin] = (OP["LOOPB"], 0, count.reg, 0, 0, depth | end << 4, 1, False)
        self.code[end] = (OP["LOOPE"], 0, count.reg, 0, 0, depth | begin << 4, 1, False)
        self.loop_ranges.append((begin, end))

    # ------------------------------------------------------------ registers
    def allocate(self) -> list:
        """Linear scan, with values read inside a loop but defined before it kept
        allocated to the loop's end (the back edge reads them again)."""
        defined: dict = {}
        for pc, (op, dst, a, b, c, aux, nsrc, has_dst) in enumerate(self.code):
            if has_dst and dst >= 0:
                defined.setdefault(dst, pc)
        extend: dict = {}
        for begin, end in self.loop_ranges:
            for pc in range(begin, end + 1):
                op, dst, a, b, c, aux, nsrc, has_dst = self.code[pc]
                for r in (a, b, c)[:nsrc]:
                    if r >= 0 and defined.get(r, 0) < begin:
                        extend[r] = max(extend.get(r, 0), end)
        return super().allocate(extend)

    # ------------------------------------------------------------ finishing
    def serial_coverage(self) -> str:
        outs = {b for b, _, _ in self.store_loops}
        if len(outs) != 1:
            raise CompileError("serial programs write one output")
        out = outs.pop()
        size = math.prod(self.pkg.buffers[out].shape or (1,))
        points = math.prod(self.extents[:self.tile_axes])
        total = sum(points * math.prod(ext for _, ext in loops) for _, _, loops in self.store_loops)
        if total != size or total > (1 << 26):
            raise CompileError(f"serial writes cover {total} elements of {out} ({size})")
        seen = np.zeros(size, np.int64)
        for _, f, loops in self.store_loops:
            form = self.forms[f]
            dims = list(range(self.tile_axes)) + [self.tile_axes + depth for depth, _ in loops]
            sizes = list(self.extents[:self.tile_axes]) + [ext for _, ext in loops]
            grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for e in sizes], indexing="ij")
            flat = form.base + sum(form.coef[d] * g for d, g in zip(dims, grids))
            np.add.at(seen, np.asarray(flat).ravel(), 1)
        if np.any(seen != 1):
            raise CompileError("serial writes do not cover the output exactly once")
        return out

    def compile_serial(self, body: tuple) -> Program:
        previous = None
        for s in body:
            self.previous = previous
            self.statement(s)
            previous = s
        if not self.store_loops:
            raise CompileError("serial program writes nothing")
        out = self.serial_coverage()
        n_coords = self.tile_axes + len(self.loop_extents)
        for f in self.forms:
            f.coef = tuple(f.coef) + (0,) * (n_coords - len(f.coef))
        code, nregs = self.allocate()
        if len(code) > MAX_CODE or len(self.consts) > MAX_CONST:
            raise CompileError("serial program too long")
        consts = [0] * len(self.consts)
        for word, i in self.consts.items():
            consts[i] = word
        names = list(self.slots)
        prog = Program(code, consts, self.forms, names, tuple(self.extents[:self.tile_axes]), nregs,
                       [math.prod(self.pkg.buffers[b].shape or (1,)) for b in names], list(self.loop_extents))
        self.out = out
        return prog


def _is_int(e, value: int) -> bool:
    if e is None:
        return True
    if isinstance(e, int):
        return e == value
    return isinstance(e, Node) and e.kind == "Literal" and e.value == value


def compile_serial(pkg: KernelPackage, tile: Node):
    """Plan of a per-point body with runtime loops as a serial program."""
    from .recognize import _plan
    comp = SerialCompiler(pkg, tile)
    prog = comp.compile_serial(tuple(tile.body))
    bind = {f"buf{i}": name for i, name in enumerate(prog.buffers)}
    return _plan(pkg, "pointwise", "lc_pointwise", bind,
                 {"program": prog.to_json(), "out": comp.out, "points": math.prod(prog.extents), "serial": True},
                 {name: pkg.buffers[name].dtype for name in prog.buffers})


