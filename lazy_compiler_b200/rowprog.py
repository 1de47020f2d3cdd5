"""Row programs: reductions and fused row operations of any op mix.

The reference's categories 2 and 4 (ptx_backend.py:1496-1744) share one
shape: a Tile over [row,] cooperating threads; StridedLoop passes that
stride the threads over the row's columns, Accum statements folding
per-element expressions into accumulators, WarpShuffle / TreeHalve combines
across the block, then either a guarded per-row Write of expressions of the
accumulators or a further pass writing per-element expressions of them.
The fixed kernels cover sum, mean, row sum, RMSNorm, softmax, L2 norm and
row dot products at full bandwidth; this module compiles every other such
body to a row program for csrc/pointwise.cu's ``lc_rowprog``:

* each pass's per-element expressions compile, with the scalar rules of
  pointwise programs, to register operations over (row, column); each
  accumulator's value feeds an ACC operation into its state;
* after the pass the states combine across the CTA in a fixed order (their
  Accum operation: add, multiply, maximum or minimum) and later passes and
  the final per-row writes read them with STATE;
* every written element must be written exactly once.

Accumulators that fold through an explicit ``base`` (coupled online states)
are not taken here; the online softmax has its own kernel.
"""
from __future__ import annotations

import math

import numpy as np

from .ir import CompileError, KernelPackage, Node, static_extent
from .pointwise import MAX_CODE, MAX_CONST, PointwiseCompiler, Program, Val

MAX_PASSES = 4
MAX_STATES = 8
FOLDS = {"add": 0, "multiply": 1, "maximum": 2, "minimum": 3}


def _aff_dict(form) -> dict:
    return {term: coef for term, coef in form}


class RowProgramCompiler(PointwiseCompiler):
    """Compiles the symbolic form of a row-reduction Tile (see the module docstring)."""

    def __init__(self, pkg: KernelPackage, tile: Node, ev):
        axes = [(a.name, static_extent(a.extent)) for a in tile.axes]
        if not 1 <= len(axes) <= 2:
            raise CompileError("row programs take a [row,] cooperative Tile")
        self.pkg = pkg
        self.ev = ev
        self.co, self.block = axes[-1]
        block = tile.get("block_threads") or self.block
        if block != self.block:
            raise CompileError("the cooperative axis must span the block")
        self.row = axes[0][0] if len(axes) == 2 else "__row"
        self.rows = axes[0][1] if len(axes) == 2 else 1
        self.code, self.consts, self.forms, self.form_index = [], {}, [], {}
        self.slots, self.env, self.nvreg, self.writes = {}, {}, 0, []
        self.state_slot: dict = {}
        self.state_op: list = []
        self.state_pass: list = []
        self.pass_ranges: list = []
        self.pass_writes: list = []      # (buffer, form) of per-element writes
        self.final_writes: list = []     # (buffer, form) of per-row writes
        self.cols = None

    # ------------------------------------------------------------ symbolic expressions
    def sym(self, e) -> Val:
        if isinstance(e, tuple) and e:
            tag = e[0]
            if tag == "lit":
                return self.literal(float(e[1]), "f32")
            if tag == "ld":
                _, buf, index = e
                b = self.pkg.buffers.get(buf)
                if b is None:
                    raise CompileError(f"load from unknown buffer {buf}")
                dt = {"f32": "f32", "f16": "f16", "bf16": "bf16"}.get(b.dtype)
                if dt is None:
                    raise CompileError(f"row programs load f32, f16 or bf16, not {b.dtype}")
                f = self.sym_form(buf, index)
                return self.convert(self.emit("LD_" + dt.upper(), dt, aux=f), "f32")
            if tag in ("red", "acc"):
                if e[1] not in self.state_slot:
                    raise CompileError(f"{e[1]} is read before its pass completes")
                return self.emit("STATE", "f32", aux=self.state_slot[e[1]])
            if tag == "cast":
                return self.convert(self.sym(e[2]), e[1])
            if tag == "op":
                args = [self.sym(a) for a in e[2:]]
                return self.convert(self.operation(e[1], args, "f32"), "f32")
        raise CompileError(f"unsupported expression in a row program: {e!r}")

    def sym_form(self, buf: str, index: tuple) -> int:
        shape = tuple(self.pkg.buffers[buf].shape) or (1,)
        total: dict = {}
        if len(index) == 1 or (len(index) > 1 and len(index) != len(shape)):
            parts = [(_aff_dict(i), 1) for i in index]
        else:
            parts = [(_aff_dict(i), math.prod(shape[d + 1:])) for d, i in enumerate(index)]
        for aff, stride in parts:
            for term, coef in aff.items():
                if not (term == 1 or term in self.axes):
                    raise CompileError(f"row-program index depends on {term!r}")
                total[term] = total.get(term, 0) + coef * stride
        base = total.pop(1, 0)
        coef = tuple(total.get(a, 0) for a in self.axes)
        size = math.prod(shape)
        lo = base + sum(min(0, c * (e - 1)) for c, e in zip(coef, self.extents))
        hi = base + sum(max(0, c * (e - 1)) for c, e in zip(coef, self.extents))
        if lo < 0 or hi >= size:
            raise CompileError(f"index of {buf} leaves the buffer")
        if buf not in self.slots:
            self.slots[buf] = len(self.slots)
        key = (buf, base, coef)
        if key not in self.form_index:
            if len(self.forms) >= 32:
                raise CompileError("row program has too many distinct indices")
            from .pointwise import Form, vm_type
            self.form_index[key] = len(self.forms)
            self.forms.append(Form(self.slots[buf], vm_type(self.pkg.buffers[buf].dtype), base, coef))
        return self.form_index[key]

    def store(self, w: dict, final: bool) -> None:
        buf = self.pkg.buffers.get(w["buffer"])
        if buf is None or buf.role != "output":
            raise CompileError("row programs write the kernel's outputs only")
        if w["atomic"]:
            raise CompileError("row programs do not take atomic writes")
        dt = {"f32": "F32", "f16": "F16", "bf16": "BF16"}.get(buf.dtype)
        if dt is None:
            raise CompileError(f"row programs write f32, f16 or bf16, not {buf.dtype}")
        for lane, value in enumerate(w["values"]):
            index = w["index"]
            if lane:   # a vector write stores consecutive elements along the last dimension
                index = index[:-1] + (_add_const(index[-1], lane),)
            f = self.sym_form(w["buffer"], index)
            v = self.convert(self.sym(value), buf.dtype)
            self.emit("ST_" + dt, None, v, aux=f)
            (self.final_writes if final else self.pass_writes).append((w["buffer"], f))

    # ------------------------------------------------------------ structure
    def compile_rows(self) -> tuple:
        ev = self.ev
        loops = ev.loops
        if not loops or len(loops) > MAX_PASSES:
            raise CompileError("row programs take one to four passes")
        for loop in loops:
            if loop.get("parent") is not None:
                raise CompileError("row-program passes are not nested")
            if loop["start"] != frozenset({(self.co, 1)}) or loop["step"] != self.block:
                raise CompileError("each pass must stride the block's threads over the row")
            if "end" in loop:
                raise CompileError("row-program passes run over the whole row")
            if self.cols is None:
                self.cols = loop["extent"]
            elif loop["extent"] != self.cols:
                raise CompileError("row-program passes cover different column counts")
        reds = ev.reductions
        combined = ev.trees | ev.shuffled
        for name, red in reds.items():
            if red["base"] is not None:
                raise CompileError("accumulators with an explicit base (coupled states) are not row programs")
            if red["op"] not in FOLDS:
                raise CompileError(f"accumulator operation {red['op']} is not add, multiply, maximum or minimum")
            if name not in combined:
                raise CompileError(f"accumulator {name} is not combined across the block")
        if len(reds) > MAX_STATES:
            raise CompileError("row program has too many accumulators")
        self.extents = (self.rows, self.cols)
        for p, loop in enumerate(loops):
            self.axes = [self.row, loop["axis"]]
            begin = len(self.code)
            accs = [n for n in loop["accums"] if n in reds]
            for name in accs:
                value = self.sym(reds[name]["value"])
                slot = len(self.state_op)
                self.emit("ACC", None, value, aux=slot)
                self.state_op.append(FOLDS[reds[name]["op"]])
                self.state_pass.append(p)
            for w in ev.writes:
                if w["loop"] == loop["axis"]:
                    if w["cond"]:
                        raise CompileError("conditional writes inside a row pass are not supported")
                    self.store(w, final=False)
            self.pass_ranges.append((begin, len(self.code)))
            for slot, name in zip(range(len(self.state_op) - len(accs), len(self.state_op)), accs):
                self.state_slot[name] = slot
        self.axes = [self.row, "__col"]
        final_begin = len(self.code)
        for w in ev.writes:
            if w["loop"] is None:
                if w["cond"] and not self.lead_guard(w["cond"]):
                    raise CompileError("per-row writes must be unconditional or guarded to one thread")
                self.store(w, final=True)
        final_end = len(self.code)
        if not self.pass_writes and not self.final_writes:
            raise CompileError("row program writes nothing")
        self.check_coverage()
        return final_begin, final_end

    def lead_guard(self, conds) -> bool:
        c = conds[0] if len(conds) == 1 else None
        return (c is not None and c.kind == "BinaryExpr" and c.op == "==" and c.left.kind == "Var"
                and c.left.name == self.co and c.right.kind == "Literal" and c.right.value == 0)

    def check_coverage(self) -> None:
        outs = {b for b, _ in self.pass_writes + self.final_writes}
        rows = np.arange(self.rows, dtype=np.int64)
        for out in outs:
            size = math.prod(self.pkg.buffers[out].shape or (1,))
            if size > (1 << 26):
                raise CompileError("row-program outputs above 2^26 elements are not verified")
            seen = np.zeros(size, np.int64)
            for b, f in self.pass_writes:
                if b != out:
                    continue
                form = self.forms[f]
                r, c = np.meshgrid(rows, np.arange(self.cols, dtype=np.int64), indexing="ij")
                np.add.at(seen, (form.base + form.coef[0] * r + form.coef[1] * c).ravel(), 1)
            for b, f in self.final_writes:
                if b != out:
                    continue
                form = self.forms[f]
                np.add.at(seen, form.base + form.coef[0] * rows, 1)
            if np.any(seen != 1):
                raise CompileError(f"row-program writes do not cover {out} exactly once")

    def layout(self, final: tuple) -> dict:
        return {"passes": [list(r) for r in self.pass_ranges], "final": list(final),
                "state_op": list(self.state_op), "state_pass": list(self.state_pass)}


def _add_const(form, k: int):
    d = dict(form)
    d[1] = d.get(1, 0) + k
    return frozenset((t, c) for t, c in d.items() if c != 0)


def _check_combines(tile: Node, reds: dict) -> None:
    """Each WarpShuffle / TreeHalve combine must fold a state with its partner
    by the state's own Accum operation (state = op(state, partner))."""
    from .recognize import _walk
    for s in _walk(tile.body):
        if s.kind not in ("WarpShuffle", "TreeHalve"):
            continue
        pairs = dict(zip(s.state, s.state_b))
        for a in s.get("combine_states") or ():
            op = a.op.name if isinstance(a.op, Node) else str(a.op)
            name = a.name
            if a.kind != "Assign" or name not in pairs or tuple(a.args) != (name, pairs[name]):
                raise CompileError("a combine step is not state = op(state, partner)")
            if name in reds and op != reds[name]["op"]:
                raise CompileError(f"{name} combines by {op} but accumulates by {reds[name]['op']}")


def compile_rowprog(pkg: KernelPackage, tile: Node, ev):
    """Plan of a reduction / fused row Tile as a row program."""
    from .recognize import _plan
    _check_combines(tile, ev.reductions)
    comp = RowProgramCompiler(pkg, tile, ev)
    final = comp.compile_rows()
    code, nregs = comp.allocate()
    if len(code) > MAX_CODE or len(comp.consts) > MAX_CONST:
        raise CompileError("row program too long")
    consts = [0] * len(comp.consts)
    for word, i in comp.consts.items():
        consts[i] = word
    names = list(comp.slots)
    prog = Program(code, consts, comp.forms, names, (comp.rows, comp.cols), nregs,
                   [math.prod(pkg.buffers[b].shape or (1,)) for b in names])
    bind = {f"buf{i}": name for i, name in enumerate(names)}
    outs = sorted({b for b, _ in comp.pass_writes + comp.final_writes})
    return _plan(pkg, "rowprog", "lc_rowprog", bind,
                 {"program": prog.to_json(), "layout": comp.layout(final), "out": outs[0],
                  "rows": comp.rows, "cols": comp.cols},
                 {name: pkg.buffers[name].dtype for name in names})
