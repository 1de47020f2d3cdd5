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
  pointwise programs, to register operations over (row, column); every
  Accum is an explicit update of the thread's running partial
  (``partial = op(base or partial, value)``, PARTIAL / SETP), in statement
  order, so coupled online states (the f02 softmax's max and rescaled sum)
  are as expressible as plain sums;
* after the pass the partials combine with the Tile's own combine programs:
  the WarpShuffle's ``combine_states`` at every level of a lane butterfly,
  the TreeHalve's across the warps in order; later passes and the final
  per-row writes read the combined states with STATE;
* every written element must be written exactly once.
"""
from __future__ import annotations

import math

import numpy as np

from .ir import CompileError, KernelPackage, Node, static_extent
from .pointwise import MAX_CODE, MAX_CONST, PointwiseCompiler, Program, Val

MAX_PASSES = 4
MAX_STATES = 8
# Fold identities as Emmy seeds them: max / min start at the finite -1e30 / 1e30
# (an empty lane's state then combines without inf - inf).
IDENTITY = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "prod": 1.0, "maximum": -1e30, "max": -1e30,
            "minimum": 1e30, "min": 1e30, "fmax": -1e30, "fmin": 1e30}


def _aff_dict(form) -> dict:
    return {term: coef for term, coef in form}


class RowProgramCompiler(PointwiseCompiler):
    """Compiles the symbolic form of a row-reduction Tile (see the module docstring)."""

    def __init__(self, pkg: KernelPackage, tile: Node, ev):
        axes = [(a.name, static_extent(a.extent)) for a in tile.axes]
        if not 1 <= len(axes) <= 7:
            raise CompileError("row programs take row axes and one cooperative axis")
        self.pkg = pkg
        self.ev = ev
        self.co, self.block = axes[-1]
        block = tile.get("block_threads") or self.block
        if block != self.block:
            raise CompileError("the cooperative axis must span the block")
        self.row_axes = axes[:-1] or [("__row", 1)]
        self.rows = math.prod(e for _, e in self.row_axes)
        self.code, self.consts, self.forms, self.form_index = [], {}, [], {}
        self.slots, self.env, self.nvreg, self.writes = {}, {}, 0, []
        self.state_slot: dict = {}   # accumulator -> slot, once its pass has combined
        self.live: dict = {}         # accumulator -> slot, inside its pass
        self.state_init: list = []
        self.state_pass: list = []
        self.pass_ranges: list = []
        self.warp_ranges: list = []
        self.tree_ranges: list = []
        self.tile = tile
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
            if tag == "acc":
                if e[1] not in self.live:
                    raise CompileError(f"{e[1]} is read outside the pass that accumulates it")
                return self.emit("PARTIAL", "f32", aux=self.live[e[1]])
            if tag == "red":
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
    def begin_range(self) -> int:
        self.__dict__["_memo"] = {}     # a range runs on its own: no value crosses ranges
        return len(self.code)

    def combines(self) -> list:
        """(WarpShuffle, TreeHalve) after each pass, in pass order."""
        found, p = [], -1
        for s in self.tile.body:
            if s.kind in ("StridedLoop", "Loop"):
                p += 1
                found.append([None, None])
            elif s.kind == "WarpShuffle" and p >= 0:
                found[p][0] = s
            elif s.kind == "TreeHalve" and p >= 0:
                found[p][1] = s
        return found

    def combine_program(self, node: Node, slots: dict) -> tuple:
        """Compile a combine_states program: state names read the own partial,
        partner names the other's; the states' final values are written back."""
        begin = self.begin_range()
        saved = self.env
        self.env = {}
        for a, b in zip(node.state, node.state_b):
            if a not in slots:
                raise CompileError(f"{a} is combined but not accumulated in this pass")
            self.env[a] = self.emit("PARTIAL", "f32", aux=slots[a])
            self.env[b] = self.emit("PARTNER", "f32", aux=slots[a])
        for st in node.get("combine_states") or ():
            if st.kind not in ("Assign", "Let"):
                raise CompileError(f"unsupported combine statement {st.kind}")
            PointwiseCompiler.statement(self, st)
        for a in node.state:
            self.emit("SETP", None, self.convert(self.env[a], "f32"), aux=slots[a])
        self.env = saved
        return begin, len(self.code)

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
        if len(reds) > MAX_STATES:
            raise CompileError("row program has too many accumulators")
        combines = self.combines()
        if len(combines) != len(loops):
            raise CompileError("row-program passes must be top-level loops")
        inits = {s.name: float(s.identity) for s in self.tile.body if s.kind == "Init"}
        self.extents = tuple(e for _, e in self.row_axes) + (self.cols,)
        for p, loop in enumerate(loops):
            self.axes = [n for n, _ in self.row_axes] + [loop["axis"]]
            accs = [n for n in loop["accums"] if n in reds]
            slots = {}
            for name in accs:
                slots[name] = len(self.state_pass)
                op = reds[name]["op"]
                seed = inits.get(name, IDENTITY.get(op))
                if seed is None:
                    raise CompileError(f"no seed for accumulator {name} ({op})")
                from .pointwise import f32_word
                self.state_init.append(f32_word(seed))
                self.state_pass.append(p)
            self.live = slots
            begin = self.begin_range()
            for name in accs:
                red = reds[name]
                if red["base"] is not None:
                    new = self.sym(red["value"])         # op(base, value) as the IR states it
                else:
                    partial = self.emit("PARTIAL", "f32", aux=slots[name])
                    new = self.convert(self.operation(red["op"], [partial, self.sym(red["value"])], "f32"), "f32")
                self.emit("SETP", None, new, aux=slots[name])
            for w in ev.writes:
                if w["loop"] == loop["axis"]:
                    if w["cond"]:
                        raise CompileError("conditional writes inside a row pass are not supported")
                    self.store(w, final=False)
            self.pass_ranges.append((begin, len(self.code)))
            warp, tree = combines[p]
            if accs:
                if warp is None or tree is None or int(warp.get("length") or 0) != 32 or \
                        int(tree.get("length") or 0) * 32 != self.block or tree.get("tid_var") != "warp" or \
                        tree.get("inner"):
                    raise CompileError("a pass's accumulators must be combined by a warp butterfly and a block tree")
                if set(warp.state) != set(accs) or set(tree.state) != set(accs):
                    raise CompileError("the combines do not cover exactly the pass's accumulators")
                self.warp_ranges.append(self.combine_program(warp, slots))
                self.tree_ranges.append(self.combine_program(tree, slots))
            else:
                self.warp_ranges.append((0, 0))
                self.tree_ranges.append((0, 0))
            self.live = {}
            self.state_slot.update(slots)
        self.axes = [n for n, _ in self.row_axes] + ["__col"]
        final_begin = self.begin_range()
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
        R = len(self.row_axes)
        row_grid = np.meshgrid(*[np.arange(e, dtype=np.int64) for _, e in self.row_axes], indexing="ij")
        row_coords = [g.ravel() for g in row_grid]
        for out in outs:
            size = math.prod(self.pkg.buffers[out].shape or (1,))
            if size > (1 << 26):
                raise CompileError("row-program outputs above 2^26 elements are not verified")
            seen = np.zeros(size, np.int64)
            for b, f in self.pass_writes:
                if b != out:
                    continue
                form = self.forms[f]
                flat = form.base + sum(form.coef[d] * row_coords[d] for d in range(R))
                cols = np.arange(self.cols, dtype=np.int64)
                np.add.at(seen, (flat[:, None] + form.coef[R] * cols[None, :]).ravel(), 1)
            for b, f in self.final_writes:
                if b != out:
                    continue
                form = self.forms[f]
                np.add.at(seen, form.base + sum(form.coef[d] * row_coords[d] for d in range(R)), 1)
            if np.any(seen != 1):
                raise CompileError(f"row-program writes do not cover {out} exactly once")

    def layout(self, final: tuple) -> dict:
        return {"passes": [list(r) for r in self.pass_ranges], "warp": [list(r) for r in self.warp_ranges],
                "tree": [list(r) for r in self.tree_ranges], "final": list(final),
                "state_init": list(self.state_init), "state_pass": list(self.state_pass), "threads": self.block}


def _add_const(form, k: int):
    d = dict(form)
    d[1] = d.get(1, 0) + k
    return frozenset((t, c) for t, c in d.items() if c != 0)


def compile_rowprog(pkg: KernelPackage, tile: Node, ev):
    """Plan of a reduction / fused row Tile as a row program."""
    from .recognize import _plan
    comp = RowProgramCompiler(pkg, tile, ev)
    final = comp.compile_rows()
    code, nregs = comp.allocate()
    if len(code) > MAX_CODE or len(comp.consts) > MAX_CONST:
        raise CompileError("row program too long")
    consts = [0] * len(comp.consts)
    for word, i in comp.consts.items():
        consts[i] = word
    names = list(comp.slots)
    prog = Program(code, consts, comp.forms, names, tuple(e for _, e in comp.row_axes) + (comp.cols,), nregs,
                   [math.prod(pkg.buffers[b].shape or (1,)) for b in names])
    bind = {f"buf{i}": name for i, name in enumerate(names)}
    outs = sorted({b for b, _ in comp.pass_writes + comp.final_writes})
    return _plan(pkg, "rowprog", "lc_rowprog", bind,
                 {"program": prog.to_json(), "layout": comp.layout(final), "out": outs[0],
                  "rows": comp.rows, "cols": comp.cols},
                 {name: pkg.buffers[name].dtype for name in names})
