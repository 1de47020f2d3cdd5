"""One-warp fragment programs compiled to lane programs.

A Tile of one 32-lane warp that declares m16n8k16 fragments and works on
them — gathers (LdmatrixLoad from global), MmaSyncPtx, FragmentApply (the
per-element algebra with FRAG / ROW / UNIFORM / COORD / GMEM operands, lazy
``where`` and unary ``post`` chains), FragmentRowReduce (the quad fold),
FragmentRepack and RegStore with an epilogue lambda — next to scalar Let /
Assign statements, compiles here to a register program that
csrc/pointwise.cu runs with one kernel point per lane: the point space is
(g, t) = (lane / 4, lane % 4), 8 x 4, so each warp of the kernel is the
reference's warp.

Every step is the reference's per-lane lowering (ptx_tensor.py), in its
order and rounding:

* a fragment is its lane's registers: C four f32 (rows g, g+8; columns 2t,
  2t+1), A four and B two packed 16-bit pairs (ptx_tensor.py:164-180);
* global gathers clamp M/N to the last valid row and zero-fill the K tail
  per element, converting to the fragment type (:324-363);
* mma.sync m16n8k16 row.col with f32 accumulation (:365-381);
* FragmentApply evaluates its operation per element with the coordinate
  bindings __frow = row_base + g (+8), __fcol = col_base + 2t (+1), loads
  GMEM operands, takes ``where`` lazily and applies the ``post`` chain in
  f32 (:480-588);
* FragmentRowReduce folds each row's parts left to right over the listed
  fragments, then combines with the lanes 2 and 1 apart (:590-618);
* FragmentRepack rounds two C fragments into one A fragment (:459-473);
* RegStore writes each element whose guards hold, through the epilogue
  lambda with the element's fragment-local row and column (:383-457).

Loops run at compile time (fragment subscripts must be static); scalar
statements compile as in pointwise programs.  The kernel's loads are
clamped into their buffers and its stores skip indices outside them, so a
program cannot touch memory outside its arguments.
"""
from __future__ import annotations

import math
import re

from .ir import CompileError, KernelPackage, Node, static_extent
from .pointwise import PointwiseCompiler, Program, Val, vm_type

SHAPE = (16, 8, 16)
FRAG_ROW, FRAG_COL = "__frow", "__fcol"
ELEM_ROW, ELEM_COL = "__M__", "__N__"
_STORE = {"f32": "STX_F32", "f16": "STX_F16", "bf16": "STX_BF16", "s32": "STX_S32"}
_LOADX = {"f32": "LDX_F32", "f16": "LDX_F16", "bf16": "LDX_BF16", "s32": "LDX_S32"}


class Frag:
    def __init__(self, role: str, dtype: str, members: list):
        self.role, self.dtype, self.members = role, dtype, members   # members: lists of fixed register ids


class LaneCompiler(PointwiseCompiler):
    """Lowers a one-warp fragment program to lane operations (see the module docstring)."""

    def __init__(self, pkg: KernelPackage, tile: Node):
        axes = tuple(tile.axes)
        if len(axes) != 1 or static_extent(axes[0].extent) != 32:
            raise CompileError("fragment programs run on one 32-lane warp")
        self.pkg = pkg
        self.axes = ["__g", "__t"]
        self.extents = (8, 4)
        self.code, self.consts, self.forms, self.form_index = [], {}, [], {}
        self.slots, self.env, self.nvreg, self.writes = {}, {}, 0, []
        self.static: dict = {}
        self.frags: dict = {}
        self.n_fixed = 0
        self.steps = 0
        self.outputs: set = set()
        g = self.emit("COORD", "s32", aux=0)
        t = self.emit("COORD", "s32", aux=1)
        self.g, self.t = g, t
        self.lane = self.binary("+", self.binary("*", g, self.literal(4, "s32")), t)
        self.env[axes[0].name] = self.lane

    # ------------------------------------------------------------ registers
    def fixed(self, count: int) -> list:
        regs = list(range(self.n_fixed, self.n_fixed + count))
        self.n_fixed += count
        return [-1 - r for r in regs]

    def fval(self, reg: int, dt: str = "f32") -> Val:
        return Val(reg, dt)

    def put(self, reg: int, v: Val) -> None:
        self.code.append((self.op_id("MOV"), reg, v.reg, 0, 0, 0, 1, True))

    @staticmethod
    def op_id(name: str) -> int:
        from .pointwise import OP
        return OP[name]

    def raw(self, op: str, dst: int | None, srcs: list, aux: int = 0) -> None:
        regs = list(srcs) + [0] * (3 - len(srcs))
        self.code.append((self.op_id(op), 0 if dst is None else dst, *regs, aux, len(srcs), dst is not None))

    def slot(self, buffer: str) -> int:
        if buffer not in self.pkg.buffers:
            raise CompileError(f"unknown buffer {buffer}")
        if buffer not in self.slots:
            self.slots[buffer] = len(self.slots)
        return self.slots[buffer]

    # ------------------------------------------------------------ expressions with static loop values
    def expr(self, e) -> Val:
        if isinstance(e, Node) and e.kind == "Var" and e.name in self.static:
            return self.literal(self.static[e.name], "s32")
        if isinstance(e, str) and e in self.static:
            return self.literal(self.static[e], "s32")
        return super().expr(e)

    def static_int(self, e) -> int:
        """A compile-time integer (literals and unrolled loop variables only)."""
        if isinstance(e, bool):
            raise CompileError("boolean where an integer is needed")
        if isinstance(e, int):
            return e
        if isinstance(e, Node):
            if e.kind == "Literal" and isinstance(e.value, int):
                return e.value
            if e.kind == "Var" and e.name in self.static:
                return self.static[e.name]
            if e.kind == "BinaryExpr" and e.op in ("+", "-", "*", "/", "%"):
                a, b = self.static_int(e.left), self.static_int(e.right)
                if e.op in ("/", "%") and b == 0:
                    raise CompileError("division by zero in a static index")
                q = abs(a) // abs(b) * (1 if (a >= 0) == (b >= 0) else -1) if e.op in ("/", "%") else 0
                return {"+": a + b, "-": a - b, "*": a * b, "/": q, "%": a - b * q}[e.op]
        raise CompileError(f"{e!r} is not a compile-time integer")

    def int_expr(self, e) -> Val:
        return self.convert(self.expr(e), "s32")

    def flat_index(self, buffer: str, index: tuple) -> Val:
        """Row-major element index of an IR index tuple (ptx_backend.py:1216-1239)."""
        shape = tuple(self.pkg.buffers[buffer].shape) or (1,)
        if not index:
            return self.literal(0, "s32")
        if len(index) == 1:
            return self.int_expr(index[0])
        total = self.literal(0, "s32")
        for d, i in enumerate(index):
            stride = math.prod(shape[d + 1:]) if len(index) == len(shape) else 1
            total = self.binary("+", total, self.binary("*", self.int_expr(i), self.literal(stride, "s32")))
        return total

    # ------------------------------------------------------------ fragments
    def ref(self, text: str, role: str | None = None) -> tuple:
        m = re.fullmatch(r"([A-Za-z_$][\w$]*)(?:\[([A-Za-z_$][\w$]*|[0-9]+)\])?", str(text))
        if m is None:
            raise CompileError(f"unsupported fragment reference {text!r}")
        stem, sub = m.groups()
        frag = self.frags.get(stem)
        if frag is None:
            raise CompileError(f"undeclared fragment {stem!r}")
        if role is not None and frag.role != role:
            raise CompileError(f"fragment {stem!r} must have role {role}")
        if sub is None:
            if len(frag.members) != 1:
                raise CompileError(f"fragment family {stem!r} needs a subscript")
            return frag, 0
        idx = int(sub) if sub.isdecimal() else self.static.get(sub)
        if idx is None:
            raise CompileError("fragment subscripts must be compile-time values")
        if not 0 <= idx < len(frag.members):
            raise CompileError(f"fragment index {idx} outside {stem!r}")
        return frag, idx

    def regs_of(self, text: str, role: str | None = None) -> list:
        frag, idx = self.ref(text, role)
        return frag.members[idx]

    # ------------------------------------------------------------ statements
    def statement(self, s: Node) -> None:
        self.steps += 1
        if self.steps > 4096:
            raise CompileError("fragment program too long")
        k = s.kind
        handler = getattr(self, "do_" + k, None)
        if handler is not None:
            handler(s)
        elif k in ("Let", "Assign", "Select"):
            super().statement(s)
        else:
            raise CompileError(f"{k} is not supported in fragment lane programs")

    def do_StridedLoop(self, s: Node) -> None:
        name = s.axis.name
        start = self.static_int(s.start) if s.kind == "StridedLoop" and s.get("start") is not None else 0
        step = self.static_int(s.step) if s.kind == "StridedLoop" and s.get("step") is not None else 1
        end = s.get("end") if s.kind == "StridedLoop" else None
        bound = self.static_int(end) if end is not None else static_extent(s.axis.extent)
        if step <= 0:
            raise CompileError("loop step must be positive")
        saved = self.static.get(name)
        for v in range(start, bound, step):
            self.static[name] = v
            for inner in s.body:
                self.statement(inner)
        if saved is None:
            self.static.pop(name, None)
        else:
            self.static[name] = saved

    do_Loop = do_StridedLoop

    def do_RegFragment(self, s: Node) -> None:
        if tuple(s.shape) != SHAPE:
            raise CompileError(f"fragment shape {s.shape} is not m16n8k16")
        dt = vm_type(s.dtype)
        width = {"a": 4, "b": 2, "c": 4}.get(s.role)
        if width is None or (s.role == "c" and dt != "f32") or (s.role != "c" and dt not in ("f16", "bf16")):
            raise CompileError("fragments must be f16/bf16 A/B or f32 C")
        count = int(s.get("count") or 1)
        if not 1 <= count <= 16:
            raise CompileError("fragment family too large for a lane program")
        members = [self.fixed(width) for _ in range(count)]
        if s.role == "c":
            zero = self.literal(0.0, "f32")
            for regs in members:
                for r in regs:
                    self.put(r, zero)
        self.frags[s.name] = Frag(s.role, dt, members)

    def do_LdmatrixLoad(self, s: Node) -> None:
        if s.get("staged") or s.get("pair_frag") is not None or s.get("swizzle", "NONE") not in (None, "NONE"):
            raise CompileError("lane programs gather fragments from global memory only")
        if s.role not in ("a", "b") or (s.role == "a" and s.get("b_trans")):
            raise CompileError("invalid tensor operand role or orientation")
        frag, idx = self.ref(s.frag, s.role)
        buf = self.pkg.buffers.get(s.src_buffer)
        if buf is None or buf.dtype not in ("f32", "f16", "bf16"):
            raise CompileError("tensor gathers read f32, f16 or bf16 buffers")
        ldm = int(s.get("ldm") or buf.shape[-1])
        base = self.flat_index(s.src_buffer, tuple(s.src_index))
        rem_mn = rem_k = None
        if s.get("gmem_guard") is not None:
            rem_mn = self.binary("-", self.int_expr(s.gmem_guard[1]), self.int_expr(s.gmem_guard[0]))
        if s.get("k_zero") is not None:
            rem_k = self.binary("-", self.int_expr(s.k_zero[1]), self.int_expr(s.k_zero[0]))
        pair = self.binary("*", self.t, self.literal(2, "s32"))
        regs = frag.members[idx]
        for i in range(4 if s.role == "a" else 2):
            mn = self.binary("+", self.g, self.literal(8 if s.role == "a" and i & 1 else 0, "s32"))
            kk = self.binary("+", pair, self.literal(8 if (i & 2 if s.role == "a" else i) else 0, "s32"))
            valid_mn = None
            if rem_mn is not None:
                valid_mn = self.compare("gt", rem_mn, self.literal(0, "s32"))
                last = self.emit("IMAX", "s32", self.binary("-", rem_mn, self.literal(1, "s32")),
                                 self.literal(0, "s32"))
                mn = self.emit("IMIN", "s32", mn, last)
            halves = []
            for half in (0, 1):
                kh = self.binary("+", kk, self.literal(half, "s32"))
                row, col = (mn, kh) if s.role == "a" or s.get("b_trans") else (kh, mn)
                at = self.binary("+", base, self.binary("+", self.binary("*", row, self.literal(ldm, "s32")), col))
                value = self.emit(_LOADX[vm_type(buf.dtype)], vm_type(buf.dtype), at, aux=self.slot(s.src_buffer))
                valid = valid_mn
                if rem_k is not None:
                    vk = self.compare("lt", kh, rem_k)
                    valid = vk if valid is None else self.binary("&&", valid, vk)
                value = self.convert(value, "f32")
                if valid is not None:
                    value = self.select(valid, value, self.literal(0.0, "f32"), "f32")
                halves.append(value)
            self.raw("PACK_F16X2" if frag.dtype == "f16" else "PACK_BF16X2", regs[i], [halves[0].reg, halves[1].reg])

    def do_MmaSyncPtx(self, s: Node) -> None:
        if tuple(s.shape) != SHAPE or s.ab_dtype not in ("f16", "bf16") or s.c_dtype != "f32":
            raise CompileError("MMA must be m16n8k16 with f16/bf16 operands and f32 accumulation")
        if s.get("b_row_major") or s.get("sfa_frag") is not None or s.get("sfb_frag") is not None:
            raise CompileError("row-major B and block-scaled MMA forms are not supported")
        a, ai = self.ref(s.a_frag, "a")
        b, bi = self.ref(s.b_frag, "b")
        c = self.regs_of(s.c_frag, "c")
        if a.dtype != s.ab_dtype or b.dtype != s.ab_dtype:
            raise CompileError("MMA type disagrees with its fragments")
        self.raw("MMA_F16" if s.ab_dtype == "f16" else "MMA_BF16", c[0],
                 [a.members[ai][0], b.members[bi][0], c[0]])

    def do_FragmentRepack(self, s: Node) -> None:
        if int(s.get("part") or 0) != 0 or len(s.srcs) != 2 or s.ab_dtype not in ("f16", "bf16"):
            raise CompileError("repack takes two C fragments into a 16-bit A fragment")
        frag, idx = self.ref(s.frag, "a")
        if frag.dtype != s.ab_dtype:
            raise CompileError("repack type disagrees with its A fragment")
        srcs = [list(self.regs_of(name, "c")) for name in s.srcs]
        values = []
        for regs in srcs:
            for pr in (0, 2):
                values.append((regs[pr], regs[pr + 1]))
        op = "PACK_F16X2" if s.ab_dtype == "f16" else "PACK_BF16X2"
        temps = []
        for lo, hi in values:   # read every source before writing the A registers
            t = self.new(frag.dtype)
            self.code.append((self.op_id(op), t.reg, lo, hi, 0, 0, 2, True))
            temps.append(t)
        for reg, t in zip(frag.members[idx], temps):
            self.put(reg, t)

    def element_coords(self, e: int, row_base, col_base) -> None:
        self.env.pop(FRAG_ROW, None)
        self.env.pop(FRAG_COL, None)
        if row_base is not None:
            self.env[FRAG_ROW] = self.binary("+", self.int_expr(row_base),
                                             self.binary("+", self.g, self.literal(8 if e >= 2 else 0, "s32")))
        if col_base is not None:
            self.env[FRAG_COL] = self.binary("+", self.int_expr(col_base),
                                             self.binary("+", self.binary("*", self.t, self.literal(2, "s32")),
                                                         self.literal(e & 1, "s32")))

    def do_FragmentApply(self, s: Node) -> None:
        layout = s.layout
        if tuple(layout.elem_row) != (0, 0, 1, 1):
            raise CompileError("fragment algebra needs the m16n8k16 C layout")
        kinds = tuple(s.kinds)
        if len(kinds) != len(s.args):
            raise CompileError("fragment operation argument/kind counts disagree")
        inputs = {i: list(self.regs_of(a, "c")) for i, (a, k) in enumerate(zip(s.args, kinds)) if k == "frag"}
        results = []
        saved = dict(self.env)
        for e in range(4):
            self.env = dict(saved)
            self.element_coords(e, s.get("row_base"), s.get("col_base"))

            def operand(i):
                arg, kind = s.args[i], kinds[i]
                if kind == "frag":
                    return self.fval(inputs[i][e])
                if kind == "row":
                    return self.convert(self.lookup(arg[layout.elem_row[e]]), "f32")
                if kind in ("coord", "uniform"):
                    v = self.lookup(arg) if isinstance(arg, str) else self.expr(arg)
                    return v if kind == "coord" else self.convert(v, "f32")
                if kind == "gmem":
                    buffer, index = arg
                    buf = self.pkg.buffers.get(buffer)
                    if buf is None or buffer not in self.pkg.arg_order:
                        raise CompileError("fragment GMEM operand needs a kernel argument")
                    at = self.flat_index(buffer, tuple(index))
                    v = self.emit(_LOADX[vm_type(buf.dtype)], vm_type(buf.dtype), at, aux=self.slot(buffer))
                    return self.convert(v, "f32")
                raise CompileError(f"unsupported fragment operand kind {kind!r}")

            opname = s.op.name if isinstance(s.op, Node) else str(s.op)
            if opname == "where":
                if len(s.args) != 3:
                    raise CompileError("fragment where takes three operands")
                cond = self.convert(operand(0), "pred")
                # clamped loads make the unselected operand harmless to evaluate
                value = self.select(cond, self.convert(operand(1), "f32"), self.convert(operand(2), "f32"), "f32")
            else:
                value = self.operation(opname, [operand(i) for i in range(len(s.args))], "f32")
            for post in s.get("post") or ():
                value = self.operation(post.name if isinstance(post, Node) else str(post), [value], "f32")
            results.append(self.convert(value, "f32"))
        self.env = saved
        if s.get("in_place"):
            regs = self.regs_of(s.out, "c")
        else:
            if not re.fullmatch(r"[A-Za-z_$][\w$]*", str(s.out)):
                raise CompileError("a new fragment output must be a plain name")
            regs = self.fixed(4)
            self.frags[s.out] = Frag("c", "f32", [regs])
        for reg, v in zip(regs, results):
            self.put(reg, v)

    def do_FragmentRowReduce(self, s: Node) -> None:
        layout = s.layout
        if tuple(layout.elem_row) != (0, 0, 1, 1) or tuple(layout.reduce_xors) != (2, 1):
            raise CompileError("fragment row reduction needs the m16n8k16 C layout")
        opname = s.op.name if isinstance(s.op, Node) else str(s.op)
        if opname not in ("add", "multiply", "maximum", "minimum") or not s.frags or s.top == s.bot:
            raise CompileError("unsupported fragment row reduction")
        if s.get("dtype") is not None and vm_type(s.dtype) != "f32":
            raise CompileError("fragment row reductions are f32")
        fragments = [list(self.regs_of(name, "c")) for name in s.frags]
        reduced = []
        for row in range(2):
            parts = [self.fval(regs[i]) for regs in fragments for i, r in enumerate(layout.elem_row) if r == row]
            result = parts[0]
            for part in parts[1:]:
                result = self.operation(opname, [result, part], "f32")
            reduced.append(result)
        for delta in layout.reduce_xors:
            for row, value in enumerate(reduced):
                peer = self.emit("SHFL_XOR", "f32", value, aux=int(delta))
                reduced[row] = self.operation(opname, [value, peer], "f32")
        self.env[s.top], self.env[s.bot] = reduced

    def do_RegStore(self, s: Node) -> None:
        if tuple(s.shape) != SHAPE or s.get("volta_interleaved") or s.get("extra_frags"):
            raise CompileError("fragment stores must be plain m16n8k16 stores")
        if s.get("swizzle", "NONE") not in (None, "NONE"):
            raise CompileError("swizzled global stores are not supported")
        regs = list(self.regs_of(s.frag, "c"))
        buf = self.pkg.buffers.get(s.dst_buffer)
        if buf is None or buf.role != "output":
            raise CompileError("fragment stores must write the kernel's output")
        dt = vm_type(buf.dtype)
        if s.get("atomic") and dt != "f32":
            raise CompileError("atomic tensor stores need an f32 output")
        shape = tuple(buf.shape)
        rd, cd = s.get("row_dim"), s.get("col_dim")
        row_stride = int(s.get("ldm") or 0) or (math.prod(shape[rd + 1:]) if rd is not None else shape[-1])
        col_stride = math.prod(shape[cd + 1:]) if cd is not None else 1
        base = self.flat_index(s.dst_buffer, tuple(s.dst_index))
        pair = self.binary("*", self.t, self.literal(2, "s32"))
        for i in range(4):
            row = self.binary("+", self.g, self.literal(8 if i >= 2 else 0, "s32"))
            col = self.binary("+", pair, self.literal(i & 1, "s32"))
            ok = self.literal(1, "pred")
            for guard, off in ((s.get("m_guard"), row), (s.get("n_guard"), col)):
                if guard is not None:
                    lim = self.compare("lt", self.binary("+", self.int_expr(guard[0]), off), self.int_expr(guard[1]))
                    ok = self.binary("&&", ok, lim)
            value = self.fval(regs[i])
            if s.get("epilogue") is not None:
                value = self.epilogue(s.epilogue, value, row, col)
            at = self.binary("+", base, self.binary("+", self.binary("*", row, self.literal(row_stride, "s32")),
                                                    self.binary("*", col, self.literal(col_stride, "s32"))))
            value = self.convert(value, dt)
            op = "STX_ADD_F32" if s.get("atomic") else _STORE[dt]
            self.raw(op, None, [at.reg, value.reg, self.convert(ok, "pred").reg], aux=self.slot(s.dst_buffer))
            self.outputs.add(s.dst_buffer)

    def epilogue(self, lam: Node, acc: Val, row: Val, col: Val) -> Val:
        params = list(lam.params)
        saved = dict(self.env)
        self.env[params[0]] = acc
        self.env[ELEM_ROW], self.env[ELEM_COL] = row, col
        for p in params[1:]:
            if p not in self.env:
                raise CompileError(f"unbound epilogue coordinate {p!r}")
        for st in lam.body:
            if st.kind == "Load":
                if len(st.names) != 1:
                    raise CompileError("epilogue loads must be scalar")
                buf = self.pkg.buffers[st.input]
                v = self.emit(_LOADX[vm_type(buf.dtype)], vm_type(buf.dtype), self.flat_index(st.input, tuple(st.index)),
                              aux=self.slot(st.input))
                self.env[st.names[0]] = self.convert(v, "f32")
            elif st.kind in ("Assign", "Let", "Select"):
                PointwiseCompiler.statement(self, st)
            else:
                raise CompileError(f"unsupported epilogue statement {st.kind}")
        (result,) = lam.results
        out = self.lookup(result)
        self.env = saved
        return out

    # ------------------------------------------------------------ finishing
    def compile_lanes(self, body: tuple) -> Program:
        for s in body:
            self.statement(s)
        if not self.outputs:
            raise CompileError("fragment program stores nothing")
        code, nregs = self.allocate()
        from .pointwise import MAX_CODE, MAX_CONST
        if len(code) > MAX_CODE:
            raise CompileError(f"fragment program has {len(code)} operations (at most {MAX_CODE})")
        if len(self.consts) > MAX_CONST:
            raise CompileError("fragment program has too many constants")
        consts = [0] * len(self.consts)
        for word, i in self.consts.items():
            consts[i] = word
        names = list(self.slots)
        return Program(code, consts, [], names, self.extents, nregs,
                       [math.prod(self.pkg.buffers[b].shape or (1,)) for b in names])


def compile_fragment_lanes(pkg: KernelPackage, tile: Node):
    """Plan of a one-warp fragment program run as a lane program."""
    from .recognize import _plan
    comp = LaneCompiler(pkg, tile)
    prog = comp.compile_lanes(tuple(tile.body))
    bind = {f"buf{i}": name for i, name in enumerate(prog.buffers)}
    outs = sorted(comp.outputs)
    return _plan(pkg, "pointwise", "lc_pointwise", bind,
                 {"program": prog.to_json(), "out": outs[0], "points": 32, "lanes": True},
                 {name: pkg.buffers[name].dtype for name in prog.buffers})
