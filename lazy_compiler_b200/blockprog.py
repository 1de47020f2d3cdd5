"""Block programs: any Tile body, run the way the reference's kernel runs it.

The fixed classes and the row, serial, lane and pointwise programs each
take one shape of Tile body.  A body none of them takes — a staged matmul
whose operands pass through an elementwise function, a block-cooperative
attention with another score function, any mix of loops, conditions,
shuffles and shared trees — compiles here to a register program that one
CTA per block of the Tile runs statement for statement (csrc/pointwise.cu,
``lc_blockprog``), following the reference's lowering of each statement:

* the Tile's trailing axes whose extents multiply to ``block_threads`` are a
  block's threads, the leading axes number the blocks (ptx_backend.py
  :1574-1642); ``lane`` and ``warp`` are the thread index mod 32 and / 32;
* Loop / StridedLoop run per thread from their start in steps of their step
  while below their extent (:1496-1554), the loop variable a coordinate;
  an accumulator lives in a fixed register, seeded with its identity on
  entry to a seeding loop (or by Init) and updated as op(base or acc, v);
* Cond branches (else bodies too); Load / Write address global memory with
  computed row-major indices (loads clamped into their buffer, stores
  skipped outside it, atomic writes as f32 atomic adds, :1216-1330);
* Smem arrays are per-CTA shared memory, CpAsyncCopy a synchronous copy
  (the program's own waits and barriers order it, :1457-1492), Sync a
  barrier (:1644-1657);
* WarpShuffle is the reference's butterfly — each level exchanges the
  states with shfl.bfly and runs the Tile's combine statements (:1659-1703)
  — and TreeHalve its shared-memory tree with one writer per slot and a
  barrier per level (:1705-1744).

Barriers and shuffles must be reached by every thread: they may not sit
inside a Cond or inside a loop whose range depends on the thread.  The
scalar rules are the pointwise programs' (``PointwiseCompiler``).
"""
from __future__ import annotations

import math

from .ir import CompileError, KernelPackage, Node, static_extent
from .pointwise import MAX_AXES, MAX_CODE, MAX_CONST, OP, Program, Val, _STORAGE, vm_type
from .serial import IDENTITY, SerialCompiler

MAX_SMEM = 8
MAX_SMEM_WORDS = 200 * 1024 // 4


class BlockCompiler(SerialCompiler):
    """Lowers a Tile body to a block program (see the module docstring)."""

    _IMPURE = SerialCompiler._IMPURE + ("LDS", "STS", "BAR", "WSYNC", "BRA", "BRZ", "SLB", "SLE")

    def __init__(self, pkg: KernelPackage, tile: Node):
        super().__init__(pkg, tile)
        threads = int(tile.get("block_threads") or (pkg.kernel_meta.get("block") or [0])[0])
        prod, split = 1, len(self.axes)
        while split > 0 and prod < threads:
            split -= 1
            prod *= self.extents[split]
        if threads < 1 or threads > 1024 or prod != threads:
            raise CompileError("the Tile's trailing axes do not form a thread block of at most 1024 threads")
        self.threads = threads
        self.n_block_axes = split
        self.smem: dict = {}            # name -> (array index, offset, shape)
        self.smem_words = 0
        self.uniform_depth = 0          # > 0 inside a Cond or a loop with a per-thread range
        tid = self.emit("TID", "s32")
        self.env["lane"] = self.binary("&", tid, self.literal(31))
        self.env["warp"] = self.binary(">>", tid, self.literal(5))

    # ------------------------------------------------------------ indices
    def int_expr(self, e) -> Val:
        v = self.expr(e)
        if v.type == "pred":
            return self.convert(v, "s32")
        if v.type != "s32":
            raise CompileError("an index is not an integer")
        return v

    def flat(self, shape: tuple, index: tuple) -> Val:
        shape = tuple(shape) or (1,)
        parts = [self.int_expr(i) for i in index]
        if not parts:
            return self.literal(0)
        if len(parts) == 1 or len(parts) != len(shape):
            total = parts[0]
            for p in parts[1:]:
                total = self.binary("+", total, p)
            return total
        total = None
        for d, p in enumerate(parts):
            stride = math.prod(shape[d + 1:])
            term = p if stride == 1 else self.binary("*", p, self.literal(stride))
            total = term if total is None else self.binary("+", total, term)
        return total

    def slot(self, buffer: str) -> int:
        if buffer not in self.slots:
            if len(self.slots) >= 16:
                raise CompileError("block program uses too many buffers")
            self.slots[buffer] = len(self.slots)
        return self.slots[buffer]

    def barrier_allowed(self, what: str) -> None:
        if self.uniform_depth:
            raise CompileError(f"{what} inside a condition or a per-thread loop is not reached by every thread")

    # ------------------------------------------------------------ control flow
    def clear_memo(self) -> None:
        self.__dict__["_memo"] = {}

    def branch(self, op: str, cond: Val | None = None) -> int:
        at = len(self.code)
        self.code.append((OP[op], 0, cond.reg if cond else 0, 0, 0, 0, 1 if cond else 0, False))
        return at

    def patch(self, at: int) -> None:
        op, dst, a, b, c, _, nsrc, has_dst = self.code[at]
        self.code[at] = (op, dst, a, b, c, len(self.code), nsrc, has_dst)

    def fixed_const(self, value: int) -> Val:
        """A loop bound in a fixed register written once, by CONST (the host's
        test that a loop around a barrier has the same range in every thread)."""
        word = value % (1 << 32)
        if word not in self.consts:
            if len(self.consts) >= MAX_CONST:
                raise CompileError("block program has too many constants")
            self.consts[word] = len(self.consts)
        reg = -1 - self.n_fixed
        self.n_fixed += 1
        self.code.append((OP["CONST"], reg, 0, 0, 0, self.consts[word], 0, True))
        return Val(reg, "s32")

    # ------------------------------------------------------------ statements
    def statement(self, s: Node) -> None:
        k = s.kind
        if k == "Smem":
            self.declare_smem(s)
        elif k == "Load" and s.input in self.smem:
            arr, _, shape = self.smem[s.input]
            at = self.flat(shape, tuple(s.index))
            for lane, name in enumerate(s.names):
                idx = at if lane == 0 else self.binary("+", at, self.literal(lane))
                self.env[name] = self.emit("LDS", "f32", idx, aux=arr)
        elif k == "Load":
            buf = self.pkg.buffers.get(s.input)
            if buf is None:
                raise CompileError(f"Load from unknown buffer {s.input}")
            dt = vm_type(buf.dtype)
            if dt not in _STORAGE:
                raise CompileError(f"cannot load {buf.dtype}")
            at = self.flat(buf.shape, tuple(s.index))
            for lane, name in enumerate(s.names):
                idx = at if lane == 0 else self.binary("+", at, self.literal(lane))
                self.env[name] = self.emit("LDX_" + _STORAGE[dt], dt, idx, aux=self.slot(s.input))
        elif k == "Write":
            self.write(s)
        elif k == "CpAsyncCopy":
            self.copy(s)
        elif k in ("CpAsyncCommit", "CpAsyncWait"):
            pass  # copies complete synchronously
        elif k == "Sync":
            if s.get("barrier_id") or s.get("count") is not None:
                raise CompileError("named barriers are not supported")
            self.barrier_allowed("a barrier")
            self.code.append((OP["WSYNC" if s.get("warp") else "BAR"], 0, 0, 0, 0, 0, 0, False))
        elif k == "Cond":
            self.cond(s)
        elif k in ("Loop", "StridedLoop"):
            self.block_loop(s)
        elif k == "WarpShuffle":
            self.shuffle(s)
        elif k == "TreeHalve":
            self.tree(s)
        elif k in ("Accum", "Init", "Let", "Assign", "Select"):
            if k in ("Let", "Assign", "Select"):
                from .pointwise import PointwiseCompiler
                PointwiseCompiler.statement(self, s)
            else:
                super().statement(s)
        else:
            raise CompileError(f"{k} is not part of a block program")

    def declare_smem(self, s: Node) -> None:
        if s.name in self.smem:
            return
        if str(s.get("dtype") or "float") not in ("float", "f32"):
            raise CompileError("shared arrays hold f32")
        shape = tuple(int(x) for x in s.extents)
        size = max(1, math.prod(shape))
        if len(self.smem) >= MAX_SMEM or self.smem_words + size > MAX_SMEM_WORDS:
            raise CompileError("block program needs too much shared memory")
        self.smem[s.name] = (len(self.smem), self.smem_words, shape)
        self.smem_words += size

    def write(self, s: Node) -> None:
        if s.output in self.smem:
            if s.get("atomic"):
                raise CompileError("atomic shared-memory writes are not supported")
            arr, _, shape = self.smem[s.output]
            at = self.flat(shape, tuple(s.index))
            for lane, name in enumerate(s.values):
                idx = at if lane == 0 else self.binary("+", at, self.literal(lane))
                self.emit("STS", None, idx, self.convert(self.lookup(name), "f32"), aux=arr)
            return
        buf = self.pkg.buffers.get(s.output)
        if buf is None or buf.role != "output":
            raise CompileError("block programs write the kernel's outputs or shared arrays")
        if s.get("swizzle", "NONE") not in (None, "NONE"):
            raise CompileError("swizzled writes are not supported")
        dt = vm_type(buf.dtype)
        if dt == "pred":
            raise CompileError("predicate outputs are not supported")
        atomic = bool(s.get("atomic"))
        if atomic and dt != "f32":
            raise CompileError("atomic writes add f32")
        at = self.flat(buf.shape, tuple(s.index))
        yes = self.literal(1, "pred")
        for lane, name in enumerate(s.values):
            idx = at if lane == 0 else self.binary("+", at, self.literal(lane))
            v = self.convert(self.lookup(name), dt)
            self.emit("STX_ADD_F32" if atomic else "STX_" + _STORAGE[dt], None, idx, v, yes,
                      aux=self.slot(s.output))
            self.writes.append((s.output, None))

    def copy(self, s: Node) -> None:
        if s.get("swizzle", "NONE") not in (None, "NONE"):
            raise CompileError("swizzled copies are not supported")
        if s.smem not in self.smem:
            raise CompileError(f"copy into undeclared shared array {s.smem}")
        src = self.pkg.buffers.get(s.src)
        if src is None or vm_type(src.dtype) != "f32":
            raise CompileError("copies read an f32 argument")
        elems = int(s.nbytes) // 4
        if elems < 1 or elems * 4 != int(s.nbytes):
            raise CompileError("copy size is not a whole number of f32 elements")
        arr, _, shape = self.smem[s.smem]
        sidx = list(s.smem_index)
        lane = s.get("lane_index")
        if lane is not None:
            if len(lane) != len(sidx):
                raise CompileError("lane index rank differs from the shared index")
            sidx = [Node("BinaryExpr", (("op", "+"), ("left", a), ("right", b))) for a, b in zip(sidx, lane)]
        dst = self.flat(shape, tuple(sidx))
        at = self.flat(src.shape, tuple(s.src_index))
        for e in range(elems):
            g = at if e == 0 else self.binary("+", at, self.literal(e))
            d = dst if e == 0 else self.binary("+", dst, self.literal(e))
            v = self.emit("LDX_F32", "f32", g, aux=self.slot(s.src))
            self.emit("STS", None, d, v, aux=arr)

    def cond(self, s: Node) -> None:
        p = self.convert(self.expr(s.cond), "pred")
        self.clear_memo()
        self.uniform_depth += 1
        skip = self.branch("BRZ", p)
        self.body(s.body)
        self.clear_memo()
        if s.get("else_body"):
            done = self.branch("BRA")
            self.patch(skip)
            self.body(s.else_body)
            self.clear_memo()
            self.patch(done)
        else:
            self.patch(skip)
        self.uniform_depth -= 1

    def block_loop(self, s: Node) -> None:
        extent = static_extent(s.axis.extent)
        start, step, end_expr = s.get("start"), s.get("step"), s.get("end")
        depth = len(self.loop_stack)
        if self.tile_axes + depth + 1 > MAX_AXES:
            raise CompileError("loops nested too deep for a block program")
        internal = f"#{depth}"
        if depth == len(self.loop_extents):
            self.loop_extents.append(extent)
            self.axes.append(internal)
        else:
            self.loop_extents[depth] = max(self.loop_extents[depth], extent)
        literal = lambda e: e is None or isinstance(e, int) or (isinstance(e, Node) and e.kind == "Literal")  # noqa: E731
        value = lambda e, default: default if e is None else (e if isinstance(e, int) else int(e.value))  # noqa: E731
        uniform = literal(start) and literal(step) and literal(end_expr)
        if s.get("seed", True):
            for inner in s.body:
                if isinstance(inner, Node) and inner.kind == "Accum":
                    op = inner.op.name if isinstance(inner.op, Node) else str(inner.op)
                    if op not in IDENTITY:
                        raise CompileError(f"no identity for accumulator operation {op}")
                    self.put(self.acc_register(inner.name), self.literal(IDENTITY[op], "f32"))
                    self.clear_low(inner.name)
        if uniform:
            step_v = value(step, 1)
            if step_v < 1:
                raise CompileError("loop step must be positive")
            first = self.fixed_const(value(start, 0))
            stride = self.fixed_const(step_v)
            limit = self.fixed_const(value(end_expr, extent))
        else:
            first = self.int_expr(start) if start is not None else self.literal(0)
            stride = self.int_expr(step) if step is not None else self.literal(1)
            # a captured end is evaluated once on entry (ptx_backend.py:1531-1543)
            limit = self.int_expr(end_expr) if end_expr is not None else self.literal(extent)
        if end_expr is not None:
            self.env[s.axis.name + "_end"] = limit
        outer_binding = self.active.get(s.axis.name)
        self.active[s.axis.name] = internal
        self.clear_memo()
        begin = len(self.code)
        self.code.append(None)
        self.loop_stack.append((depth, extent))
        if not uniform:
            self.uniform_depth += 1
        saved = dict(self.env)
        self.body(s.body)
        self.env = {**saved, **{n: Val(r, "f32") for n, r in self.accs.items()}}
        if not uniform:
            self.uniform_depth -= 1
        self.loop_stack.pop()
        if outer_binding is None:
            self.active.pop(s.axis.name, None)
        else:
            self.active[s.axis.name] = outer_binding
        self.clear_memo()
        end = len(self.code)
        self.code.append(None)
        self.code[begin] = (OP["SLB"], 0, first.reg, limit.reg, 0, depth | end << 4, 2, False)
        self.code[end] = (OP["SLE"], 0, stride.reg, limit.reg, 0, depth | begin << 4, 2, False)
        self.loop_ranges.append((begin, end))

    # ------------------------------------------------------------ shuffles and trees
    def body(self, statements) -> None:
        """Statements of one body in order, each knowing the statement before it (Dot2 adjacency)."""
        previous = None
        for inner in statements:
            self.previous = previous
            self.statement(inner)
            previous = inner

    def state_register(self, name: str) -> int:
        """The fixed register of a shuffled or tree state (prepare_state)."""
        if name in self.accs:
            return self.accs[name]
        value = self.lookup(name)
        reg = self.acc_register(name)
        self.put(reg, value)
        self.clear_low(name)
        return reg

    def merge(self, s: Node) -> None:
        for a in s.combine_states:
            op = a.op.name if isinstance(a.op, Node) else str(a.op)
            value = self.operation(op, [self.convert(self.lookup(n), "f32") for n in a.args], "f32")
            if a.name in s.state:
                self.put(self.accs[a.name], value)
                self.clear_low(a.name)
                self.env[a.name] = Val(self.accs[a.name], "f32")
            else:
                self.env[a.name] = self.convert(value, "f32")

    def shuffle(self, s: Node) -> None:
        length = int(s.length)
        if length < 1 or length > 32 or length & (length - 1):
            raise CompileError("shuffle length must be a power of two in 1..32")
        # whole warps, or one partial warp of a power-of-two size the butterfly stays inside
        partial = self.threads < 32 and not self.threads & (self.threads - 1) and length <= self.threads
        if self.threads % 32 and length > 1 and not partial:
            raise CompileError("shuffles need whole warps (or one power-of-two partial warp)")
        self.barrier_allowed("a shuffle")
        for name in s.state:
            self.state_register(name)
        saved = dict(self.env)
        delta = length // 2
        while delta:
            for a, b in zip(s.state, s.state_b):
                self.env[b] = self.emit("SHFL_XOR", "f32", self.convert(self.lookup(a), "f32"), aux=delta)
            self.merge(s)
            delta //= 2
        self.env = {**saved, **{n: Val(self.accs[n], "f32") for n in s.state}}

    def tree(self, s: Node) -> None:
        length = int(s.length)
        if length < 1 or length & (length - 1):
            raise CompileError("tree length must be a power of two")
        if s.get("barrier_id") or s.get("barrier_count") is not None:
            raise CompileError("named barriers are not supported")
        self.barrier_allowed("a shared tree")
        for buf in s.bufs:
            if buf not in self.smem:
                raise CompileError(f"tree over undeclared shared array {buf}")
        for name in s.state:
            self.state_register(name)
        saved = dict(self.env)
        tid = self.int_expr(Node("Var", (("name", s.tid_var),)))
        inner = s.get("inner")
        if inner:
            base, scale = self.int_expr(Node("Var", (("name", inner[0]),))), int(inner[1])
        else:
            base, scale = self.literal(0), 1
        slot = self.binary("+", self.binary("*", tid, self.literal(scale)), base)
        delta = length // 2
        while delta:
            worker = self.binary("<", tid, self.literal(delta))
            if s.tid_var == "warp" and not inner:
                worker = self.binary("&&", worker, self.binary("==", self.lookup("lane"), self.literal(0)))
            worker = self.convert(worker, "pred")
            self.clear_memo()
            skip = self.branch("BRZ", worker)
            other = self.binary("+", slot, self.literal(delta * scale))
            for buf, a, b in zip(s.bufs, s.state, s.state_b):
                arr = self.smem[buf][0]
                self.put(self.accs[a], self.emit("LDS", "f32", slot, aux=arr))
                self.clear_low(a)
                self.env[a] = Val(self.accs[a], "f32")
                self.env[b] = self.emit("LDS", "f32", other, aux=arr)
            self.merge(s)
            for buf, name in zip(s.bufs, s.state):
                self.emit("STS", None, slot, self.convert(self.lookup(name), "f32"), aux=self.smem[buf][0])
            self.clear_memo()
            self.patch(skip)
            self.code.append((OP["BAR"], 0, 0, 0, 0, 0, 0, False))
            delta //= 2
        self.env = {**saved, **{n: Val(self.accs[n], "f32") for n in s.state}}
        for buf, name in zip(s.bufs, s.state):
            self.put(self.accs[name], self.emit("LDS", "f32", base, aux=self.smem[buf][0]))
            self.clear_low(name)

    # ------------------------------------------------------------ finishing
    def compile_block(self, body: tuple) -> tuple:
        self.body(body)
        if not self.writes:
            raise CompileError("block program writes nothing")
        if len({b for b, _ in self.writes}) != 1:
            raise CompileError("block programs write one output")
        code, nregs = self.allocate()
        if len(code) > MAX_CODE or len(self.consts) > MAX_CONST:
            raise CompileError("block program too long")
        consts = [0] * len(self.consts)
        for word, i in self.consts.items():
            consts[i] = word
        names = list(self.slots)
        tile_extents = tuple(self.extents[:self.tile_axes])
        prog = Program(code, consts, [], names, tile_extents, nregs,
                       [math.prod(self.pkg.buffers[b].shape or (1,)) for b in names], list(self.loop_extents))
        layout = {"threads": self.threads, "n_block_axes": self.n_block_axes,
                  "smem": [[off, max(1, math.prod(shape))] for _, off, shape in
                           sorted(self.smem.values())]}
        return prog, layout, self.writes[0][0]


def compile_blockprog(pkg: KernelPackage, tile: Node):
    """Plan of any Tile body as a block program."""
    from .recognize import _plan
    comp = BlockCompiler(pkg, tile)
    prog, layout, out = comp.compile_block(tuple(tile.body))
    bind = {f"buf{i}": name for i, name in enumerate(prog.buffers)}
    blocks = math.prod(prog.extents[:layout["n_block_axes"]]) if layout["n_block_axes"] else 1
    return _plan(pkg, "blockprog", "lc_blockprog", bind,
                 {"program": prog.to_json(), "layout": layout, "out": out, "blocks": blocks, "block": True},
                 {name: pkg.buffers[name].dtype for name in prog.buffers})
