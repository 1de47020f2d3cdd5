"""CPU oracle of block-cooperative Tile bodies — TEST INFRASTRUCTURE ONLY.

Evaluates a Tile the way its blocks run it, over every thread of every block
at once with numpy, in lockstep: statement by statement, loop iteration by
loop iteration.  It covers the reference's staged scalar matmul
(ptx_backend.py:1496-1554 Loop / StridedLoop / Accum, the cp.async copies
into shared memory and their commit / wait, bar.sync, :1597-1631 plain and
atomic Writes) and any body built from the same statements:

* the trailing Tile axes whose extents multiply to ``block_threads`` are a
  block's threads, the leading axes number the blocks; every Smem array is
  one copy per block, filled with NaN so a read of an element no copy wrote
  shows in the result;
* a CpAsyncCopy lands at once (lockstep is one valid order of a race-free
  program, and the copy's own wait comes before any read of it);
* a loop with a per-thread start runs, for each thread, the iterations
  ``start, start + step, ... < extent``; statements of an iteration a thread
  does not run change nothing for it (accumulators, copies and writes are
  masked; loads are clamped for masked threads);
* Init / Accum as in the serial oracle: op(base or accumulator, value) in
  statement order, an accumulator seeded with its identity on entry to a
  seeding loop; integer index division and remainder as on non-negative
  values, TernaryExpr indices per thread.

When the package states a tolerance, the dot accumulators the reference
compensates are Dot2 pairs (oracle/dot2_ir.py), read as hi + lo; shuffle and
tree merges and every other write clear lo.  Scalar rules and accurate
float64 transcendentals come from oracle/pointwise_ir.py.  It shares only
the IR reader with the product.
"""
from __future__ import annotations

import math

import numpy as np

from oracle import dot2_ir

from oracle.pointwise_ir import PointwiseOracle, V, _t, conv
from oracle.serial_ir import _IDENTITY


class StagedOracle(PointwiseOracle):
    def __init__(self, pkg, tile, arrays: dict):
        super().__init__(pkg, tile, arrays)
        threads = int(tile.get("block_threads") or (pkg.kernel_meta.get("block") or [0])[0])
        prod, split = 1, len(self.axes)
        while split > 0 and prod < threads:
            split -= 1
            prod *= self.ext[split]
        if prod != threads:
            raise ValueError("oracle: the trailing Tile axes do not form the thread block")
        n = len(next(iter(self.coord.values())))
        self.n = n
        block = np.zeros(n, np.int64)
        for name, extent in zip(self.axes[:split], self.ext[:split]):
            block = block * extent + self.coord[name]
        self.block = block
        self.n_blocks = int(math.prod(self.ext[:split]))
        self.mask = np.ones(n, bool)
        self.smem: dict = {}
        self.smem_shape: dict = {}
        tid = np.zeros(n, np.int64)
        for name, extent in zip(self.axes[split:], self.ext[split:]):
            tid = tid * extent + self.coord[name]
        self.threads = threads
        self.coord["lane"], self.coord["warp"] = tid % 32, tid // 32
        self.env["lane"] = V((tid % 32).astype(np.int32), "s32")
        self.env["warp"] = V((tid // 32).astype(np.int32), "s32")
        zero = set(pkg.kernel_meta.get("zero_outputs", []))
        for name, buf in pkg.buffers.items():
            if buf.role == "output" and name in zero:
                t = _t(buf.dtype)
                self.out[name] = np.zeros(math.prod(buf.shape or (1,)), np.float32 if t != "s32" else np.int32)

    # -------------------------------------------------------- indices
    def index(self, e):
        if isinstance(e, int):
            return np.int64(e)
        if e.kind == "BinaryExpr" and e.op in ("/", "//", "%"):
            a, b = self.index(e.left), self.index(e.right)
            b = np.where(b == 0, 1, b)
            return a // b if e.op != "%" else a % b
        if e.kind == "BinaryExpr" and e.op in ("<", "<=", ">", ">=", "==", "!="):
            a, b = self.index(e.left), self.index(e.right)
            return {"<": a < b, "<=": a <= b, ">": a > b, ">=": a >= b, "==": a == b, "!=": a != b}[e.op]
        if e.kind == "TernaryExpr":
            return np.where(self.index(e.cond), self.index(e.if_true), self.index(e.if_false))
        return super().index(e)

    def _flat_smem(self, name, index):
        shape = self.smem_shape[name]
        idx = [np.asarray(self.index(i), np.int64) for i in index]
        flat = sum(i * math.prod(shape[d + 1:]) for d, i in enumerate(idx))
        return np.broadcast_to(flat, (self.n,))

    def _clamped(self, flat, size):
        flat = np.broadcast_to(np.asarray(flat, np.int64), (self.n,))
        bad = self.mask & ((flat < 0) | (flat >= size))
        if bad.any():
            raise IndexError("oracle: an active thread addresses outside its buffer")
        return np.where(self.mask, flat, 0)

    # -------------------------------------------------------- statements
    # -------------------------------------------------------- compensated (Dot2) states
    def comp(self) -> set:
        return self.__dict__.setdefault("_comp", dot2_ir.compensated(self.pkg.body, self.pkg))

    def put(self, name, new, lo=None, masked=True) -> None:
        """An accumulator's new value where the threads are active; a compensated one
        keeps (hi, lo) and reads as their value, every other write clearing lo."""
        new = np.broadcast_to(np.asarray(new, np.float32), (self.n,))
        lo = np.zeros(self.n, np.float32) if lo is None else np.broadcast_to(lo, (self.n,))
        old = self.env.get(name)
        if name in self.comp():
            pairs = self.__dict__.setdefault("_dot2", {})
            old_hi, old_lo = pairs.get(name, (np.zeros(self.n, np.float32), np.zeros(self.n, np.float32)))
            hi = np.where(self.mask, new, old_hi) if masked else np.array(new)
            lo = np.where(self.mask, lo, old_lo) if masked else np.array(lo)
            pairs[name] = (hi.astype(np.float32), lo.astype(np.float32))
            self.env[name] = V(dot2_ir.value(*pairs[name]), "f32")
        elif masked and old is not None:
            self.env[name] = V(np.where(self.mask, new, conv(old, "f32").a), "f32")
        else:
            self.env[name] = V(np.array(new, np.float32), "f32")

    def run_block(self, body) -> None:
        previous = None
        for s in body:
            prev, previous = previous, s
            k = s.kind
            if k == "Smem":
                shape = tuple(int(x) for x in s.extents)
                self.smem_shape[s.name] = shape
                self.smem[s.name] = np.full((self.n_blocks, math.prod(shape)), np.nan, np.float32)
            elif k == "CpAsyncCopy":
                self.copy(s)
            elif k in ("CpAsyncCommit", "CpAsyncWait", "Sync"):
                pass
            elif k == "Load" and s.input in self.smem:
                size = self.smem[s.input].shape[1]
                flat = self._flat_smem(s.input, s.index)
                for lane, name in enumerate(s.names):
                    self.env[name] = V(self.smem[s.input][self.block, self._clamped(flat + lane, size)], "f32")
            elif k == "Load":
                buf = self.pkg.buffers[s.input]
                size = math.prod(buf.shape or (1,))
                flat = self.flat(s.input, s.index)
                t = _t(buf.dtype)
                for lane, name in enumerate(s.names):
                    vals = self.arrays[s.input][self._clamped(flat + lane, size)]
                    self.env[name] = V(np.asarray(vals, np.float32 if t != "s32" else np.int32), t)
            elif k in ("Loop", "StridedLoop"):
                self.loop(s)
            elif k == "Init":
                self.put(s.name, np.full(self.n, float(s.identity), np.float32), masked=False)
            elif k == "Accum" and s.name in self.__dict__.get("_dot2", {}) and dot2_ir.adjacent(prev, s):
                hi, lo = self._dot2[s.name]
                a, b = (conv(self.env[x] if isinstance(x, str) else self.expr(x), "f32").a for x in prev.args)
                self.put(s.name, *dot2_ir.step(hi, lo, np.broadcast_to(a, (self.n,)), np.broadcast_to(b, (self.n,))))
            elif k == "Accum":
                opname = s.op.name if hasattr(s.op, "name") else str(s.op)
                old = self.env[s.name]
                base = self.env[s.base] if s.get("base") else old
                value = self.env[s.value] if isinstance(s.value, str) else self.expr(s.value)
                new = conv(self.op(opname, [conv(base, "f32"), conv(value, "f32")], "f32"), "f32")
                self.put(s.name, new.a)
            elif k == "Cond":
                saved = self.mask
                self.mask = saved & np.broadcast_to(conv(self.expr(s.cond), "pred").a, (self.n,))
                self.run_block(s.body)
                self.mask = saved
                if s.get("else_body"):
                    self.mask = saved & ~np.broadcast_to(conv(self.expr(s.cond), "pred").a, (self.n,))
                    self.run_block(s.else_body)
                    self.mask = saved
            elif k == "Write" and s.output in self.smem:
                size = self.smem[s.output].shape[1]
                flat = self._flat_smem(s.output, s.index)
                live = self.mask
                for lane, name in enumerate(s.values):
                    idx = np.broadcast_to(flat + lane, (self.n,))
                    ok = live & (idx >= 0) & (idx < size)
                    vals = np.broadcast_to(conv(self.env[name], "f32").a, (self.n,))
                    self.smem[s.output][self.block[ok], idx[ok]] = vals[ok]
            elif k == "Write":
                self.write(s)
            elif k == "WarpShuffle":
                self.shuffle(s)
            elif k == "TreeHalve":
                self.tree(s)
            else:
                self.run([s])

    def copy(self, s) -> None:
        if s.get("swizzle", "NONE") not in (None, "NONE"):
            raise ValueError("oracle: swizzled copies")
        src = self.pkg.buffers[s.src]
        elems = int(s.nbytes) // np.dtype(np.float32 if _t(src.dtype) == "f32" else np.float16).itemsize
        sidx = list(s.smem_index)
        lane = s.get("lane_index")
        shape = self.smem_shape[s.smem]
        pos = [np.asarray(self.index(i), np.int64) for i in sidx]
        if lane is not None:
            pos = [p + np.asarray(self.index(i), np.int64) for p, i in zip(pos, lane)]
        dst = np.broadcast_to(sum(p * math.prod(shape[d + 1:]) for d, p in enumerate(pos)), (self.n,))
        gsrc = self.flat(s.src, s.src_index)
        size = math.prod(src.shape or (1,))
        live = self.mask
        for e in range(elems):
            g = self._clamped(gsrc + e, size)
            d = self._clamped(dst + e, self.smem[s.smem].shape[1])
            vals = np.asarray(self.arrays[s.src][g], np.float32)
            self.smem[s.smem][self.block[live], d[live]] = vals[live]

    def write(self, s) -> None:
        buf = self.pkg.buffers[s.output]
        t = _t(buf.dtype)
        size = math.prod(buf.shape or (1,))
        out = self.out.setdefault(s.output, np.full(size, np.nan if t != "s32" else -1,
                                                    np.float32 if t != "s32" else np.int32))
        flat = self.flat(s.output, s.index)
        live = self.mask
        for lane, name in enumerate(s.values):
            idx = self._clamped(flat + lane, size)
            vals = np.broadcast_to(conv(self.env[name], t).a, (self.n,))
            if s.get("atomic"):
                acc = out.astype(np.float64)
                np.add.at(acc, idx[live], vals[live].astype(np.float64))
                out[:] = acc.astype(out.dtype)
            else:
                out[idx[live]] = vals[live]

    def loop(self, s) -> None:
        extent = int(s.axis.extent.value)
        start = s.get("start")
        step = s.get("step")
        start_v = np.broadcast_to(np.asarray(self.index(start) if start is not None else 0, np.int64), (self.n,))
        step_v = int(np.asarray(self.index(step))) if step is not None else 1
        if step_v <= 0:
            raise ValueError("oracle: loops count up in positive steps")
        end = s.get("end")
        # a captured end is evaluated once on entry and replaces the extent as the bound
        bound = np.broadcast_to(np.asarray(self.index(end), np.int64), (self.n,)) if end is not None \
            else np.full(self.n, extent, np.int64)
        if end is not None:
            self.env[s.axis.name + "_end"] = V(bound.astype(np.int32), "s32")
        if s.get("seed", True):
            for inner in s.body:
                if inner.kind == "Accum":
                    opname = inner.op.name if hasattr(inner.op, "name") else str(inner.op)
                    seed = np.full(self.n, _IDENTITY[opname], np.float32)
                    self.put(inner.name, seed, masked=inner.name in self.env)
        saved = self.mask
        i = 0
        while True:
            var = start_v + i * step_v
            live = saved & (var < bound)
            if not live.any():
                break
            self.mask = live
            self.coord[s.axis.name] = var
            self.run_block(s.body)
            i += 1
        self.mask = saved
        self.coord.pop(s.axis.name, None)

    def merge(self, s) -> None:
        for a in s.combine_states:
            opname = a.op.name if hasattr(a.op, "name") else str(a.op)
            new = conv(self.op(opname, [conv(self.env[x], "f32") for x in a.args], "f32"), "f32")
            if a.name in s.state:
                self.put(a.name, new.a, masked=False)
            else:
                self.env[a.name] = new

    def shuffle(self, s) -> None:
        """The reference's butterfly: at each level every lane takes the states of
        the lane ``delta`` away and runs the combine statements."""
        partial = self.threads < 32 and not self.threads & (self.threads - 1) and int(s.length) <= self.threads
        if self.threads % 32 and int(s.length) > 1 and not partial:
            raise ValueError("oracle: shuffles need whole warps (or one power-of-two partial warp)")
        saved = dict(self.env)
        points = np.arange(self.n)
        delta = int(s.length) // 2
        while delta:
            for a, b in zip(s.state, s.state_b):
                self.env[b] = V(conv(self.env[a], "f32").a[points ^ delta], "f32")
            self.merge(s)
            delta //= 2
        kept = {name: self.env[name] for name in s.state}
        self.env = {**saved, **kept}

    def tree(self, s) -> None:
        """The reference's shared tree: at each level the threads below ``delta``
        (lane 0 of each warp when the tree runs over warps) fold the slot
        ``delta`` away into their own; then every thread reads slot ``inner``."""
        tid = np.asarray(self.coord[s.tid_var] if s.tid_var in self.coord else self.env[s.tid_var].a, np.int64)
        inner = s.get("inner")
        if inner:
            base = np.asarray(self.coord.get(inner[0], None) if inner[0] in self.coord
                              else self.env[inner[0]].a, np.int64)
            scale = int(inner[1])
        else:
            base, scale = np.zeros(self.n, np.int64), 1
        slot = tid * scale + base
        saved = dict(self.env)
        delta = int(s.length) // 2
        while delta:
            worker = self.mask & (tid < delta)
            if s.tid_var == "warp" and not inner:
                worker = worker & (self.coord["lane"] == 0)
            other = slot + delta * scale
            for buf, a, b in zip(s.bufs, s.state, s.state_b):
                arr = self.smem[buf]
                size = arr.shape[1]
                self.env[a] = V(arr[self.block, np.clip(slot, 0, size - 1)], "f32")
                self.env[b] = V(arr[self.block, np.clip(other, 0, size - 1)], "f32")
            self.merge(s)
            for buf, name in zip(s.bufs, s.state):
                arr = self.smem[buf]
                vals = np.broadcast_to(conv(self.env[name], "f32").a, (self.n,))
                arr[self.block[worker], slot[worker]] = vals[worker]
            delta //= 2
        self.env = saved
        for buf, name in zip(s.bufs, s.state):
            arr = self.smem[buf]
            self.put(name, arr[self.block, np.clip(base, 0, arr.shape[1] - 1)], masked=False)

    def result(self) -> dict:
        return {k: v.reshape(tuple(self.pkg.buffers[k].shape) or (1,)) for k, v in self.out.items()}


def evaluate(ir_path, arrays: dict) -> dict:
    """Outputs of the block-cooperative package at ``ir_path`` on named input arrays."""
    from lazy_compiler_b200.ir import load_package
    pkg = load_package(ir_path)
    (tile,) = pkg.body
    oracle = StagedOracle(pkg, tile, arrays)
    oracle.run_block(tile.body)
    return oracle.result()
