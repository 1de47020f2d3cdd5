"""CPU oracle of reduction / fused row Tiles — TEST INFRASTRUCTURE ONLY.

Evaluates a Tile of [row,] cooperating threads directly from its IR with
numpy, by what the schedule computes rather than how: the threads of a
StridedLoop pass collectively visit every column of the row, so a pass's
body is evaluated on all (row, column) points at once, each Accum folds its
per-element values over the columns (float64, then rounded to f32), and
after the pass the accumulator is that row's fold — the WarpShuffle /
TreeHalve combines only distribute it.  A write guarded to the first thread
is a per-row write.  Scalar statements follow oracle/pointwise_ir.py's rules.

A pass whose accumulators fold through an explicit base (coupled online
states, the f02 softmax) has no closed-form fold: there every one of the
block's threads updates its running states over its strided columns in
order, and the threads' states merge one after another through the
WarpShuffle's own combine statements.
"""
from __future__ import annotations


import numpy as np

from oracle.pointwise_ir import PointwiseOracle, V, conv

_FOLD = {"add": np.sum, "sum": np.sum, "multiply": np.prod, "mul": np.prod,
         "maximum": np.max, "max": np.max, "minimum": np.min, "min": np.min}
# Fold identities as Emmy seeds them: max / min start at the finite -1e30 / 1e30
# (an empty lane's state then combines without inf - inf).
_IDENTITY = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "mul": 1.0, "maximum": -1e30, "max": -1e30,
             "minimum": 1e30, "min": 1e30, "fmax": -1e30, "fmin": 1e30}


class RowOracle(PointwiseOracle):
    def __init__(self, pkg, tile, arrays):
        axes = [(a.name, int(a.extent.value)) for a in tile.axes]
        self.pkg = pkg
        self.co, self.block = axes[-1]
        self.row_axes = axes[:-1] or [("__row", 1)]
        self.rows = int(np.prod([e for _, e in self.row_axes]))
        grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for _, e in self.row_axes], indexing="ij")
        self.row_coords = {n: g.ravel() for (n, _), g in zip(self.row_axes, grids)}
        self.arrays = {k: np.asarray(v).ravel() for k, v in arrays.items()}
        self.env = {}
        self.out = {}
        self.set_domain(None, 1)

    def set_domain(self, col, cols):
        self.coord = {n: np.repeat(v, cols) for n, v in self.row_coords.items()}
        self.coord[self.co] = np.zeros(self.rows * cols, np.int64)
        if col is not None:
            self.coord[col] = np.tile(np.arange(cols, dtype=np.int64), self.rows)
        self.cols = cols

    def widen(self, cols):
        """Row values seen inside a pass: one copy per column."""
        for k, v in list(self.env.items()):
            if isinstance(v, V) and v.a.shape == (self.rows,):
                self.env[k] = V(np.repeat(v.a, cols), v.t)

    def narrow(self, cols):
        for k, v in list(self.env.items()):
            if isinstance(v, V) and v.a.shape == (self.rows * cols,):
                self.env[k] = V(v.a.reshape(self.rows, cols)[:, 0], v.t)

    def coupled_pass(self, loop, combine, block):
        """Per-thread sequential folds, then thread-by-thread merges (see the module docstring)."""
        cols = int(loop.axis.extent.value)
        accs = [st for st in loop.body if st.kind == "Accum"]
        names = [a.name for a in accs]
        inits = {st.name: float(st.identity) for st in self.tile_body if st.kind == "Init"}
        ident = {a.name: inits.get(a.name, _IDENTITY[a.op.name if hasattr(a.op, "name") else str(a.op)])
                 for a in accs}
        n = self.rows * block
        part = {nm: np.full(n, ident[nm], np.float32) for nm in names}
        saved = dict(self.env)
        t = np.tile(np.arange(block, dtype=np.int64), self.rows)
        for it in range(-(-cols // block)):
            c = it * block + t
            valid = c < cols
            self.coord = {n: np.repeat(v, block) for n, v in self.row_coords.items()}
            self.coord.update({self.co: t, loop.axis.name: np.minimum(c, cols - 1)})
            self.env = {k: (V(np.repeat(v.a, block), v.t) if isinstance(v, V) and v.a.shape == (self.rows,) else v)
                        for k, v in saved.items()}
            for nm in names:
                self.env[nm] = V(part[nm], "f32")
            for st in loop.body:
                if st.kind == "Accum":
                    opname = st.op.name if hasattr(st.op, "name") else str(st.op)
                    base = self.env[st.base] if st.get("base") else self.env[st.name]
                    value = self.env[st.value] if isinstance(st.value, str) else self.expr(st.value)
                    new = conv(self.op(opname, [conv(base, "f32"), conv(value, "f32")], "f32"), "f32").a
                    part[st.name] = np.where(valid, new, part[st.name]).astype(np.float32)
                    self.env[st.name] = V(part[st.name], "f32")
                elif st.kind != "Write":
                    self.run([st])
        self.env = saved
        self.set_domain(None, 1)
        own = {nm: part[nm].reshape(self.rows, block)[:, 0].copy() for nm in names}
        for th in range(1, block):
            env = dict(self.env)
            self.env = dict(env)
            for a, b in zip(combine.state, combine.state_b):
                self.env[a] = V(own[a], "f32")
                self.env[b] = V(part[a].reshape(self.rows, block)[:, th], "f32")
            for st in combine.get("combine_states") or ():
                self.run([st])
            for a in combine.state:
                own[a] = conv(self.env[a], "f32").a.copy()
            self.env = env
        for nm in names:
            self.env[nm] = V(own[nm], "f32")

    def run_rows(self, body) -> dict:
        self.tile_body = body
        items = list(body)
        for i, s in enumerate(items):
            k = s.kind
            if k in ("StridedLoop", "Loop") and any(st.kind == "Accum" and st.get("base") for st in s.body):
                combine = next(x for x in items[i + 1:] if x.kind == "WarpShuffle")
                self.coupled_pass(s, combine, self.block)
                continue
            if k in ("StridedLoop", "Loop"):
                cols = int(s.axis.extent.value)
                folds = {}
                self.widen(cols)
                self.set_domain(s.axis.name, cols)
                for inner in s.body:
                    if inner.kind == "Accum":
                        opname = inner.op.name if hasattr(inner.op, "name") else str(inner.op)
                        value = conv(self.env[inner.value] if isinstance(inner.value, str)
                                     else self.expr(inner.value), "f32").a
                        folds[inner.name] = (opname, value)
                    else:
                        self.run_rows([inner])
                self.narrow(cols)
                self.set_domain(None, 1)
                for name, (opname, value) in folds.items():
                    with np.errstate(all="ignore"):
                        r = _FOLD[opname](value.reshape(self.rows, cols).astype(np.float64), axis=1)
                    self.env[name] = V(r.astype(np.float32), "f32")
            elif k == "Init":
                self.env[s.name] = V(np.full(self.rows, _IDENTITY.get(str(s.identity), float(s.identity)),
                                             np.float32), "f32")
            elif k in ("WarpShuffle", "TreeHalve", "Smem", "Sync"):
                continue    # the pass above already produced the combined states
            elif k == "Cond":
                self.run_rows(s.body)
            elif k == "Write" and s.output not in self.pkg.buffers:
                continue                    # shared-memory staging of partials
            else:
                self.run([s])
        return {k: v.reshape(tuple(self.pkg.buffers[k].shape) or (1,)) for k, v in self.out.items()}


def evaluate(ir_path, arrays: dict) -> dict:
    """Outputs of the reduction package at ``ir_path`` on named input arrays."""
    from lazy_compiler_b200.ir import load_package
    pkg = load_package(ir_path)
    (tile,) = pkg.body
    return RowOracle(pkg, tile, arrays).run_rows(tile.body)
