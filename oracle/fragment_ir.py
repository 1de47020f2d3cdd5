"""CPU oracle of one-warp tensor-fragment programs — TEST INFRASTRUCTURE ONLY.

Evaluates a fragment program on whole matrices rather than lanes: a C
fragment is a 16 x 8 f32 array, an A fragment the 16 x 16 and a B fragment
the 16 x 8 operand values rounded to the fragment type.  It follows the
reference's definitions (ptx_tensor.py):

* global gathers: rows past the M/N guard repeat the last valid row, the K
  tail reads as zero (:324-363); operands round to nearest to f16/bf16;
* MMA: the float64 product of the rounded operands plus C, rounded to f32;
* FragmentApply: the operation per element with __frow = row_base + row and
  __fcol = col_base + column, GMEM operands gathered, ``where`` selecting,
  the ``post`` chain applied, all in f32 (:480-588);
* FragmentRowReduce: each lane folds its two columns of every listed
  fragment left to right, then lanes 2 apart and 1 apart combine — per row
  the value (L0 op L2) op (L1 op L3) with L_t lane t's fold (:590-618);
* FragmentRepack: two C fragments side by side, rounded (:459-473);
* RegStore: elements whose guards hold, through the epilogue lambda with the
  element's fragment-local row and column (:383-457).

Transcendentals are numpy's accurate float64 functions rounded to f32; the
GPU program uses the reference's ex2.approx sequence, so values agree to the
packages' tolerances.  It shares only the IR reader and the scalar rules of
oracle/pointwise_ir.py with anything else.
"""
from __future__ import annotations

import math
import re

import numpy as np

from oracle.expressions import quantize
from oracle.pointwise_ir import PointwiseOracle, V, conv

ROWS = np.repeat(np.arange(16), 8)        # element e of a 16 x 8 tile: row e // 8, column e % 8
COLS = np.tile(np.arange(8), 16)


class FragmentOracle(PointwiseOracle):
    def __init__(self, pkg, tile, arrays):
        self.pkg = pkg
        self.axes = ["__row", "__col"]
        self.coord = {"__row": ROWS.astype(np.int64), "__col": COLS.astype(np.int64)}
        self.arrays = {k: np.asarray(v).ravel() for k, v in arrays.items()}
        self.env = {}
        self.static = {}
        self.frags = {}
        self.out = {}
        lane_axis = tile.axes[0].name
        self.env[lane_axis] = V(((ROWS % 8) * 4 + COLS // 2).astype(np.int32), "s32")   # the element's lane

    # -------------------------------------------------------- scalars
    def expr(self, e):
        if hasattr(e, "kind") and e.kind == "Var" and e.name in self.static:
            return self.lit(self.static[e.name], "s32")
        return super().expr(e)

    def ints(self, e) -> np.ndarray:
        return conv(self.expr(e), "s32").a.astype(np.int64)

    def flat(self, buffer, index):
        shape = tuple(self.pkg.buffers[buffer].shape) or (1,)
        if not index:
            return np.zeros(128, np.int64)
        if len(index) == 1:
            return self.ints(index[0])
        total = np.zeros(128, np.int64)
        for d, i in enumerate(index):
            stride = math.prod(shape[d + 1:]) if len(index) == len(shape) else 1
            total = total + self.ints(i) * stride
        return total

    def gather(self, buffer, at):
        data = self.arrays[buffer]
        return np.asarray(data, np.float32)[np.clip(at, 0, data.size - 1)]

    # -------------------------------------------------------- fragments
    def ref(self, text):
        m = re.fullmatch(r"([A-Za-z_$][\w$]*)(?:\[([A-Za-z_$][\w$]*|[0-9]+)\])?", str(text))
        stem, sub = m.groups()
        idx = 0 if sub is None else (int(sub) if sub.isdecimal() else self.static[sub])
        return self.frags[stem], idx

    def run_fragments(self, body):
        for s in body:
            k = s.kind
            if k in ("StridedLoop", "Loop"):
                start = int(self.expr(s.start).a[0]) if k == "StridedLoop" and s.get("start") is not None else 0
                step = int(self.expr(s.step).a[0]) if k == "StridedLoop" and s.get("step") is not None else 1
                end = s.get("end") if k == "StridedLoop" else None
                bound = int(self.expr(end).a[0]) if end is not None else int(s.axis.extent.value)
                for v in range(start, bound, step):
                    self.static[s.axis.name] = v
                    self.run_fragments(s.body)
                self.static.pop(s.axis.name, None)
            elif k == "RegFragment":
                shape = {"a": (16, 16), "b": (16, 8), "c": (16, 8)}[s.role]
                self.frags[s.name] = {"role": s.role, "dtype": s.dtype.name if hasattr(s.dtype, "name")
                                      else str(s.dtype), "m": [np.zeros(shape) for _ in range(int(s.get("count") or 1))]}
            elif k == "LdmatrixLoad":
                self.load(s)
            elif k == "MmaSyncPtx":
                a, ai = self.ref(s.a_frag)
                b, bi = self.ref(s.b_frag)
                c, ci = self.ref(s.c_frag)
                c["m"][ci] = (a["m"][ai] @ b["m"][bi] + c["m"][ci]).astype(np.float32).astype(np.float64)
            elif k == "FragmentApply":
                self.apply(s)
            elif k == "FragmentRowReduce":
                self.row_reduce(s)
            elif k == "FragmentRepack":
                a, ai = self.ref(s.frag)
                c0, c1 = (self.ref(x) for x in s.srcs)
                m = np.concatenate([c0[0]["m"][c0[1]], c1[0]["m"][c1[1]]], axis=1)
                a["m"][ai] = quantize(m, s.ab_dtype).astype(np.float64)
            elif k == "RegStore":
                self.store(s)
            elif k in ("Let", "Assign", "Select"):
                self.run([s])
            else:
                raise ValueError(f"oracle: fragment statement {k}")
        return {k: v.reshape(tuple(self.pkg.buffers[k].shape) or (1,)) for k, v in self.out.items()}

    def load(self, s):
        frag, idx = self.ref(s.frag)
        buf = self.pkg.buffers[s.src_buffer]
        ldm = int(s.get("ldm") or buf.shape[-1])
        base = int(self.flat(s.src_buffer, tuple(s.src_index))[0])
        if s.role == "a":
            mn, kk = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
        else:
            kk, mn = np.meshgrid(np.arange(16), np.arange(8), indexing="ij")
        valid = np.ones(mn.shape, bool)
        if s.get("gmem_guard") is not None:
            rem = int(self.ints(s.gmem_guard[1])[0] - self.ints(s.gmem_guard[0])[0])
            valid &= rem > 0
            mn = np.minimum(mn, max(rem - 1, 0))
        if s.get("k_zero") is not None:
            remk = int(self.ints(s.k_zero[1])[0] - self.ints(s.k_zero[0])[0])
            valid &= kk < remk
        row, col = (mn, kk) if s.role == "a" or s.get("b_trans") else (kk, mn)
        data = np.asarray(self.arrays[s.src_buffer], np.float32)
        at = np.clip(base + row * ldm + col, 0, data.size - 1)
        vals = np.where(valid, data[at], np.float32(0))
        frag["m"][idx] = quantize(vals, frag["dtype"]).astype(np.float64)

    def element_coords(self, s):
        self.env.pop("__frow", None)
        self.env.pop("__fcol", None)
        if s.get("row_base") is not None:
            self.env["__frow"] = V((self.ints(s.row_base) + ROWS).astype(np.int32), "s32")
        if s.get("col_base") is not None:
            self.env["__fcol"] = V((self.ints(s.col_base) + COLS).astype(np.int32), "s32")

    def apply(self, s):
        saved = dict(self.env)
        self.element_coords(s)
        ops = []
        for arg, kind in zip(s.args, s.kinds):
            if kind == "frag":
                f, i = self.ref(arg)
                ops.append(V(f["m"][i].ravel().astype(np.float32), "f32"))
            elif kind == "row":
                top, bot = (conv(self.env[n], "f32").a for n in arg)
                ops.append(V(np.where(ROWS < 8, top, bot).astype(np.float32), "f32"))
            elif kind in ("coord", "uniform"):
                v = self.env[arg] if isinstance(arg, str) else self.expr(arg)
                ops.append(v if kind == "coord" else conv(v, "f32"))
            elif kind == "gmem":
                buffer, index = arg
                ops.append(V(self.gather(buffer, self.flat(buffer, tuple(index))), "f32"))
            else:
                raise ValueError(kind)
        name = s.op.name if hasattr(s.op, "name") else str(s.op)
        if name == "where":
            c = conv(ops[0], "pred").a
            value = V(np.where(c, conv(ops[1], "f32").a, conv(ops[2], "f32").a), "f32")
        else:
            value = self.op(name, ops, "f32")
        for post in s.get("post") or ():
            value = self.op(post.name if hasattr(post, "name") else str(post), [value], "f32")
        self.env = saved
        result = conv(value, "f32").a.reshape(16, 8).astype(np.float64)
        if s.get("in_place"):
            f, i = self.ref(s.out)
            f["m"][i] = result
        else:
            self.frags[s.out] = {"role": "c", "dtype": "f32", "m": [result]}

    def row_reduce(self, s):
        name = s.op.name if hasattr(s.op, "name") else str(s.op)
        fn = {"add": np.add, "multiply": np.multiply, "maximum": np.fmax, "minimum": np.fmin}[name]
        mats = [self.ref(f) for f in s.frags]
        mats = [f["m"][i].astype(np.float32) for f, i in mats]
        with np.errstate(all="ignore"):
            lanes = []
            for t in range(4):
                part = None
                for m in mats:
                    for col in (2 * t, 2 * t + 1):
                        part = m[:, col] if part is None else fn(part, m[:, col]).astype(np.float32)
                lanes.append(part)
            rows = fn(fn(lanes[0], lanes[2]), fn(lanes[1], lanes[3])).astype(np.float32)
        self.env[s.top] = V(rows[:8][ROWS % 8], "f32")
        self.env[s.bot] = V(rows[8:][ROWS % 8], "f32")

    def store(self, s):
        f, i = self.ref(s.frag)
        buf = self.pkg.buffers[s.dst_buffer]
        dt = buf.dtype
        shape = tuple(buf.shape)
        rd, cd = s.get("row_dim"), s.get("col_dim")
        row_stride = int(s.get("ldm") or 0) or (math.prod(shape[rd + 1:]) if rd is not None else shape[-1])
        col_stride = math.prod(shape[cd + 1:]) if cd is not None else 1
        base = int(self.flat(s.dst_buffer, tuple(s.dst_index))[0])
        ok = np.ones(128, bool)
        for guard, off in ((s.get("m_guard"), ROWS), (s.get("n_guard"), COLS)):
            if guard is not None:
                ok &= self.ints(guard[0]) + off < self.ints(guard[1])
        value = V(f["m"][i].ravel().astype(np.float32), "f32")
        if s.get("epilogue") is not None:
            value = self.epilogue(s.epilogue, value)
        value = conv(value, "f32").a
        if dt in ("f16", "bf16"):
            value = quantize(value, dt)
        out = self.out.setdefault(s.dst_buffer, np.full(math.prod(shape), np.nan, np.float32))
        at = base + ROWS * row_stride + COLS * col_stride
        live = ok & (at >= 0) & (at < out.size)
        if s.get("atomic"):
            out[np.isnan(out)] = 0.0
            np.add.at(out, at[live], value[live])
        else:
            out[at[live]] = value[live]

    def epilogue(self, lam, acc):
        saved = dict(self.env)
        self.env[lam.params[0]] = acc
        self.env["__M__"] = V(ROWS.astype(np.int32), "s32")
        self.env["__N__"] = V(COLS.astype(np.int32), "s32")
        for st in lam.body:
            if st.kind == "Load":
                self.env[st.names[0]] = V(self.gather(st.input, self.flat(st.input, tuple(st.index))), "f32")
            else:
                self.run([st])
        out = self.env[lam.results[0]]
        self.env = saved
        return out


def evaluate(ir_path, arrays: dict) -> dict:
    """Outputs of the one-warp fragment package at ``ir_path`` on named input arrays."""
    from lazy_compiler_b200.ir import load_package
    pkg = load_package(ir_path)
    (tile,) = pkg.body
    return FragmentOracle(pkg, tile, arrays).run_fragments(tile.body)
