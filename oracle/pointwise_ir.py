"""CPU oracle of straight-line pointwise Tile bodies — TEST INFRASTRUCTURE ONLY.

Evaluates a Tile body of Load / Let / Assign / Select / Write statements over
every tile point at once with numpy, following the reference's typing rules
(ptx_backend.py:470-537 conversions, :618-630 promotion, :650-716 comparisons
and binary operators with per-node f16/bf16 rounding, :981-984 per-statement
narrow rounding) but with accurate transcendentals: exp, log, sin, cos,
tanh and erf come from numpy / math in float64 and are rounded to f32 once,
GELU from the formula of tests/test_gelu.py:51-66.  The GPU program uses the
reference's approximations (ex2.approx, the Abramowitz-Stegun erf), so
values agree to the packages' tolerances, not bit for bit.

It shares only the IR reader with the product; the evaluation is its own.
"""
from __future__ import annotations

import math

import numpy as np

from oracle.expressions import quantize

_TYPES = {"float": "f32", "int": "s32", "i32": "s32", "__half": "f16", "half": "f16",
          "__nv_bfloat16": "bf16", "bool": "pred"}
_FLOATS = ("f32", "f16", "bf16")


def _t(dt) -> str:
    name = getattr(dt, "name", None) if not isinstance(dt, str) else dt
    if name is None and hasattr(dt, "get"):
        name = dt.get("name")
    name = _TYPES.get(str(name), str(name))
    if name not in ("f32", "f16", "bf16", "s32", "pred"):
        raise ValueError(f"oracle: unsupported type {name}")
    return name


class V:
    def __init__(self, a, t):
        self.a, self.t = a, t


def conv(v: V, t: str) -> V:
    """Conversion with the reference's rounding (ptx_backend.py:470-537)."""
    if v.t == t:
        return v
    a = v.a
    with np.errstate(all="ignore"):
        if t == "pred":
            return V(a != 0, "pred")                       # NaN != 0 is true
        if v.t == "pred":
            return V(a.astype(np.int32) if t == "s32" else a.astype(np.float32), t)
        if v.t == "s32" and t in _FLOATS:
            x = a.astype(np.float64)                       # exact; then one rounding
            if t == "f32":
                return V(x.astype(np.float32), t)
            if t == "f16":
                return V(x.astype(np.float16).astype(np.float32), t)
            m, e = np.frexp(x)
            return V(np.ldexp(np.rint(np.ldexp(m, 8)), e - 8).astype(np.float32), t)
        if t in _FLOATS:
            return V(quantize(a, t) if t != "f32" else a.astype(np.float32), t)
        # float -> s32: truncate toward zero, saturate, NaN -> 0 (cvt.rzi.s32)
        x = np.nan_to_num(np.trunc(a.astype(np.float64)), nan=0.0, posinf=2.0 ** 31, neginf=-2.0 ** 31)
        return V(np.clip(x, -2 ** 31, 2 ** 31 - 1).astype(np.int32), "s32")


def common(a: str, b: str) -> str:
    for t in _FLOATS:
        if t in (a, b):
            return t
    return "pred" if a == b == "pred" else "s32"


class PointwiseOracle:
    def __init__(self, pkg, tile, arrays: dict):
        self.pkg = pkg
        self.axes = [a.name for a in tile.axes]
        self.ext = [int(a.extent.value) for a in tile.axes]
        grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for e in self.ext], indexing="ij")
        self.coord = {n: g.ravel() for n, g in zip(self.axes, grids)}
        self.arrays = {k: np.asarray(v).ravel() for k, v in arrays.items()}
        self.env: dict = {}
        self.out: dict = {}

    # -------------------------------------------------------- values
    def lit(self, x, t="s32") -> V:
        n = len(next(iter(self.coord.values())))
        if t == "pred":
            return V(np.full(n, bool(x)), t)
        if t == "s32":
            return V(np.full(n, np.int64(int(x)) % (1 << 32), np.int64).astype(np.uint32).view(np.int32), t)
        with np.errstate(over="ignore"):
            v = np.float32(float(x))
        return conv(V(np.full(n, v, np.float32), "f32"), t)

    def cmp(self, op, a: V, b: V) -> V:
        t = common(a.t, b.t)
        t = "f32" if t == "bf16" else t
        x, y = conv(a, t).a, conv(b, t).a
        with np.errstate(invalid="ignore"):
            r = {"eq": x == y, "ne": x != y, "lt": x < y, "le": x <= y, "gt": x > y, "ge": x >= y}[op]
        return V(r, "pred")

    def binary(self, op, a: V, b: V, t=None) -> V:
        if op in ("&&", "||"):
            x, y = conv(a, "pred").a, conv(b, "pred").a
            return V(x & y if op == "&&" else x | y, "pred")
        names = {"<": "lt", "<=": "le", ">": "gt", ">=": "ge", "==": "eq", "!=": "ne"}
        if op in names:
            return self.cmp(names[op], a, b)
        t = t or common(a.t, b.t)
        t = "s32" if t == "pred" else t
        if t in ("f16", "bf16"):
            r = self.binary(op, conv(conv(a, t), "f32"), conv(conv(b, t), "f32"))
            return conv(r, t)
        x, y = conv(a, t).a, conv(b, t).a
        with np.errstate(all="ignore"):
            if t == "f32":
                r = {"+": x + y, "-": x - y, "*": x * y, "/": x / y}[op]
                return V(r.astype(np.float32), t)
            x64, y64 = x.astype(np.int64), y.astype(np.int64)
            safe = np.where(y64 == 0, 1, y64)
            q = np.where(y64 == 0, 0, np.trunc(x64 / safe).astype(np.int64))
            r = {"+": x64 + y64, "-": x64 - y64, "*": x64 * y64, "/": q,
                 "%": np.where(y64 == 0, x64, x64 - safe * q), "&": x64 & y64, "|": x64 | y64, "^": x64 ^ y64,
                 "<<": np.where(y64 >= 32, 0, x64 << np.clip(y64, 0, 31)),
                 ">>": x64 >> np.clip(y64, 0, 31)}[op]
        return V((r % (1 << 32)).astype(np.uint32).view(np.int32), "s32")

    def op(self, name, args, t) -> V:
        aliases = {"sum": "add", "prod": "multiply", "sub": "subtract", "mul": "multiply", "neg": "negative",
                   "exp_fast": "exp", "true_divide": "divide", "amax": "maximum", "max": "maximum",
                   "min": "minimum", "absolute": "abs"}
        name = aliases.get(name, name)
        if name in ("copy", "pad"):
            return conv(args[0], t)
        if name == "bitcast":
            a = args[0]
            if a.t == t:
                return a
            return V(a.a.view(np.int32) if t == "s32" else a.a.view(np.float32), t)
        if name == "where":
            c = conv(args[0], "pred").a
            tt = t
            return V(np.where(c, conv(args[1], tt).a, conv(args[2], tt).a), tt)
        comps = {"equal": "eq", "not_equal": "ne", "less": "lt", "less_equal": "le", "greater": "gt",
                 "greater_equal": "ge"}
        if name in comps:
            return conv(self.cmp(comps[name], *args), t)
        if name == "logical_not":
            return conv(self.cmp("eq", args[0], self.lit(0, args[0].t)), t)
        if name in ("logical_and", "logical_or"):
            return conv(self.binary("&&" if name == "logical_and" else "||", *args), t)
        if t in ("f16", "bf16"):
            return conv(self.op(name, [conv(a, "f32") for a in args], "f32"), t)
        args = [conv(a, t) for a in args]
        binary = {"add": "+", "subtract": "-", "multiply": "*", "divide": "/"}
        if name in binary:
            return self.binary(binary[name], *args, t=t)
        x = args[0].a
        f = np.float32
        with np.errstate(all="ignore"):
            if t == "s32":
                y = args[1].a.astype(np.int64) if len(args) > 1 else None
                x64 = x.astype(np.int64)
                safe = np.where(y == 0, 1, y) if y is not None else None
                table = {"maximum": lambda: np.maximum(x64, y), "minimum": lambda: np.minimum(x64, y),
                         "negative": lambda: -x64, "abs": lambda: np.abs(x64), "relu": lambda: np.maximum(x64, 0),
                         "square": lambda: x64 * x64,
                         # floor division and a remainder with the divisor's sign (ptx_backend.py:996-1024)
                         "floor_divide": lambda: np.floor_divide(x64, safe),
                         "remainder": lambda: np.remainder(x64, safe), "mod": lambda: np.remainder(x64, safe),
                         "bitwise_and": lambda: x64 & y, "bitwise_or": lambda: x64 | y,
                         "bitwise_xor": lambda: x64 ^ y, "bitwise_not": lambda: ~x64}
                return V((table[name]() % (1 << 32)).astype(np.uint32).view(np.int32), t)
            x64 = x.astype(np.float64)
            one = {
                "negative": lambda: -x, "abs": lambda: np.abs(x),
                "maximum": lambda: np.fmax(x, args[1].a), "minimum": lambda: np.fmin(x, args[1].a),
                "sqrt": lambda: np.sqrt(x), "square": lambda: x * x, "reciprocal": lambda: f(1) / x,
                "rsqrt": lambda: f(1) / np.sqrt(x), "floor": lambda: np.floor(x), "ceil": lambda: np.ceil(x),
                "trunc": lambda: np.trunc(x), "rint": lambda: np.rint(x), "relu": lambda: np.fmax(x, f(0)),
                "exp": lambda: np.exp(x64), "exp2": lambda: np.exp2(x64), "log": lambda: np.log(x64),
                "log2": lambda: np.log2(x64), "log10": lambda: np.log10(x64), "sin": lambda: np.sin(x64),
                "cos": lambda: np.cos(x64), "tanh": lambda: np.tanh(x64),
                "erf": lambda: np.asarray([math.erf(v) for v in x64]),
                "sigmoid": lambda: 1.0 / (1.0 + np.exp(-x64)), "silu": lambda: x64 / (1.0 + np.exp(-x64)),
                "fma": lambda: x64 * args[1].a.astype(np.float64) + args[2].a.astype(np.float64),
            }
            if name in ("mod", "remainder"):
                y = args[1].a
                r = np.fmod(x, y)                                   # exact, sign of x
                adjust = (r != 0) & ((x < 0) != (y < 0))
                r = np.where(adjust, (r + y).astype(np.float32), r)
                r = np.where(r == 0, np.copysign(np.float32(0), y), r)
                r = np.where(~np.isfinite(x) | np.isnan(y) | (y == 0), np.float32(np.nan), r)
                return V(r.astype(np.float32), "f32")
            if name in one:
                return V(np.asarray(one[name]()).astype(np.float32), "f32")
            if name in ("gelu", "gelu_tanh"):
                from oracle.expressions import gelu
                return V(gelu(x, "none" if name == "gelu" else "tanh", "f32").reshape(x.shape), "f32")
        raise ValueError(f"oracle: no pointwise operation {name}")

    # -------------------------------------------------------- statements
    def index(self, e):
        if isinstance(e, int):
            return np.int64(e)
        k = e.kind
        if k == "Literal":
            return np.int64(e.value)
        if k == "Var":
            return self.coord[e.name]
        if k == "BinaryExpr":
            a, b = self.index(e.left), self.index(e.right)
            if e.op in ("/", "//", "%"):   # C integer division and remainder, truncating toward zero
                q = np.trunc(np.asarray(a, np.float64) / np.asarray(b, np.float64)).astype(np.int64)
                return q if e.op != "%" else a - b * q
            return {"+": a + b, "-": a - b, "*": a * b}[e.op]
        raise ValueError(f"oracle: index {e!r}")

    def flat(self, buf, index):
        shape = tuple(self.pkg.buffers[buf].shape) or (1,)
        idx = [self.index(i) for i in index]
        if len(idx) == 1 or len(idx) != len(shape):
            return sum(idx)
        return sum(i * math.prod(shape[d + 1:]) for d, i in enumerate(idx))

    def expr(self, e) -> V:
        if isinstance(e, bool):
            return self.lit(e, "pred")
        if isinstance(e, int):
            return self.lit(e, "s32")
        if isinstance(e, float):
            return self.lit(e, "f32")
        if isinstance(e, str):
            return self.env[e]
        k = e.kind
        if k == "Var":
            if e.name not in self.env and e.name in self.coord:
                # a tile coordinate or loop counter as a value: s32
                return V(np.asarray(self.coord[e.name]).astype(np.int32), "s32")
            return self.env[e.name]
        if k == "Literal":
            dt = e.get("dtype")
            return self.lit(e.value, _t(dt) if dt else ("f32" if isinstance(e.value, float) else "s32"))
        if k == "BinaryExpr":
            return self.binary(e.op, self.expr(e.left), self.expr(e.right))
        if k == "CastExpr":
            return conv(self.expr(e.get("expr", e.get("value"))), _t(e.dtype))
        if k == "FuncCallExpr":
            args = [self.expr(a) for a in e.args]
            return self.op(e.name, args, args[0].t)
        if k == "TernaryExpr":
            c = conv(self.expr(e.cond), "pred").a
            a, b = self.expr(e.if_true), self.expr(e.if_false)
            t = common(a.t, b.t)
            return V(np.where(c, conv(a, t).a, conv(b, t).a), t)
        raise ValueError(f"oracle: expression {k}")

    def run(self, body) -> dict:
        for s in body:
            k = s.kind
            if k == "Load":
                buf = self.pkg.buffers[s.input]
                t = _t(buf.dtype)
                data = self.arrays[s.input]
                for lane, name in enumerate(s.names):
                    vals = data[self.flat(s.input, s.index) + lane]
                    if t == "s32":
                        vals = np.asarray(vals).astype(np.int64).astype(np.uint32).view(np.int32) \
                            if np.asarray(vals).dtype != np.int32 else vals
                    else:
                        vals = np.asarray(vals, np.float32)
                    self.env[name] = V(vals, t)
            elif k == "Let":
                v = self.expr(s.value)
                self.env[s.name] = conv(v, _t(s.dtype) if s.get("dtype") else v.t)
            elif k == "Assign":
                opname = s.op.name if hasattr(s.op, "kind") else str(s.op)
                args = [self.env[a] if isinstance(a, str) else self.expr(a) for a in s.args]
                dt = s.get("dtype")
                t = _t(dt) if dt is not None else (args[0].t if all(a.t == args[0].t for a in args) else "f32")
                self.env[s.name] = self.op(opname, args, t)
            elif k == "Select":
                branches = list(s.branches)
                value = conv(self.env[branches[-1].value], "f32").a
                for br in reversed(branches[:-1]):
                    c = conv(self.expr(br.select), "pred").a
                    value = np.where(c, conv(self.env[br.value], "f32").a, value)
                self.env[s.name] = V(value, "f32")
            elif k == "Write":
                buf = self.pkg.buffers[s.output]
                t = _t(buf.dtype)
                out = self.out.setdefault(s.output, np.full(math.prod(buf.shape or (1,)), np.nan
                                                           if t != "s32" else -1,
                                                           np.float32 if t != "s32" else np.int32))
                for lane, name in enumerate(s.values):
                    vals = conv(self.env[name], t).a
                    out[np.broadcast_to(self.flat(s.output, s.index) + lane, vals.shape)] = vals
            else:
                raise ValueError(f"oracle: statement {k}")
        return {k: v.reshape(tuple(self.pkg.buffers[k].shape) or (1,)) for k, v in self.out.items()}


def evaluate(ir_path, arrays: dict) -> dict:
    """Outputs of the pointwise package at ``ir_path`` on named input arrays."""
    from lazy_compiler_b200.ir import load_package
    pkg = load_package(ir_path)
    (tile,) = pkg.body
    return PointwiseOracle(pkg, tile, arrays).run(tile.body)
