"""Operation-class recogniser: Emmy Kernel IR -> a launch plan for a B200 kernel.

The reference lowers every IR statement to PTX text one by one
(ptx_backend.py:1375-1456 ``statement``).  This backend instead has one
hand-written sm_100a kernel per operation class, so the IR is evaluated
symbolically once and the resulting dataflow is matched against the classes
the reference's public problems and generated examples exercise:

=============  ====================================================  =====================
op             IR signature (reference file)                          C-ABI entry point
=============  ====================================================  =====================
add_f32        Tile; Load x0[i], x1[i]; add; Write (p00/p01)         lc_add_f32
axpb_f32       Tile; multiply(c_mul, x); add(c_add, .) (p02)          lc_axpb_f32
relumul_f32    Tile; relu(x) * y (p03)                                lc_relumul_f32
gelu           erf or tanh GELU chain, decomposed (phase9_gelu_*) or  lc_gelu
               the direct ``gelu``/``gelu_tanh`` op; f32/f16/bf16
sum_f32        Tile[co]; StridedLoop(Load; Accum add); WarpShuffle;   lc_sum_f32
               TreeHalve; Cond co==0 Write (r01/r02)
mean_f32       sum + divide(acc, count[0]) (r03)                      lc_mean_f32
rowsum_f32     Tile[row, co]; same loop over columns (r04)            lc_rowsum_f32
l2norm_f32     sum of squares; x * recip(sqrt(acc)) (f03)             lc_l2norm_f32
rmsnorm_f32    x * recip(sqrt(eps + acc*recip(count))) * w (f01)      lc_rmsnorm_f32
softmax_f32    online (max, sum) pass; exp(x-max)*recip(sum) (f02)   lc_softmax_f32
gemm           RegFragment/LdmatrixLoad/MmaSyncPtx/RegStore with an  lc_gemm
               optional erf/tanh GELU epilogue (generated_tensor,
               phase9_half_gelu_gemm, tensor/packages/*)
=============  ====================================================  =====================

An IR that matches none of them is rejected with :class:`CompileError`, the
same fail-closed behaviour as the reference (ptx_backend.py:1371-1372).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

from .ir import CompileError, KernelPackage, Node, dtype_name, static_extent

PLAN_FORMAT = "lazyb200-plan/1"

# ----------------------------------------------------------------------------
# Symbolic expressions: nested tuples.
#   ("ld", buffer, index)      index: tuple of affine forms
#   ("lit", value)
#   ("op", name, arg, ...)     elementwise op named as in Emmy's ElementwiseImpl
#   ("red", acc)               completed block/row reduction of an accumulator
#   ("cast", dtype, expr)      a typed Let/Assign narrowing (f16/bf16)
# Affine forms are frozensets of (term, coefficient) where term is an axis name,
# 1 (the constant) or a ("div"|"mod", affine, divisor) tuple.
# ----------------------------------------------------------------------------

_COMMUTATIVE = {"add", "multiply", "maximum", "minimum"}
_BINOPS = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide"}


def _aff(d: dict) -> frozenset:
    return frozenset((k, v) for k, v in d.items() if v != 0)


def _aff_add(a: frozenset, b: frozenset, sign: int = 1) -> frozenset:
    d = dict(a)
    for k, v in b:
        d[k] = d.get(k, 0) + sign * v
    return _simplify(d)


def _aff_scale(a: frozenset, c: int) -> frozenset:
    return _aff({k: v * c for k, v in a})


def _simplify(d: dict) -> frozenset:
    # c * (X // c) + (X % c) == X  for the row-major flattening of div/mod pairs
    changed = True
    while changed:
        changed = False
        for term, coef in list(d.items()):
            if isinstance(term, tuple) and term[0] == "mod" and coef != 0:
                inner, divisor = term[1], term[2]
                div = ("div", inner, divisor)
                if d.get(div, 0) == coef * divisor:
                    d[div] = 0
                    d[term] = 0
                    for k, v in inner:
                        d[k] = d.get(k, 0) + coef * v
                    changed = True
                    break
    return _aff(d)


def _aff_const(a: frozenset) -> int | None:
    terms = dict(a)
    if all(k == 1 for k in terms):
        return terms.get(1, 0)
    return None


def _is_lit(node: Any) -> bool:
    return isinstance(node, Node) and node.kind == "Literal"


class _Eval:
    """Symbolic evaluation of one Tile body."""

    def __init__(self, pkg: KernelPackage):
        self.pkg = pkg
        self.env: dict[str, Any] = {}
        self.axes: dict[str, int] = {}
        self.loops: list[dict] = []          # loops in program order
        self.reductions: dict[str, dict] = {}
        self.shuffled: set[str] = set()
        self.trees: set[str] = set()
        self.writes: list[dict] = []
        self.cond_stack: list[Any] = []
        self.loop_stack: list[dict] = []
        self.tree_length: int | None = None
        self.shuffle_length: int | None = None

    # -- index arithmetic ----------------------------------------------------
    def index(self, node: Any) -> frozenset:
        if isinstance(node, Node):
            if node.kind == "Literal":
                if not isinstance(node.value, int):
                    raise CompileError("non-integer index literal")
                return _aff({1: node.value})
            if node.kind == "Var":
                return _aff({node.name: 1})
            if node.kind == "BinaryExpr":
                left, right = self.index(node.left), self.index(node.right)
                if node.op == "+":
                    return _aff_add(left, right)
                if node.op == "-":
                    return _aff_add(left, right, -1)
                if node.op == "*":
                    cl, cr = _aff_const(left), _aff_const(right)
                    if cr is not None:
                        return _aff_scale(left, cr)
                    if cl is not None:
                        return _aff_scale(right, cl)
                    raise CompileError("non-affine index product")
                if node.op in ("//", "/", "%"):
                    c = _aff_const(right)
                    if c is None or c <= 0:
                        raise CompileError("index division by a non-constant")
                    cl = _aff_const(left)
                    if cl is not None:
                        return _aff({1: cl // c if node.op != "%" else cl % c})
                    kind = "mod" if node.op == "%" else "div"
                    return _aff({(kind, left, c): 1})
        raise CompileError(f"unsupported index expression {node!r}")

    # -- value expressions ---------------------------------------------------
    def value(self, node: Any) -> Any:
        if isinstance(node, str):
            if node not in self.env:
                raise CompileError(f"use of undefined value {node}")
            return self.env[node]
        if isinstance(node, Node):
            if node.kind == "Literal":
                return ("lit", float(node.value))
            if node.kind == "Var":
                if node.name in self.env:
                    return self.env[node.name]
                raise CompileError(f"use of undefined value {node.name}")
            if node.kind == "FuncCallExpr":
                return ("op", node.name, *(self.value(a) for a in node.args))
            if node.kind == "BinaryExpr" and node.op in _BINOPS:
                return ("op", _BINOPS[node.op], self.value(node.left), self.value(node.right))
            if node.kind == "CastExpr":
                return ("cast", dtype_name(node.get("dtype")), self.value(node.get("value")))
        raise CompileError(f"unsupported value expression {node!r}")

    def typed(self, expr: Any, dtype: Any) -> Any:
        name = dtype_name(dtype)
        if name in ("f16", "bf16"):
            return ("cast", name, expr)
        return expr

    # -- statements ----------------------------------------------------------
    def run(self, stmts: tuple) -> None:
        for stmt in stmts:
            self.stmt(stmt)

    def stmt(self, s: Node) -> None:
        k = s.kind
        if k == "Load":
            buf = self.pkg.buffers.get(s.input)
            if buf is None and s.input not in self.smem:
                raise CompileError(f"Load from unknown buffer {s.input}")
            index = tuple(self.index(i) for i in s.index)
            if len(s.names) > 1 and not index:
                raise CompileError("vector Load of a scalar")
            for lane, name in enumerate(s.names):
                # a vector load reads consecutive elements along the last dimension
                lane_index = index if lane == 0 else index[:-1] + (_aff_add(index[-1], _aff({1: lane})),)
                self.env[name] = ("ld", s.input, lane_index)
        elif k == "Assign":
            op = s.op.name if isinstance(s.op, Node) else str(s.op)
            args = tuple(self.value(a) for a in s.args)
            self.env[s.name] = self.typed(("op", op, *args), s.get("dtype"))
        elif k == "Let":
            self.env[s.name] = self.typed(self.value(s.value), s.get("dtype"))
        elif k == "Init":
            self.env[s.name] = ("init", s.name)
        elif k == "Accum":
            if not self.loop_stack:
                raise CompileError("Accum outside a loop")
            loop = self.loop_stack[-1]
            op = s.op.name if isinstance(s.op, Node) else str(s.op)
            value = self.value(s.value)
            base = s.get("base")
            if base is not None:
                # coupled online state: acc <- op(base, value) with an explicit base
                value = ("op", op, self.value(base), value)
            self.reductions[s.name] = {
                "op": op, "value": value, "loop": loop["axis"], "base": base,
            }
            loop["accums"].append(s.name)
            self.env[s.name] = ("acc", s.name)
        elif k in ("StridedLoop", "Loop"):
            self.loop(s)
        elif k == "Cond":
            self.cond_stack.append(s.cond)
            self.run(s.body)
            self.cond_stack.pop()
            if s.get("else_body"):
                raise CompileError("Cond else-branches are not supported by the recogniser")
        elif k == "Write":
            if self.pkg.buffers.get(s.output) is None:
                # shared-memory staging of partials (reduction epilogue), not a result
                if s.output not in self.smem:
                    raise CompileError(f"Write to unknown buffer {s.output}")
                return
            self.writes.append({
                "buffer": s.output,
                "index": tuple(self.index(i) for i in s.index),
                "values": tuple(self.value(v) for v in s.values),
                "dtype": dtype_name(s.get("value_dtype")),
                "atomic": bool(s.get("atomic")),
                "loop": self.loop_stack[-1]["axis"] if self.loop_stack else None,
                "cond": tuple(self.cond_stack),
            })
        elif k == "WarpShuffle":
            self.shuffled.update(s.state)
            self.shuffle_length = s.length
            for name in s.state:
                self.env[name] = ("red", name)
        elif k == "TreeHalve":
            self.trees.update(s.state)
            self.tree_length = s.length
            for name in s.state:
                self.env[name] = ("red", name)
        elif k == "Smem":
            self.smem.add(s.name)
        elif k == "Sync":
            pass
        else:
            raise CompileError(f"{k}: not part of a recognised operation class")

    smem: set

    def loop(self, s: Node) -> None:
        axis = s.axis
        name = axis.name
        extent = static_extent(axis.extent)
        start = s.get("start")
        step = s.get("step")
        info = {
            "axis": name, "extent": extent, "accums": [],
            "start": self.index(start) if start is not None else _aff({}),
            "step": _aff_const(self.index(step)) if step is not None else 1,
            "parent": self.loop_stack[-1]["axis"] if self.loop_stack else None,
        }
        if s.get("end") is not None:
            info["end"] = s.end
        self.loops.append(info)
        self.loop_stack.append(info)
        self.axes[name] = extent
        # accumulators are live (seeded with their identity) across the whole loop body
        for inner in s.body:
            if isinstance(inner, Node) and inner.kind == "Accum":
                self.env[inner.name] = ("acc", inner.name)
        self.run(s.body)
        self.loop_stack.pop()


# ----------------------------------------------------------------------------
# pattern matching with commutative operands and placeholder binding
# ----------------------------------------------------------------------------

def _match(pattern: Any, expr: Any, binds: dict) -> dict | None:
    if isinstance(pattern, tuple) and pattern and pattern[0] == "?":
        key = pattern[1]
        pred = pattern[2] if len(pattern) > 2 else None
        if pred is not None and not pred(expr):
            return None
        if key in binds:
            return binds if binds[key] == expr else None
        out = dict(binds)
        out[key] = expr
        return out
    if isinstance(pattern, tuple) and isinstance(expr, tuple):
        if len(pattern) != len(expr):
            return None
        if pattern[0] == "op" and expr[0] == "op" and pattern[1] == expr[1] \
                and pattern[1] in _COMMUTATIVE and len(pattern) == 4:
            for order in ((2, 3), (3, 2)):
                b = _match(pattern[order[0]], expr[2], binds)
                if b is not None:
                    b = _match(pattern[order[1]], expr[3], b)
                    if b is not None:
                        return b
            return None
        b = binds
        for p, e in zip(pattern, expr):
            b = _match(p, e, b)
            if b is None:
                return None
        return b
    return binds if pattern == expr else None


def V(key: str, pred=None) -> tuple:
    return ("?", key) if pred is None else ("?", key, pred)


def op(name: str, *args) -> tuple:
    return ("op", name, *args)


def _strip_casts(expr: Any) -> tuple[Any, set]:
    """Remove ("cast", dt, e) wrappers, returning the plain expression and the dtypes seen."""
    seen: set = set()

    def walk(e):
        if isinstance(e, tuple) and e and e[0] == "cast":
            seen.add(e[1])
            return walk(e[2])
        if isinstance(e, tuple) and e and e[0] == "op":
            return (e[0], e[1], *(walk(a) for a in e[2:]))
        return e

    return walk(expr), seen


# ----------------------------------------------------------------------------
# plans
# ----------------------------------------------------------------------------

@dataclass
class Plan:
    op: str
    abi: str
    entry: str
    bind: dict            # C-ABI parameter role -> meta.json argument name
    params: dict          # shape and mode parameters
    dtypes: dict
    arg_order: list
    launch_meta: dict     # the reference geometry, recorded (not used: kernels size their own grid)
    zero_outputs: list = field(default_factory=list)

    def to_json(self) -> dict:
        return {
            "format": PLAN_FORMAT, "entry": self.entry, "op": self.op, "abi": self.abi,
            "bind": self.bind, "params": self.params, "dtypes": self.dtypes,
            "arg_order": self.arg_order, "zero_outputs": self.zero_outputs,
            "reference_launch": self.launch_meta,
        }


def _numel(shape) -> int:
    return int(math.prod(shape)) if shape else 1


def _scalar_buffer(pkg: KernelPackage, name: str) -> bool:
    buf = pkg.buffers.get(name)
    return buf is not None and _numel(buf.shape) == 1


def _scalar_value(pkg: KernelPackage, name: str) -> float | None:
    """Value of a one-element constant argument from meta ``data`` or the ConstantOp."""
    for arg in pkg.kernel_meta.get("args", []):
        if arg.get("name") == name and "data" in arg:
            data = arg["data"]
            if isinstance(data, list) and len(data) == 1:
                return float(data[0])
    buf = pkg.buffers.get(name)
    if buf is not None and buf.constant is not None and isinstance(buf.constant, (int, float)):
        return float(buf.constant)
    return None


def _launch_meta(pkg: KernelPackage) -> dict:
    km = pkg.kernel_meta
    return {"grid": km.get("grid"), "block": km.get("block"), "smem_bytes": km.get("smem_bytes", 0)}


def _plan(pkg, op_, abi, bind, params, dtypes) -> Plan:
    return Plan(op=op_, abi=abi, entry=pkg.entry, bind=bind, params=params, dtypes=dtypes,
                arg_order=list(pkg.arg_order), launch_meta=_launch_meta(pkg),
                zero_outputs=list(pkg.kernel_meta.get("zero_outputs", [])))


# ----------------------------------------------------------------------------
# pointwise
# ----------------------------------------------------------------------------

def _flat(pkg: KernelPackage, buffer: str, index: tuple) -> frozenset:
    shape = pkg.buffers[buffer].shape or (1,)
    if len(index) == 0:
        return _aff({})
    if len(index) != len(shape):
        raise CompileError(f"index rank {len(index)} does not match {buffer}{list(shape)}")
    total = _aff({})
    stride = 1
    for dim, idx in zip(reversed(shape), reversed(index)):
        total = _aff_add(total, _aff_scale(idx, stride))
        stride *= dim
    return total


def _canon_pointwise(pkg, expr, flat):
    """Replace element loads at the written position by ("in", buf) and scalar loads by ("s", buf)."""
    if isinstance(expr, tuple) and expr and expr[0] == "ld":
        buf = expr[1]
        if _scalar_buffer(pkg, buf) and all(_aff_const(i) == 0 for i in expr[2]):
            return ("s", buf)
        if _flat(pkg, buf, expr[2]) != flat:
            raise CompileError(f"load of {buf} is not at the written element")
        return ("in", buf)
    if isinstance(expr, tuple) and expr and expr[0] in ("op", "cast"):
        head = expr[:2]
        return (*head, *(_canon_pointwise(pkg, a, flat) for a in expr[2:]))
    if isinstance(expr, tuple) and expr and expr[0] == "lit":
        return expr
    raise CompileError(f"unsupported pointwise operand {expr!r}")


def _isin(e):
    return isinstance(e, tuple) and e[0] == "in"


def _iss(e):
    return isinstance(e, tuple) and e[0] in ("s", "lit")


def _scalar_of(pkg, e) -> float | None:
    if e[0] == "lit":
        return e[1]
    return _scalar_value(pkg, e[1])


_GELU_ERF = op("multiply", op("add", V("one", _iss), op("erf", op("multiply", V("r2", _iss), V("x", _isin)))),
               op("multiply", V("half", _iss), V("x")))
_GELU_ERF_B = op("multiply", op("multiply", op("add", V("one", _iss), op("erf", op("multiply", V("r2", _iss), V("x", _isin)))),
                                V("half", _iss)), V("x"))
_GELU_TANH = op("multiply", op("multiply", V("half", _iss), V("x", _isin)),
                op("add", V("one", _iss), op("tanh", op("multiply", V("c0", _iss), op(
                    "add", V("x"), op("multiply", V("c1", _iss), op("multiply", V("x"), op("multiply", V("x"), V("x")))))))))


# the same chains around an arbitrary operand (activation epilogues)
_GELU_ERF_ANY = op("multiply", op("add", V("one", _iss), op("erf", op("multiply", V("r2", _iss), V("x")))),
                   op("multiply", V("half", _iss), V("x")))
_GELU_ERF_B_ANY = op("multiply", op("multiply", op("add", V("one", _iss), op("erf", op("multiply", V("r2", _iss), V("x")))),
                                    V("half", _iss)), V("x"))
_GELU_TANH_ANY = op("multiply", op("multiply", V("half", _iss), V("x")),
                    op("add", V("one", _iss), op("tanh", op("multiply", V("c0", _iss), op(
                        "add", V("x"), op("multiply", V("c1", _iss), op("multiply", V("x"), op("multiply", V("x"), V("x")))))))))


def _pointwise_class(pkg: KernelPackage, expr: Any) -> tuple[str, dict, dict]:
    plain, casts = _strip_casts(expr)
    if (b := _match(op("add", V("a", _isin), V("b", _isin)), plain, {})) and not casts:
        return "add_f32", {"x0": b["a"][1], "x1": b["b"][1]}, {}
    if (b := _match(op("add", V("b", _iss), op("multiply", V("a", _iss), V("x", _isin))), plain, {})) and not casts:
        if b["a"][0] != "s" or b["b"][0] != "s":
            raise CompileError("scale-shift constants must be kernel arguments")
        return "axpb_f32", {"a": b["a"][1], "b": b["b"][1], "x": b["x"][1]}, {}
    if (b := _match(op("multiply", V("y", _isin), op("relu", V("x", _isin))), plain, {})) and not casts:
        return "relumul_f32", {"x": b["x"][1], "y": b["y"][1]}, {}
    if (b := _match(op("gelu", V("x", _isin)), plain, {})):
        return "gelu", {"x": b["x"][1]}, {"approximate": "none"}
    if (b := _match(op("gelu_tanh", V("x", _isin)), plain, {})):
        return "gelu", {"x": b["x"][1]}, {"approximate": "tanh"}
    for pattern in (_GELU_ERF, _GELU_ERF_B):
        if (b := _match(pattern, plain, {})):
            consts = {k: _scalar_of(pkg, b[k]) for k in ("one", "r2", "half")}
            want = {"one": 1.0, "r2": math.sqrt(0.5), "half": 0.5}
            _check_consts(consts, want)
            return "gelu", {"x": b["x"][1]}, {"approximate": "none"}
    if (b := _match(_GELU_TANH, plain, {})):
        consts = {k: _scalar_of(pkg, b[k]) for k in ("one", "c0", "c1", "half")}
        want = {"one": 1.0, "c0": math.sqrt(2.0 / math.pi), "c1": 0.044715, "half": 0.5}
        _check_consts(consts, want)
        return "gelu", {"x": b["x"][1]}, {"approximate": "tanh"}
    raise CompileError("pointwise body does not match a supported operation class")


def _check_consts(got: dict, want: dict) -> None:
    for key, value in want.items():
        g = got.get(key)
        if g is None:
            raise CompileError(f"GELU constant {key} has no static value in meta.json")
        if not math.isclose(g, value, rel_tol=1e-3):
            raise CompileError(f"GELU constant {key}={g} differs from {value}")


def _recognise_pointwise(pkg: KernelPackage, tile: Node, ev: _Eval) -> Plan:
    axes = [a.name for a in tile.axes]
    if len(axes) != 1:
        raise CompileError("pointwise Tile must have one axis")
    cells = static_extent(tile.axes[0].extent)
    if not ev.writes:
        raise CompileError("pointwise body writes nothing")
    out = ev.writes[0]["buffer"]
    if any(w["buffer"] != out or w["atomic"] or w["cond"] for w in ev.writes):
        raise CompileError("pointwise body must write one buffer unconditionally")
    signatures = set()
    offsets = []
    cell = _aff({axes[0]: 1})
    for w in ev.writes:
        flat0 = _flat(pkg, out, w["index"])
        for j, v in enumerate(w["values"]):
            flat = _aff_add(flat0, _aff({1: j}))
            signatures.add(_canon_pointwise(pkg, v, flat))
            # element offset relative to (unroll * cell)
            d = dict(flat)
            offsets.append((d.get(axes[0], 0), d.get(1, 0), frozenset(k for k in d if k not in (axes[0], 1))))
    if len(signatures) != 1:
        raise CompileError("unrolled pointwise elements compute different expressions")
    unroll = len(offsets)
    if any(extra for _, _, extra in offsets):
        raise CompileError("pointwise write index is not affine in the tile axis")
    if sorted((c, o) for c, o, _ in offsets) != [(unroll, j) for j in range(unroll)]:
        raise CompileError("pointwise writes do not cover the tile densely")
    n = _numel(pkg.buffers[out].shape)
    if cells * unroll != n:
        raise CompileError(f"tile covers {cells * unroll} elements of {out} ({n})")
    expr = signatures.pop()
    op_, bind, extra = _pointwise_class(pkg, expr)
    bind["out"] = out
    in_dtypes = {pkg.buffers[bind[k]].dtype for k in bind if k not in ("out", "a", "b")}
    dtype = pkg.buffers[out].dtype
    if op_ == "gelu":
        if in_dtypes != {dtype} or dtype not in ("f32", "f16", "bf16"):
            raise CompileError(f"GELU over {in_dtypes} -> {dtype} is not supported")
        return _plan(pkg, "gelu", "lc_gelu", bind, {"n": n, **extra}, {"io": dtype})
    if dtype != "f32" or in_dtypes - {"f32"}:
        raise CompileError(f"{op_} requires f32 buffers")
    return _plan(pkg, op_, "lc_" + op_, bind, {"n": n}, {"io": "f32"})


# ----------------------------------------------------------------------------
# reductions and row operations
# ----------------------------------------------------------------------------

def _is_load(buf=None, index=None):
    def pred(e):
        return isinstance(e, tuple) and e[0] == "ld" and (buf is None or e[1] == buf) and \
            (index is None or e[2] == index)
    return pred


def _rowdot_terms(pkg: KernelPackage, value: Any, x_index: tuple):
    """y[r,c] * f(x[r,c]) with f the identity or a GELU -> (x, y, activation), else None."""
    from .recognize_f32 import strip_epilogue
    if not (isinstance(value, tuple) and value[:2] == ("op", "multiply") and len(value) == 4):
        return None
    at = _is_load(index=x_index)
    for ya, fx in ((value[2], value[3]), (value[3], value[2])):
        if not at(ya):
            continue
        act, inner = strip_epilogue(pkg, fx)
        if at(inner):
            return inner[1], ya[1], act
    return None


_COMMUTATIVE = ("add", "multiply", "maximum", "minimum")


def canon_expr(e):
    """An expression with copies dropped and commutative arguments ordered."""
    if isinstance(e, tuple) and e and e[0] == "op":
        if e[1] == "copy" and len(e) == 3:
            return canon_expr(e[2])
        args = [canon_expr(a) for a in e[2:]]
        if e[1] in _COMMUTATIVE and len(args) == 2:
            args = sorted(args, key=repr)
        return ("op", e[1], *args)
    return e


def combine_result(node: Node) -> dict | None:
    """Each state after one step of a WarpShuffle / TreeHalve combine, as an
    expression of ("self", state) and ("other", state)."""
    env: dict = {}
    for a, b in zip(node.state, node.state_b):
        env[a], env[b] = ("self", a), ("other", a)
    for st in node.get("combine_states") or ():
        if st.kind == "Assign":
            opn = st.op.name if isinstance(st.op, Node) else str(st.op)
            env[st.name] = ("op", opn, *(env.get(x, ("?", x)) if isinstance(x, str) else ("?",) for x in st.args))
        elif st.kind == "Let" and _is_lit(st.value):
            env[st.name] = ("lit", float(st.value.value))
        else:
            return None
    return {a: canon_expr(env[a]) for a in node.state}


def fold_combine(name: str, opn: str) -> tuple:
    return ("op", opn, ("self", name), ("other", name))


def online_combine(mx: str, states: list) -> dict:
    """The online-softmax merge: the larger max, and every state rescaled to it."""
    gn = ("op", "maximum", ("self", mx), ("other", mx))
    out = {mx: gn}
    for s in states:
        out[s] = ("op", "add", ("op", "multiply", ("op", "exp", ("op", "subtract", ("self", mx), gn)), ("self", s)),
                  ("op", "multiply", ("op", "exp", ("op", "subtract", ("other", mx), gn)), ("other", s)))
    return out


def combines_are(tile: Node, expected: dict) -> bool:
    """Every WarpShuffle / TreeHalve of the Tile combines the given states as expected."""
    seen = set()
    for node in _walk(tile.body):
        if not isinstance(node, Node) or node.kind not in ("WarpShuffle", "TreeHalve"):
            continue
        result = combine_result(node)
        if result is None:
            return False
        for name in node.state:
            seen.add(name)
            if name not in expected or result[name] != canon_expr(expected[name]):
                return False
    return seen >= set(expected)


def _recognise_reduction(pkg: KernelPackage, tile: Node, ev: _Eval) -> Plan:
    axes = [(a.name, static_extent(a.extent)) for a in tile.axes]
    block = tile.get("block_threads") or axes[-1][1]
    co_name, co_extent = axes[-1]
    if co_extent != block:
        raise CompileError("cooperative axis must span the block")
    if ev.shuffle_length != 32 or ev.tree_length is None or ev.tree_length * 32 != block:
        raise CompileError("reduction must combine a full warp butterfly and a block tree")
    accums = [name for loop in ev.loops for name in loop["accums"]]
    if not accums or set(accums) - ev.trees:
        raise CompileError("every accumulator must be block-reduced")
    first = ev.loops[0]
    if first["start"] != _aff({co_name: 1}) or first["step"] != block:
        raise CompileError("reduction loop must stride the block across the axis")
    cols = first["extent"]
    two_d = len(axes) == 2
    if len(axes) > 2:
        raise CompileError("reductions over more than one row axis are not supported")
    row_name = axes[0][0] if two_d else None
    rows = axes[0][1] if two_d else 1
    col = first["axis"]
    x_index = (_aff({row_name: 1}), _aff({col: 1})) if two_d else (_aff({col: 1}),)

    reds = {name: ev.reductions[name] for name in accums}
    done_cond = ((_aff({co_name: 1}),),)

    def cond_ok(w):
        # the single writer of a reduced scalar guards on co == 0
        return len(w["cond"]) == 1 and w["cond"][0].kind == "BinaryExpr" and w["cond"][0].op == "==" \
            and w["cond"][0].left.kind == "Var" and w["cond"][0].left.name == co_name \
            and _is_lit(w["cond"][0].right) and w["cond"][0].right.value == 0
    del done_cond

    # --- sum / mean / rowsum: one accumulator of loads, one guarded scalar write
    if len(reds) == 1 and len(ev.loops) == 1:
        (acc, red), = reds.items()
        if red["op"] != "add" or red["base"] is not None:
            raise CompileError("unsupported accumulator")
        if not combines_are(tile, {acc: fold_combine(acc, "add")}):
            raise CompileError("the partial sums are not combined by addition")
        if len(ev.writes) != 1 or not cond_ok(ev.writes[0]):
            raise CompileError("reduction result must be written once by thread 0")
        w = ev.writes[0]
        value = w["values"][0]
        out = w["buffer"]
        square = _match(op("multiply", V("x", _is_load(index=x_index)), V("x")), red["value"], {})
        plain = _is_load(index=x_index)(red["value"])
        if two_d and not plain:
            dot = _rowdot_terms(pkg, red["value"], x_index)
            if dot is not None:
                xb, yb, act = dot
                if len(ev.writes) != 1 or not cond_ok(ev.writes[0]):
                    raise CompileError("row dot product must be written once by thread 0")
                w = ev.writes[0]
                if w["values"][0] != ("red", acc) or w["index"] != (_aff({row_name: 1}),):
                    raise CompileError("row dot product must write acc[row]")
                if _numel(pkg.buffers[w["buffer"]].shape) != rows:
                    raise CompileError("row dot output does not have one element per row")
                for b_ in (xb, yb, w["buffer"]):
                    if pkg.buffers[b_].dtype != "f32":
                        raise CompileError("row dot products are f32")
                for b_ in (xb, yb):
                    if pkg.buffers[b_].shape != (rows, cols):
                        raise CompileError("row dot operand shape does not match the loop extent")
                return _plan(pkg, "rowdot_f32", "lc_rowdot_f32", {"x": xb, "y": yb, "out": w["buffer"]},
                             {"rows": rows, "cols": cols, "activation": act}, {"io": "f32"})
        if not plain or square:
            raise CompileError("reduction accumulates an unsupported expression")
        x = red["value"][1]
        if pkg.buffers[x].dtype != "f32" or pkg.buffers[out].dtype != "f32":
            raise CompileError("reductions are f32")
        if pkg.buffers[x].shape != ((rows, cols) if two_d else (cols,)):
            raise CompileError("reduced buffer shape does not match the loop extent")
        if two_d:
            if value != ("red", acc) or w["index"] != (_aff({row_name: 1}),):
                raise CompileError("row reduction must write acc[row]")
            if _numel(pkg.buffers[out].shape) != rows:
                raise CompileError("row reduction output does not have one element per row")
            return _plan(pkg, "rowsum_f32", "lc_rowsum_f32", {"x": x, "out": out},
                         {"rows": rows, "cols": cols}, {"io": "f32"})
        if w["index"] not in ((), (_aff({}),)) or _numel(pkg.buffers[out].shape) != 1:
            raise CompileError("whole-array reduction writes a scalar")
        if value == ("red", acc):
            return _plan(pkg, "sum_f32", "lc_sum_f32", {"x": x, "out": out}, {"n": cols}, {"io": "f32"})
        b = _match(op("divide", ("red", acc), V("count", _is_load())), value, {})
        if b and _scalar_buffer(pkg, b["count"][1]):
            return _plan(pkg, "mean_f32", "lc_mean_f32", {"x": x, "count": b["count"][1], "out": out},
                         {"n": cols}, {"io": "f32"})
        raise CompileError("scalar reduction epilogue is not sum or mean")

    if not two_d:
        raise CompileError("fused row operations need a row axis")
    if any(w["loop"] is None for w in ev.writes) or len(ev.loops) != 2:
        raise CompileError("row operation must write in a second pass over the row")
    second = ev.loops[1]
    if second["start"] != _aff({co_name: 1}) or second["step"] != block or second["extent"] != cols:
        raise CompileError("second row pass must stride the block across the row")
    if len(ev.writes) != 1:
        raise CompileError("row operation must write one output")
    w = ev.writes[0]
    out = w["buffer"]
    col2 = second["axis"]
    if w["index"] != (_aff({row_name: 1}), _aff({col2: 1})):
        raise CompileError("row output must be written at [row, col]")
    x2 = (_aff({row_name: 1}), _aff({col2: 1}))
    value = w["values"][0]

    # --- softmax: coupled (max, sum) online state
    if len(reds) == 2:
        mx = [n for n, r in reds.items() if r["op"] == "maximum"]
        sm = [n for n, r in reds.items() if r["op"] == "add"]
        if len(mx) != 1 or len(sm) != 1:
            raise CompileError("two-accumulator row op is not an online softmax")
        mx, sm = mx[0], sm[0]
        if not _is_load(index=x_index)(reds[mx]["value"]):
            raise CompileError("softmax max must accumulate the row")
        x = reds[mx]["value"][1]
        pattern = op("multiply", op("reciprocal", ("red", sm)), op("exp", op("subtract", V("x", _is_load(x, x2)), ("red", mx))))
        if not _match(pattern, value, {}):
            raise CompileError("softmax output expression not recognised")
        # the running sum must rescale by exp(old - new) and add exp(x - new)
        xl = reds[mx]["value"]
        gn = ("op", "maximum", ("acc", mx), xl)
        online = ("op", "add", ("op", "multiply", ("acc", sm), ("op", "exp", ("op", "subtract", ("acc", mx), gn))),
                  ("op", "multiply", ("op", "exp", ("op", "subtract", xl, gn)), ("lit", 1.0)))
        if canon_expr(reds[sm]["value"]) != canon_expr(online):
            raise CompileError("softmax sum is not an online rescaled exponential sum")
        if not combines_are(tile, online_combine(mx, [sm])):
            raise CompileError("softmax partial states are not merged online")
        return _plan(pkg, "softmax_f32", "lc_softmax_f32", {"x": x, "out": out},
                     {"rows": rows, "cols": cols}, {"io": "f32"})

    (acc, red), = reds.items()
    b = _match(op("multiply", V("x", _is_load(index=x_index)), V("x")), red["value"], {})
    if red["op"] != "add" or not b:
        raise CompileError("row norm must accumulate a sum of squares")
    if red["base"] is not None or not combines_are(tile, {acc: fold_combine(acc, "add")}):
        raise CompileError("the partial sums of squares are not combined by addition")
    x = b["x"][1]
    # L2: x * recip(sqrt(acc))
    if _match(op("multiply", V("x", _is_load(x, x2)), op("reciprocal", op("sqrt", ("red", acc)))), value, {}):
        return _plan(pkg, "l2norm_f32", "lc_l2norm_f32", {"x": x, "out": out},
                     {"rows": rows, "cols": cols}, {"io": "f32"})
    # RMSNorm: w[col] * (x * recip(sqrt(eps + acc * recip(count))))
    w_index = (_aff({col2: 1}),)
    pattern = op("multiply", V("w", _is_load(index=w_index)), op("multiply", V("x", _is_load(x, x2)), op(
        "reciprocal", op("sqrt", op("add", V("eps", _is_load()), op("multiply", ("red", acc), op("reciprocal", V("count", _is_load()))))))))
    if (b := _match(pattern, value, {})):
        eps, count = b["eps"][1], b["count"][1]
        if not (_scalar_buffer(pkg, eps) and _scalar_buffer(pkg, count)):
            raise CompileError("RMSNorm eps and count must be one-element arguments")
        return _plan(pkg, "rmsnorm_f32", "lc_rmsnorm_f32",
                     {"count": count, "eps": eps, "x": x, "w": b["w"][1], "out": out},
                     {"rows": rows, "cols": cols}, {"io": "f32"})
    raise CompileError("row operation does not match L2 norm or RMSNorm")


# ----------------------------------------------------------------------------
# tensor-core GEMM
# ----------------------------------------------------------------------------

def _walk(stmts):
    for s in stmts:
        yield s
        if isinstance(s, Node):
            for key in ("body",):
                inner = s.get(key)
                if isinstance(inner, tuple):
                    yield from _walk(inner)


def _epilogue_kind(pkg: KernelPackage, lam: Node | None) -> str:
    if lam is None:
        return "none"
    ev = _Eval(pkg)
    ev.smem = set()
    (param,) = lam.params
    ev.env[param] = ("in", "__acc")
    for s in lam.body:
        if s.kind == "Load":
            if not _scalar_buffer(pkg, s.input):
                raise CompileError("GEMM epilogue may only load one-element constants")
            ev.env[s.names[0]] = ("s", s.input)
        else:
            ev.stmt(s)
    (result,) = lam.results
    expr, _ = _strip_casts(ev.env[result])
    if _match(op("copy", V("x")), expr, {}):
        expr = expr
    expr = _drop_copy(expr)
    if expr == ("in", "__acc"):
        return "none"
    for pattern in (_GELU_ERF, _GELU_ERF_B):
        if (b := _match(pattern, expr, {})):
            _check_consts({k: _scalar_of(pkg, b[k]) for k in ("one", "r2", "half")},
                          {"one": 1.0, "r2": math.sqrt(0.5), "half": 0.5})
            return "gelu_erf"
    if (b := _match(_GELU_TANH, expr, {})):
        _check_consts({k: _scalar_of(pkg, b[k]) for k in ("one", "c0", "c1", "half")},
                      {"one": 1.0, "c0": math.sqrt(2.0 / math.pi), "c1": 0.044715, "half": 0.5})
        return "gelu_tanh"
    raise CompileError("GEMM epilogue is not identity, erf-GELU or tanh-GELU")


def _drop_copy(e):
    if isinstance(e, tuple) and e and e[0] == "op":
        if e[1] == "copy" and len(e) == 3:
            return _drop_copy(e[2])
        return (*e[:2], *(_drop_copy(a) for a in e[2:]))
    return e


def _recognise_gemm(pkg: KernelPackage, tile: Node) -> Plan:
    stmts = list(_walk(tile.body))
    loads = [s for s in stmts if s.kind == "LdmatrixLoad"]
    mmas = [s for s in stmts if s.kind == "MmaSyncPtx"]
    stores = [s for s in stmts if s.kind == "RegStore"]
    allowed = {"RegFragment", "LdmatrixLoad", "MmaSyncPtx", "RegStore", "StridedLoop", "Loop",
               "Smem", "Sync", "CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait", "Load", "Write"}
    for s in stmts:
        if s.kind not in allowed:
            raise CompileError(f"{s.kind} inside a tensor-core tile is not supported")
    a_loads = {s.src_buffer for s in loads if s.role == "a"}
    b_loads = [s for s in loads if s.role == "b"]
    if not stores or not mmas:
        raise CompileError("tensor tile without MMA or store")
    if any(s.get("atomic") for s in stores):
        raise CompileError("atomic fragment stores are not supported")
    ab = {m.ab_dtype for m in mmas}
    if len(ab) != 1 or next(iter(ab)) not in ("f16", "bf16"):
        raise CompileError(f"MMA operand types {ab} not supported")
    ab = ab.pop()
    if any(m.c_dtype != "f32" for m in mmas):
        raise CompileError("MMA must accumulate in f32")
    staged = any(s.get("staged") for s in loads)
    if staged:
        # staged fixtures fill shared memory from global inside the tile; the
        # global operands are the sources of those copies
        raise CompileError("shared-memory staged tensor fixtures are not supported")
    if len(a_loads) != 1 or len({s.src_buffer for s in b_loads}) != 1:
        raise CompileError("GEMM must read one A and one B buffer")
    a = a_loads.pop()
    b = b_loads[0].src_buffer
    b_trans = {bool(s.b_trans) for s in b_loads}
    if len(b_trans) != 1:
        raise CompileError("mixed B layouts")
    b_trans = b_trans.pop()
    outs = {s.dst_buffer for s in stores}
    if len(outs) != 1:
        raise CompileError("GEMM must store one output")
    c = outs.pop()
    if any(s.get("row_dim", 0) != 0 or s.get("col_dim", 1) != 1 for s in stores):
        raise CompileError("transposed fragment stores are not supported")
    epilogues = {_epilogue_kind(pkg, s.get("epilogue")) for s in stores}
    if len(epilogues) != 1:
        raise CompileError("fragments use different epilogues")
    epi = epilogues.pop()
    sa, sb, sc = pkg.buffers[a].shape, pkg.buffers[b].shape, pkg.buffers[c].shape
    if len(sa) != 2 or len(sb) != 2 or len(sc) != 2:
        raise CompileError("GEMM operands must be matrices")
    m, k = sa
    n = sb[0] if b_trans else sb[1]
    kb = sb[1] if b_trans else sb[0]
    if kb != k or tuple(sc) != (m, n):
        raise CompileError(f"GEMM shapes {sa} x {sb} -> {sc} are inconsistent")
    if pkg.buffers[a].dtype != ab or pkg.buffers[b].dtype != ab:
        raise CompileError("GEMM operand buffers must match the MMA type")
    out_dtype = pkg.buffers[c].dtype
    if out_dtype not in ("f32", "f16", "bf16"):
        raise CompileError(f"GEMM output type {out_dtype} not supported")
    return _plan(pkg, "gemm", "lc_gemm", {"a": a, "b": b, "c": c},
                 {"m": m, "n": n, "k": k, "b_layout": "nk" if b_trans else "kn", "epilogue": epi},
                 {"ab": ab, "c": out_dtype})


# ----------------------------------------------------------------------------

_FRAGMENT_KINDS = {"RegFragment", "LdmatrixLoad", "MmaSyncPtx", "RegStore", "FragmentApply",
                   "FragmentRowReduce", "FragmentRepack"}


def _recognise_fragments(pkg: KernelPackage, tile: Node, kinds: set) -> Plan:
    """Tensor-fragment programs: a recognised product (tcgen05 GEMM, the
    fragment attention tile, a quantised GEMM or repack chain) when the
    program is one; otherwise, for one warp, the program itself as a lane
    program with the reference's per-lane semantics."""
    from . import fragment_vm, recognize_frag
    from . import recognize_f32 as f32
    single = recognize_frag.is_single_warp(pkg, tile)
    reason = None
    try:
        if "FragmentRowReduce" in kinds:
            return f32.recognise_fragment_attention(pkg, tile)
        if "MmaSyncPtx" in kinds:
            if single:
                return recognize_frag.recognise_fragment_tile(pkg, tile)
            return _recognise_gemm(pkg, tile)
        raise CompileError("fragment algebra without a recognised product")
    except CompileError as err:
        reason = err
    if not single:
        raise reason
    try:
        return fragment_vm.compile_fragment_lanes(pkg, tile)
    except CompileError as err:
        raise CompileError(f"{reason}; as a lane program: {err}") from err


def recognise(pkg: KernelPackage) -> Plan:
    """Map one loaded IR package to the launch plan of its B200 kernel."""
    if len(pkg.body) != 1 or pkg.body[0].kind != "Tile":
        raise CompileError("KernelOp body must be a single Tile")
    tile = pkg.body[0]
    kinds = {s.kind for s in _walk(tile.body)}
    from . import recognize_f32 as f32
    if kinds & _FRAGMENT_KINDS:
        return _recognise_fragments(pkg, tile, kinds)
    if "CpAsyncCopy" in kinds:
        try:
            return f32.recognise_staged_gemm(pkg, tile)
        except CompileError as err:
            return _block_program(pkg, tile, f"not a staged GEMM: {err}")
    ev = _Eval(pkg)
    ev.smem = set()
    for axis in tile.axes:
        ev.axes[axis.name] = static_extent(axis.extent)
    straight = not any(s.kind in ("StridedLoop", "Loop", "Cond") for s in _walk(tile.body))
    try:
        ev.run(tile.body)
    except CompileError as err:
        # the symbolic evaluation behind the fixed classes and row programs
        # does not take this body: the general per-point paths may
        if straight:
            return _pointwise_program(pkg, tile, err)
        return _serial_program(pkg, tile, str(err))
    if ev.loops and ev.reductions:
        # the fixed classes first, then the general row and serial programs
        try:
            if f32.looks_like_attention(ev):
                return f32.recognise_attention(pkg, tile, ev)
            if f32.looks_like_dot(ev):
                return f32.recognise_dot_gemm(pkg, tile, ev)
            return _recognise_reduction(pkg, tile, ev)
        except CompileError as err:
            from .rowprog import compile_rowprog
            try:
                return compile_rowprog(pkg, tile, ev)
            except CompileError as err2:
                return _serial_program(pkg, tile, f"{err}; as a row program: {err2}")
    if ev.loops:
        return _serial_program(pkg, tile, "loops without a reduction")
    try:
        return _recognise_pointwise(pkg, tile, ev)
    except CompileError as err:
        if straight:
            return _pointwise_program(pkg, tile, err)
        raise


def _serial_program(pkg: KernelPackage, tile: Node, reason: str) -> Plan:
    """A body with per-point runtime loops that no recogniser took: a serial
    program, or failing that a block program."""
    from .serial import compile_serial
    try:
        return compile_serial(pkg, tile)
    except CompileError as err:
        return _block_program(pkg, tile, f"{reason}; as a serial program: {err}")


def _block_program(pkg: KernelPackage, tile: Node, reason: str) -> Plan:
    """The last general path: the body run statement for statement, one CTA per block."""
    from .blockprog import compile_blockprog
    try:
        return compile_blockprog(pkg, tile)
    except CompileError as err:
        raise CompileError(f"{reason}; as a block program: {err}") from err


def _pointwise_program(pkg: KernelPackage, tile: Node, reason: CompileError) -> Plan:
    """A straight-line body outside the fixed pointwise classes: compile it to a register program."""
    from .pointwise import compile_pointwise
    try:
        return compile_pointwise(pkg, tile)
    except CompileError as err:
        return _block_program(pkg, tile, f"{err} (and not a fixed pointwise class: {reason})")
