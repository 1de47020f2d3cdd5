"""Recognition of the FP32 contraction classes: scalar GEMM and attention.

Emmy reaches these classes with three schedule forms, all handled here:

* serial — each thread walks the contraction for its own outputs, keeping the
  running state in registers (problems/a01_attention, a02_attention_128);
* block-cooperative — the block strides the contraction across its threads
  and merges the partial states with WarpShuffle / TreeHalve before thread 0
  writes (examples/phase9/generated/phase9_bias_gelu_gemm,
  phase9_gelu_attention);
* shared-memory staged — operand tiles are copied into ``Smem`` by cp.async
  (ptx_backend.py:1457-1492) and the inner products read them back; split-K
  variants add partial sums with atomic writes into launcher-zeroed outputs
  (problems/m01_matmul_512, m02_matmul_rect).

The first two are matched on the dataflow of the symbolic evaluation of
:mod:`.recognize`.  The staged form is evaluated by :class:`StagedEval`, which
unrolls the contraction loops with concrete loop values, records which global
element every shared-memory element was copied from (per dimension, the
copy's shared-memory index minus its global index may depend only on block
coordinates and loop values — the per-thread lane terms must cancel — and the
set of elements the block's threads copy is enumerated), resolves every
shared-memory load to the global element it reads, and keeps each
accumulator as its list of product terms.

Every form is then checked the same way: each written element is
``epilogue(sum_k A[row, k] * B[k, col] (+ bias[col]))`` (or the online-softmax
attention of one query row and value column) with the row and column of the
write, the contraction covers every k exactly once (across the split-K tiles
for atomic writes), and the writes of all threads cover the output exactly
once.  Anything else is a :class:`CompileError`.
"""
from __future__ import annotations

import itertools
import math
from typing import Any

import numpy as np

from .ir import CompileError, KernelPackage, Node, static_extent
from .dot2 import compensated_states
from .post import compile_epilogue
from .recognize import (_GELU_ERF_ANY, _GELU_ERF_B_ANY, _GELU_TANH_ANY, Plan, _aff, _aff_add, combines_are,
                        fold_combine, online_combine,
                        _aff_const, _Eval, _flat, _is_load, _match, _numel, _plan, _scalar_buffer,
                        _scalar_of, _check_consts, op, V)

# ----------------------------------------------------------------------------
# shared helpers
# ----------------------------------------------------------------------------


def aff_eval(form: frozenset, env: dict):
    """Value of an affine form under integer (or numpy array) bindings."""
    total = 0
    for term, coef in form:
        if term == 1:
            val = 1
        elif isinstance(term, str):
            if term not in env:
                raise CompileError(f"index depends on {term}, which is not bound here")
            val = env[term]
        else:
            kind, inner, c = term
            x = aff_eval(inner, env)
            val = x // c if kind == "div" else x % c
        total = total + coef * val
    return total


def aff_subst(form: frozenset, bind: dict) -> frozenset:
    """Substitute concrete values for some variables and fold what becomes constant."""
    d: dict = {}
    for term, coef in form:
        if isinstance(term, str) and term in bind:
            d[1] = d.get(1, 0) + coef * bind[term]
        elif isinstance(term, tuple):
            kind, inner, c = term
            inner2 = aff_subst(inner, bind)
            k = _aff_const(inner2)
            if k is not None:
                d[1] = d.get(1, 0) + coef * (k // c if kind == "div" else k % c)
            else:
                d[(kind, inner2, c)] = d.get((kind, inner2, c), 0) + coef
        else:
            d[term] = d.get(term, 0) + coef
    return _aff_add(_aff({}), _aff(d))


def check_cover(pkg: KernelPackage, axes: list, writes: list, out: str, fixed: dict | None = None,
                repeat: int = 1) -> None:
    """Every element of ``out`` is written exactly ``repeat`` times by the Tile's cells.

    ``axes`` are (name, extent) of the Tile; ``fixed`` pins axes (the
    cooperative axis of a block reduction writes from thread 0 only).
    """
    fixed = fixed or {}
    free = [(a, e) for a, e in axes if a not in fixed]
    size = math.prod(e for _, e in free)
    if size > (1 << 26):
        raise CompileError("Tile too large to check write coverage")
    grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for _, e in free], indexing="ij")
    env = {a: g.ravel() for (a, _), g in zip(free, grids)}
    env.update(fixed)
    n = _numel(pkg.buffers[out].shape)
    counts = np.zeros(n, np.int64)
    for w in writes:
        base = _flat(pkg, out, w["index"])
        for lane in range(len(w["values"])):
            flat = np.broadcast_to(np.asarray(aff_eval(_aff_add(base, _aff({1: lane})), env), np.int64),
                                   (size,))
            if flat.size and (flat.min() < 0 or flat.max() >= n):
                raise CompileError(f"a write of {out} falls outside the buffer")
            np.add.at(counts, flat, 1)
    if not (counts == repeat).all():
        raise CompileError(f"the writes do not cover {out} exactly once per element")


def canon_scalars(pkg: KernelPackage, e: Any) -> Any:
    """Loads of one-element arguments become ("s", buffer)."""
    if isinstance(e, tuple) and e and e[0] == "ld":
        if _scalar_buffer(pkg, e[1]) and all(_aff_const(i) == 0 for i in e[2]):
            return ("s", e[1])
        return e
    if isinstance(e, tuple) and e and e[0] in ("op", "cast"):
        return (*e[:2], *(canon_scalars(pkg, a) for a in e[2:]))
    return e


def _drop_copies(e):
    if isinstance(e, tuple) and e and e[0] == "op":
        if e[1] == "copy" and len(e) == 3:
            return _drop_copies(e[2])
        return (*e[:2], *(_drop_copies(a) for a in e[2:]))
    return e


def strip_epilogue(pkg: KernelPackage, expr: Any) -> tuple[str, Any]:
    """Split ``gelu(x)`` (decomposed or direct) into ("gelu_erf" | "gelu_tanh", x)."""
    expr = _drop_copies(canon_scalars(pkg, expr))
    if isinstance(expr, tuple) and expr[:2] == ("op", "gelu") and len(expr) == 3:
        return "gelu_erf", expr[2]
    if isinstance(expr, tuple) and expr[:2] == ("op", "gelu_tanh") and len(expr) == 3:
        return "gelu_tanh", expr[2]
    for pattern in (_GELU_ERF_ANY, _GELU_ERF_B_ANY):
        if (b := _match(pattern, expr, {})):
            _check_consts({k: _scalar_of(pkg, b[k]) for k in ("one", "r2", "half")},
                          {"one": 1.0, "r2": math.sqrt(0.5), "half": 0.5})
            return "gelu_erf", b["x"]
    if (b := _match(_GELU_TANH_ANY, expr, {})):
        _check_consts({k: _scalar_of(pkg, b[k]) for k in ("one", "c0", "c1", "half")},
                      {"one": 1.0, "c0": math.sqrt(2.0 / math.pi), "c1": 0.044715, "half": 0.5})
        return "gelu_tanh", b["x"]
    return "none", expr


def _is_state(e) -> bool:
    return isinstance(e, tuple) and len(e) == 2 and e[0] in ("acc", "red")


def _is_acc(e) -> bool:
    return isinstance(e, tuple) and len(e) == 2 and e[0] == "acc"


def _is_s(e) -> bool:
    return isinstance(e, tuple) and e[0] == "s"


def _var(name: str) -> frozenset:
    return _aff({name: 1})


def _f32(pkg: KernelPackage, *names: str) -> None:
    for n in names:
        if pkg.buffers[n].dtype != "f32":
            raise CompileError(f"{n} must be f32 for this operation class")


def _loop_info(ev: _Eval, axis: str) -> dict:
    for loop in ev.loops:
        if loop["axis"] == axis:
            return loop
    raise CompileError(f"no loop over {axis}")


def _contraction_form(tile: Node, ev: _Eval, loop: dict, extent: int, states: list[str],
                      writes: list, combine: dict) -> dict | None:
    """How a contraction loop covers [0, extent): serially, or strided over the block.

    Returns {} for the serial form, {co_axis: 0} (the pinned cooperative axis)
    for the block form; raises otherwise.
    """
    if loop["start"] == _aff({}) and loop["step"] == 1 and loop["extent"] == extent:
        if any(s in ev.trees or s in ev.shuffled for s in states):
            raise CompileError("a serially accumulated state is also block-reduced")
        if any(w["cond"] for w in writes):
            raise CompileError("conditional writes in a serial contraction")
        return {}
    axes = [(a.name, static_extent(a.extent)) for a in tile.axes]
    co, block = axes[-1]
    if loop["start"] == _var(co) and loop["step"] == block and loop["extent"] == extent:
        if ev.shuffle_length != 32 or ev.tree_length is None or ev.tree_length * 32 != block:
            raise CompileError("block contraction must combine a full warp butterfly and a block tree")
        if any(s not in ev.trees or s not in ev.shuffled for s in states):
            raise CompileError("every block-contracted state must be block-reduced")
        if not combines_are(tile, combine):
            raise CompileError("the block's partial states are not combined as the contraction needs")
        for w in writes:
            c = w["cond"]
            if not (len(c) == 1 and c[0].kind == "BinaryExpr" and c[0].op == "==" and c[0].left.kind == "Var"
                    and c[0].left.name == co and c[0].right.kind == "Literal" and c[0].right.value == 0):
                raise CompileError("block contraction results must be written by thread 0")
        return {co: 0}
    raise CompileError("contraction loop neither walks [0, K) nor strides the block across it")


def _tile_axes(tile: Node) -> list:
    return [(a.name, static_extent(a.extent)) for a in tile.axes]


# ----------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------

def looks_like_attention(ev: _Eval) -> bool:
    """A running max, a rescaled running sum and a dot product (a row softmax has no dot)."""
    reds = ev.reductions.values()
    dot = any(r["op"] == "add" and r["base"] is None and isinstance(r["value"], tuple)
              and r["value"][:2] == ("op", "multiply") and _is_load()(r["value"][2])
              and _is_load()(r["value"][3]) and r["value"][2] != r["value"][3] for r in reds)
    return dot and any(r["op"] == "maximum" for r in reds) and any(r["base"] is not None for r in reds)


def recognise_attention(pkg: KernelPackage, tile: Node, ev: _Eval) -> Plan:
    if not ev.writes:
        raise CompileError("attention body writes nothing")
    out = ev.writes[0]["buffer"]
    found = None
    states: list = []
    for w in ev.writes:
        if w["buffer"] != out or w["atomic"] or len(w["values"]) != 1 or len(w["index"]) != 2:
            raise CompileError("attention must write single elements of one matrix")
        epi, inner = strip_epilogue(pkg, w["values"][0])
        b = _match(op("multiply", V("S", _is_state), op("reciprocal", V("L", _is_state))), inner, {})
        if not b:
            raise CompileError("attention output is not acc * reciprocal(sum)")
        S, L = b["S"][1], b["L"][1]
        rs, rl = ev.reductions.get(S), ev.reductions.get(L)
        if rs is None or rl is None or rs["op"] != "add" or rl["op"] != "add":
            raise CompileError("attention accumulators are not running sums")
        bs = _match(op("add", op("multiply", ("acc", S), V("alpha")),
                       op("multiply", V("vld", _is_load()), V("beta"))), canon_scalars(pkg, rs["value"]), {})
        if not bs:
            raise CompileError("attention value sum is not acc*alpha + v*beta")
        bl = _match(op("add", op("multiply", ("acc", L), V("alpha")), op("multiply", ("lit", 1.0), V("beta"))),
                    canon_scalars(pkg, rl["value"]), {"alpha": bs["alpha"], "beta": bs["beta"]})
        if not bl:
            raise CompileError("attention normaliser is not sum*alpha + beta")
        ba = _match(op("exp", op("subtract", V("m", _is_acc), op("maximum", V("m"), V("score")))), bs["alpha"], {})
        if not ba or not _match(op("exp", op("subtract", V("score"), op("maximum", V("m"), V("score")))),
                                bs["beta"], ba):
            raise CompileError("attention rescale factors are not exp(m_old - m_new), exp(s - m_new)")
        M = ba["m"][1]
        rm = ev.reductions.get(M)
        score = ba["score"]
        if rm is None or rm["op"] != "maximum" or rm["base"] is not None or \
                canon_scalars(pkg, rm["value"]) != score:
            raise CompileError("attention running max does not track the score")
        if not (rs["loop"] == rl["loop"] == rm["loop"]):
            raise CompileError("attention states advance in different loops")
        mode = None
        for name, pattern in (("mul_recip", op("multiply", V("d", _is_acc), op("reciprocal", V("c", _is_s)))),
                              ("mul", op("multiply", V("d", _is_acc), V("c", _is_s))),
                              ("div", ("op", "divide", V("d", _is_acc), V("c", _is_s)))):
            if (bsc := _match(pattern, score, {})):
                mode = name
                break
        if mode is None:
            raise CompileError("attention score is not dot * c, dot * (1/c) or dot / c")
        D = bsc["d"][1]
        rd = ev.reductions.get(D)
        if rd is None or rd["op"] != "add" or rd["base"] is not None:
            raise CompileError("attention score is not a dot product")
        bd = _match(op("multiply", V("x", _is_load()), V("y", _is_load())), rd["value"], {})
        if not bd:
            raise CompileError("attention dot product is not a product of two loads")
        key, j = rm["loop"], rd["loop"]
        if _loop_info(ev, j)["parent"] != key:
            raise CompileError("the score's dot product must run inside the key loop")
        row, col = w["index"]
        for qa, ka in ((bd["x"], bd["y"]), (bd["y"], bd["x"])):
            if qa[2] == (row, _var(j)) and ka[2] == (_var(j), _var(key)):
                break
        else:
            raise CompileError("attention operands are not q[row, j] and kt[j, key]")
        vld = bs["vld"]
        if vld[2] != (_var(key), col):
            raise CompileError("attention values are not v[key, col]")
        sig = (qa[1], ka[1], vld[1], bsc["c"][1], mode, epi, key, j)
        if found is not None and found != sig:
            raise CompileError("attention outputs use different operands")
        found = sig
        states += [S, L, M]
    q, kt, v, c, mode, epi, key, j = found
    s_q, d = pkg.buffers[q].shape if len(pkg.buffers[q].shape) == 2 else (None, None)
    if s_q is None or len(pkg.buffers[kt].shape) != 2 or len(pkg.buffers[v].shape) != 2:
        raise CompileError("attention operands must be matrices")
    d2, s_kv = pkg.buffers[kt].shape
    s_kv2, dv = pkg.buffers[v].shape
    if d2 != d or s_kv2 != s_kv or tuple(pkg.buffers[out].shape) != (s_q, dv):
        raise CompileError("attention operand shapes are inconsistent")
    _f32(pkg, q, kt, v, out, c)
    jl = _loop_info(ev, j)
    if jl["start"] != _aff({}) or jl["step"] != 1 or jl["extent"] != d:
        raise CompileError("the score's dot product must walk the head dimension")
    merge: dict = {}
    for k in range(0, len(states), 3):
        S_, L_, M_ = states[k:k + 3]
        merge.update(online_combine(M_, [L_, S_]))
    fixed = _contraction_form(tile, ev, _loop_info(ev, key), s_kv, states, ev.writes, merge)
    check_cover(pkg, _tile_axes(tile), ev.writes, out, fixed)
    comp = bool(compensated_states(pkg.body, pkg))
    return _plan(pkg, "attention_f32", "lc_attention_f32_dot2" if comp else "lc_attention_f32",
                 {"scale": c, "q": q, "kt": kt, "v": v, "o": out},
                 {"bh": 1, "s_q": s_q, "s_kv": s_kv, "d": d, "dv": dv, "scale_mode": mode,
                  "epilogue": epi, "compensated": comp}, {"io": "f32"})


# ----------------------------------------------------------------------------
# GEMM written as one dot product per output (serial or block-cooperative)
# ----------------------------------------------------------------------------

def _gemm_terms(row, col, k, product) -> tuple[tuple, tuple, str]:
    """(A load, B load, layout) of product = A[row, k] * B[k, col] or B[col, k]."""
    x, y = product[2], product[3]
    for a, b in ((x, y), (y, x)):
        if not (_is_load()(a) and _is_load()(b)) or a[2] != (row, k):
            continue
        if b[2] == (k, col):
            return a, b, "kn"
        if b[2] == (col, k):
            return a, b, "nk"
    raise CompileError("product is not A[row, k] * B[k, col] for the written element")


def _gemm_plan(pkg: KernelPackage, a: str, b: str, bias: str | None, out: str, layout: str, epi: str,
               k: int) -> Plan:
    sa, sb, sc = pkg.buffers[a].shape, pkg.buffers[b].shape, pkg.buffers[out].shape
    if len(sa) != 2 or len(sb) != 2 or len(sc) != 2:
        raise CompileError("GEMM operands must be matrices")
    m, ka = sa
    n = sb[1] if layout == "kn" else sb[0]
    kb = sb[0] if layout == "kn" else sb[1]
    if ka != k or kb != k or tuple(sc) != (m, n):
        raise CompileError(f"GEMM shapes {sa} x {sb} -> {sc} do not match the contraction")
    _f32(pkg, a, b, out)
    bind = {"a": a, "b": b, "c": out}
    if bias is not None:
        if tuple(pkg.buffers[bias].shape) != (n,):
            raise CompileError("GEMM bias must be a vector over the output columns")
        _f32(pkg, bias)
        bind["bias"] = bias
    # the reference compensates the dot accumulation when the package states a tolerance
    comp = bool(compensated_states(pkg.body, pkg))
    return _plan(pkg, "gemm", "lc_gemm_f32_dot2" if comp else "lc_gemm", bind,
                 {"m": m, "n": n, "k": k, "b_layout": layout, "epilogue": epi, "compensated": comp},
                 {"ab": "f32", "c": "f32"})


def _split_bias(inner, is_acc_ok, col):
    """acc or add(acc, bias[col]) -> (acc, bias buffer or None)."""
    if is_acc_ok(inner):
        return inner, None
    b = _match(op("add", V("acc", is_acc_ok), V("bias", _is_load())), inner, {})
    if b and b["bias"][2] == (col,):
        return b["acc"], b["bias"][1]
    raise CompileError("GEMM result is not acc or acc + bias[col]")


def looks_like_dot(ev: _Eval) -> bool:
    return bool(ev.reductions) and all(
        r["op"] == "add" and r["base"] is None and isinstance(r["value"], tuple)
        and r["value"][:2] == ("op", "multiply") and _is_load()(r["value"][2]) and _is_load()(r["value"][3])
        and len(r["value"][2][2]) == 2 and len(r["value"][3][2]) == 2 and r["value"][2] != r["value"][3]
        for r in ev.reductions.values())


def recognise_dot_gemm(pkg: KernelPackage, tile: Node, ev: _Eval) -> Plan:
    if not ev.writes:
        raise CompileError("GEMM body writes nothing")
    out = ev.writes[0]["buffer"]
    sig = None
    states = []
    for w in ev.writes:
        if w["buffer"] != out or w["atomic"] or len(w["values"]) != 1 or len(w["index"]) != 2:
            raise CompileError("GEMM must write single elements of one matrix")
        row, col = w["index"]
        epi, inner = strip_epilogue(pkg, w["values"][0])
        acc, bias = _split_bias(inner, _is_state, col)
        red = ev.reductions.get(acc[1])
        if red is None:
            raise CompileError("GEMM result is not an accumulator")
        a, b, layout = _gemm_terms(row, col, _var(red["loop"]), red["value"])
        s = (a[1], b[1], bias, layout, epi, red["loop"])
        if sig is not None and s != sig:
            raise CompileError("GEMM outputs use different operands")
        sig = s
        states.append(acc[1])
    a, b, bias, layout, epi, kaxis = sig
    k = pkg.buffers[a].shape[1] if len(pkg.buffers[a].shape) == 2 else -1
    fixed = _contraction_form(tile, ev, _loop_info(ev, kaxis), k, states, ev.writes,
                              {name: fold_combine(name, "add") for name in states})
    if len(ev.loops) != 1:
        raise CompileError("GEMM dot form has loops besides the contraction")
    check_cover(pkg, _tile_axes(tile), ev.writes, out, fixed)
    return _gemm_plan(pkg, a, b, bias, out, layout, epi, k)


# ----------------------------------------------------------------------------
# shared-memory staged GEMM (cp.async tiles, optional split-K atomics)
# ----------------------------------------------------------------------------

_MAX_UNROLL = 1 << 16


class StagedEval(_Eval):
    """Evaluates a staged scalar-GEMM Tile with its loops unrolled.

    Block coordinates stay symbolic; the thread coordinates (the trailing Tile
    axes whose extents multiply to the block size) are enumerated when a
    shared-memory access has to be located.
    """

    def __init__(self, pkg: KernelPackage, tile: Node):
        super().__init__(pkg)
        self.smem = set()
        self.tile_axes = _tile_axes(tile)
        block = (pkg.kernel_meta.get("block") or [0])[0]
        threads, prod = [], 1
        for name, extent in reversed(self.tile_axes):
            if prod == block:
                break
            threads.insert(0, (name, extent))
            prod *= extent
        if prod != block or not threads:
            raise CompileError("the Tile's trailing axes do not form the thread block")
        self.thread_axes = threads
        grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for _, e in threads], indexing="ij")
        self.thread_env = {a: g.ravel() for (a, _), g in zip(threads, grids)}
        self.bind: dict = {}
        self.copies: dict = {}          # smem -> list of (region set, delta forms, src)
        self.terms: dict = {}           # accumulator -> list of product expressions
        self.steps = 0

    # loop variables are concrete
    def index(self, node: Any) -> frozenset:
        if isinstance(node, Node) and node.kind == "TernaryExpr":
            c = node.cond
            if not (c.kind == "BinaryExpr" and c.op in ("<", "<=", ">", ">=", "==", "!=")):
                raise CompileError("unsupported index condition")
            lv, rv = _aff_const(self.index(c.left)), _aff_const(self.index(c.right))
            if lv is None or rv is None:
                raise CompileError("index condition is not decided by loop values")
            take = {"<": lv < rv, "<=": lv <= rv, ">": lv > rv, ">=": lv >= rv, "==": lv == rv,
                    "!=": lv != rv}[c.op]
            return self.index(node.if_true if take else node.if_false)
        if isinstance(node, Node) and node.kind == "Var" and node.name in self.bind:
            return _aff({1: self.bind[node.name]})
        return aff_subst(super().index(node), self.bind)

    def _points(self, forms: tuple, lanes: int = 1, extra: dict | None = None) -> set:
        """Concrete shared-memory positions the block's threads address."""
        env = dict(self.thread_env)
        if extra:
            env.update(extra)
        cols = [np.broadcast_to(np.asarray(aff_eval(f, env), np.int64), (len(next(iter(self.thread_env.values()))),))
                for f in forms]
        pts = set()
        for lane in range(lanes):
            last = cols[-1] + lane
            pts.update(zip(*[c.tolist() for c in cols[:-1]], last.tolist()))
        return pts

    def stmt(self, s: Node) -> None:
        k = s.kind
        self.steps += 1
        if self.steps > _MAX_UNROLL * 8:
            raise CompileError("staged GEMM schedule too long to verify")
        if k == "CpAsyncCopy":
            self.copy(s)
        elif k in ("CpAsyncCommit", "CpAsyncWait", "Sync"):
            pass
        elif k == "Init":
            if float(s.identity) != 0.0:
                raise CompileError("staged accumulators must start at 0")
            self.terms[s.name] = []
            self.env[s.name] = ("acc", s.name)
        elif k == "Load" and s.input in self.smem:
            self.smem_load(s)
        elif k == "Accum":
            op_ = s.op.name if isinstance(s.op, Node) else str(s.op)
            if op_ != "add" or s.get("base") is not None or s.name not in self.terms:
                raise CompileError("staged accumulation must add into an initialised accumulator")
            value = self.value(s.value)
            if not (isinstance(value, tuple) and value[:2] == ("op", "multiply")):
                raise CompileError("staged accumulation must add products")
            self.terms[s.name].append(value)
        elif k in ("StridedLoop", "Loop"):
            self.unrolled_loop(s)
        else:
            super().stmt(s)

    def unrolled_loop(self, s: Node) -> None:
        name = s.axis.name
        extent = static_extent(s.axis.extent)
        start, step = s.get("start"), s.get("step")
        if s.get("end") is not None:
            raise CompileError("staged loops with a captured end are not supported")
        start_f = self.index(start) if start is not None else _aff({})
        step_v = _aff_const(self.index(step)) if step is not None else 1
        if step_v is None or step_v <= 0:
            raise CompileError("loop step must be a positive constant")
        start_v = _aff_const(start_f)
        if start_v is None:
            # a per-thread start: only copy loops may have one
            if any(inner.kind != "CpAsyncCopy" for inner in s.body):
                raise CompileError("a loop with a per-thread start may only hold copies")
            for inner in s.body:
                self.copy(inner, loop=(name, start_f, step_v, extent))
            return
        if (extent - start_v + step_v - 1) // step_v > _MAX_UNROLL:
            raise CompileError("staged loop too long to unroll")
        for value in range(start_v, extent, step_v):
            self.bind[name] = value
            self.run(s.body)
        self.bind.pop(name, None)

    def copy(self, s: Node, loop: tuple | None = None) -> None:
        if s.get("swizzle", "NONE") not in (None, "NONE"):
            raise CompileError("swizzled shared-memory copies are not supported")
        src = s.src
        if src not in self.pkg.buffers or self.pkg.buffers[src].dtype != "f32":
            raise CompileError("staged copies must read an f32 argument")
        lanes = int(s.nbytes) // 4
        if lanes < 1 or lanes * 4 != int(s.nbytes):
            raise CompileError("copy size is not a whole number of f32 elements")
        sidx = tuple(self.index(i) for i in s.smem_index)
        lane = s.get("lane_index")
        if lane is not None:
            lane = tuple(self.index(i) for i in lane)
            if len(lane) != 2 or len(sidx) != 2:
                raise CompileError("lane-indexed copies must address a 2-D shared buffer")
            sidx = (_aff_add(sidx[0], lane[0]), _aff_add(sidx[1], lane[1]))
        gidx = tuple(self.index(i) for i in s.src_index)
        if len(gidx) != len(sidx):
            raise CompileError("copy source and destination ranks differ")
        delta = tuple(_aff_add(g, t, -1) for g, t in zip(gidx, sidx))
        thread_vars = {a for a, _ in self.thread_axes}
        if loop is not None:
            thread_vars.add(loop[0])
        for dform in delta:
            if any(_mentions(dform, v) for v in thread_vars):
                raise CompileError("copy source is not a translate of its shared-memory position")
        if loop is None:
            pts = self._points(sidx, lanes)
        else:
            name, start_f, step_v, extent = loop
            pts = set()
            first = np.asarray(aff_eval(start_f, self.thread_env), np.int64)
            first = np.broadcast_to(first, (len(next(iter(self.thread_env.values()))),))
            for it in range(0, extent, step_v):
                vals = first + it
                live = vals < extent
                if not live.any():
                    break
                env = {a: v[live] for a, v in self.thread_env.items()}
                env[name] = vals[live]
                cols = [np.broadcast_to(np.asarray(aff_eval(f, env), np.int64), (int(live.sum()),)) for f in sidx]
                for ln in range(lanes):
                    pts.update(zip(*[c.tolist() for c in cols[:-1]], (cols[-1] + ln).tolist()))
        self.copies.setdefault(s.smem, []).append((pts, delta, src))

    def smem_load(self, s: Node) -> None:
        idx = tuple(self.index(i) for i in s.index)
        records = self.copies.get(s.input, [])
        for lane_no, name in enumerate(s.names):
            lidx = idx if lane_no == 0 else idx[:-1] + (_aff_add(idx[-1], _aff({1: lane_no})),)
            want = self._points(lidx)
            for pts, delta, src in reversed(records):
                hit = want & pts
                if not hit:
                    continue
                if hit != want:
                    raise CompileError("a shared-memory load spans several copies")
                self.env[name] = ("ld", src, tuple(_aff_add(f, d) for f, d in zip(lidx, delta)))
                break
            else:
                raise CompileError(f"load from {s.input} reads elements no copy wrote")


def _mentions(form: frozenset, var: str) -> bool:
    for term, _ in form:
        if term == var:
            return True
        if isinstance(term, tuple) and _mentions(term[1], var):
            return True
    return False


def recognise_staged_gemm(pkg: KernelPackage, tile: Node) -> Plan:
    ev = StagedEval(pkg, tile)
    for axis in tile.axes:
        ev.axes[axis.name] = static_extent(axis.extent)
    ev.run(tile.body)
    if not ev.writes:
        raise CompileError("staged GEMM writes nothing")
    out = ev.writes[0]["buffer"]
    atomic = ev.writes[0]["atomic"]
    if any(w["buffer"] != out or w["atomic"] != atomic or w["cond"] for w in ev.writes):
        raise CompileError("staged GEMM must write one matrix the same way everywhere")
    if atomic and out not in pkg.kernel_meta.get("zero_outputs", []):
        raise CompileError("atomic partial sums need the output in zero_outputs")
    thread_or_block = {a for a, _ in ev.tile_axes}
    sig = None
    k_sets = []
    for w in ev.writes:
        if len(w["index"]) != 2:
            raise CompileError("staged GEMM must write a matrix")
        row, col0 = w["index"]
        for lane, value in enumerate(w["values"]):
            col = _aff_add(col0, _aff({1: lane}))
            epi, inner = strip_epilogue(pkg, value)
            try:
                acc, bias = _split_bias(inner, _is_acc, col)
            except CompileError:
                acc, epi = general_epilogue(pkg, value, row, col)
                bias = None
            terms = ev.terms.get(acc[1])
            if not terms:
                raise CompileError("staged GEMM writes an accumulator with no products")
            ks = []
            for t in terms:
                x, y = t[2], t[3]
                for a, b in ((x, y), (y, x)):
                    if _is_load()(a) and _is_load()(b) and len(a[2]) == 2 and len(b[2]) == 2 and a[2][0] == row:
                        kf = a[2][1]
                        if b[2] == (kf, col):
                            layout = "kn"
                        elif b[2] == (col, kf):
                            layout = "nk"
                        else:
                            continue
                        break
                else:
                    raise CompileError("a staged product is not A[row, k] * B[k, col]")
                s = (a[1], b[1], bias, layout, epi)
                if sig is not None and s != sig:
                    raise CompileError("staged GEMM outputs use different operands")
                sig = s
                ks.append(kf)
            k_sets.append(ks)
    a, b, bias, layout, epi = sig
    post = None
    if isinstance(epi, tuple):
        post, epi = epi[1], "none"
        if atomic:
            raise CompileError("split-K partial sums cannot carry an epilogue")
    if atomic and (bias is not None or epi != "none"):
        raise CompileError("split-K partial sums cannot carry a bias or activation")
    k = pkg.buffers[a].shape[1]
    # the axes the write does not address split the contraction
    used = set()
    for w in ev.writes:
        for f in w["index"]:
            used |= {v for v in thread_or_block if _mentions(f, v)}
    split = [(n, e) for n, e in ev.tile_axes if n not in used]
    if split and not atomic:
        raise CompileError("Tile axes that the write ignores need atomic accumulation")
    combos = list(itertools.product(*[range(e) for _, e in split])) or [()]
    if len(combos) * max(len(x) for x in k_sets) > (1 << 22):
        raise CompileError("split-K schedule too large to verify")
    for ks in k_sets:
        seen = []
        for combo in combos:
            env = {n: v for (n, _), v in zip(split, combo)}
            for kf in ks:
                if any(_mentions(kf, v) for v in thread_or_block if v not in env):
                    raise CompileError("the contraction index depends on the output position")
                seen.append(int(aff_eval(kf, env)))
        if sorted(seen) != list(range(k)):
            raise CompileError("the products do not cover the contraction exactly once")
    check_cover(pkg, [(n, e) for n, e in ev.tile_axes if n not in dict(split)], ev.writes, out,
                repeat=1)
    plan = _gemm_plan(pkg, a, b, bias, out, layout, epi, k)
    if post is not None:
        plan.params["post"] = compile_epilogue(pkg, post, out, plan.params["m"], plan.params["n"])
    return plan


def general_epilogue(pkg: KernelPackage, value, row: frozenset, col: frozenset) -> tuple:
    """(accumulator, ("expr", e)) for a written value that is any expression of
    one accumulator, literals, scalar arguments and loads at the output's row
    and column: e has the accumulator as ("acc",) and each load index
    component as a constant or ("row" | "col", offset)."""
    accs = set()

    def component(c):
        v = _aff_const(c)
        if v is not None:
            return v
        for name, form in (("row", row), ("col", col)):
            d = _aff_const(_aff_add(c, form, -1))
            if d is not None:
                return (name, d)
        raise CompileError("an epilogue load is not addressed by the output position")

    def norm(e):
        if not isinstance(e, tuple) or not e:
            raise CompileError(f"unsupported epilogue value {e!r}")
        kind = e[0]
        if kind == "acc":
            accs.add(e)
            return ("acc",)
        if kind in ("lit", "s"):
            return e
        if kind == "ld":
            if e[1] not in pkg.buffers:
                raise CompileError("an epilogue reads shared memory")
            return ("ld", e[1], tuple(component(c) for c in e[2]))
        if kind == "op":
            return ("op", e[1], *(norm(x) for x in e[2:]))
        if kind == "cast":
            return ("cast", e[1], norm(e[2]))
        raise CompileError(f"unsupported epilogue value {kind}")

    expr = norm(_drop_copies(canon_scalars(pkg, value)))
    if len(accs) != 1:
        raise CompileError("a GEMM epilogue must read exactly one accumulator")
    return accs.pop(), ("expr", expr)


# ----------------------------------------------------------------------------
# the fragment attention tile (m16n8k16 fragment algebra)
# ----------------------------------------------------------------------------

def _op_name(x) -> str:
    return x.name if isinstance(x, Node) else str(x)


def recognise_fragment_attention(pkg: KernelPackage, tile: Node) -> Plan:
    """The FragmentRowReduce / FragmentApply / FragmentRepack attention chain.

    Matches, statement by statement, the chain of
    examples/phase9/fragments/fragment_attention_tile_f16 (ptx_tensor.py:459-618):
    A <- Q; B_i <- Kt[:, 8i:8i+8]; S_i = A B_i; pivot = rowmax(S);
    S_i = exp(S_i - pivot); denom = rowsum(S); S_i = S_i / denom; A <- f16(S);
    B <- V; O = A B; store O.  One m16 tile of queries, K = 16 (one k step),
    n_frag * 8 keys, 8 value columns.
    """
    body = [s for s in tile.body if s.kind != "RegFragment"]
    kinds = [s.kind for s in body]
    it = iter(body)

    def take(kind):
        s = next(it, None)
        if s is None or s.kind != kind:
            raise CompileError(f"fragment attention chain: expected {kind}, found {getattr(s, 'kind', None)}")
        return s

    def origin(s):
        return tuple(_aff_const(_Eval(pkg).index(i)) for i in s.src_index)

    qa = take("LdmatrixLoad")
    if qa.role != "a" or origin(qa) != (0, 0) or qa.get("b_trans"):
        raise CompileError("fragment attention: A must be Q at (0, 0)")
    n_frag = kinds.count("MmaSyncPtx") - 1
    scores = []
    for i in range(n_frag):
        kb = take("LdmatrixLoad")
        mma = take("MmaSyncPtx")
        if kb.role != "b" or kb.get("b_trans") or origin(kb) != (0, 8 * i) or mma.a_frag != qa.frag \
                or mma.b_frag != kb.frag or tuple(mma.shape) != (16, 8, 16) or mma.ab_dtype != "f16" \
                or mma.c_dtype != "f32":
            raise CompileError("fragment attention: S_i = Q Kt[:, 8i:8i+8] expected")
        if i and kb.src_buffer != kt:
            raise CompileError("fragment attention: all B fragments must come from one Kt")
        kt = kb.src_buffer
        scores.append(mma.c_frag)
    red = take("FragmentRowReduce")
    if _op_name(red.op) != "maximum" or tuple(red.frags) != tuple(scores):
        raise CompileError("fragment attention: row max of the scores expected")
    for f in scores:
        ap = take("FragmentApply")
        post = tuple(_op_name(x) for x in ap.get("post", ()))
        if ap.out != f or _op_name(ap.op) != "subtract" or ap.args[0] != f or \
                tuple(ap.args[1]) != (red.top, red.bot) or post != ("exp",):
            raise CompileError("fragment attention: exp(S - rowmax) expected")
    den = take("FragmentRowReduce")
    if _op_name(den.op) != "add" or tuple(den.frags) != tuple(scores):
        raise CompileError("fragment attention: row sum expected")
    for f in scores:
        ap = take("FragmentApply")
        if ap.out != f or _op_name(ap.op) != "divide" or ap.args[0] != f or \
                tuple(ap.args[1]) != (den.top, den.bot) or tuple(ap.get("post", ())):
            raise CompileError("fragment attention: division by the row sum expected")
    rp = take("FragmentRepack")
    if rp.frag != qa.frag or tuple(rp.srcs) != tuple(scores) or rp.ab_dtype != "f16":
        raise CompileError("fragment attention: P must be repacked to f16 into the A fragment")
    vb = take("LdmatrixLoad")
    mma = take("MmaSyncPtx")
    st = take("RegStore")
    if next(it, None) is not None:
        raise CompileError("fragment attention: statements after the store")
    if vb.role != "b" or vb.get("b_trans") or origin(vb) != (0, 0) or mma.a_frag != qa.frag \
            or mma.b_frag != vb.frag or tuple(mma.shape) != (16, 8, 16):
        raise CompileError("fragment attention: O = P V expected")
    if st.frag != mma.c_frag or st.get("epilogue") is not None or st.get("atomic") or \
            tuple(_aff_const(_Eval(pkg).index(i)) for i in st.dst_index) != (0, 0):
        raise CompileError("fragment attention: O stored at (0, 0) without an epilogue expected")
    q, v, out = qa.src_buffer, vb.src_buffer, st.dst_buffer
    sq, sk, sv, so = (pkg.buffers[b].shape for b in (q, kt, v, out))
    if tuple(sq) != (16, 16) or tuple(sk) != (16, 8 * n_frag) or tuple(sv) != (8 * n_frag, 8) or \
            tuple(so) != (16, 8):
        raise CompileError(f"fragment attention shapes {sq} {sk} {sv} -> {so} unsupported")
    _f32(pkg, q, kt, v, out)
    return _plan(pkg, "attention_tile_f16q", "lc_attention_tile_f16q", {"q": q, "kt": kt, "v": v, "o": out},
                 {"bh": 1, "s_q": 16, "s_kv": 8 * n_frag, "d": 16, "dv": 8}, {"io": "f32", "compute": "f16"})
