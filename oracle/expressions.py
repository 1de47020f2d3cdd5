"""CPU oracle for the hot path — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the thing measured or shipped: only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import it.  The product path (``compile.py``,
``lazy_compiler_b200``) never does, and fails loudly when the CUDA library is
missing.

It restates, in numpy with float64 intermediates, the reference's own
independent references for each operation class:

* inputs: ``default_rng(seed + offset).standard_normal(shape)`` drawn in
  float64 then cast, ``data`` arguments taken verbatim
  (tools/check_compiler.py:124-143 ``input_array``);
* sum / mean / row sum, RMSNorm, softmax (float64 max-subtraction) and L2 norm
  (tools/expressions_open.py:27-30, 54-63, 77-89);
* matmul and attention in float64 (tools/expressions_open.py:66-73, 92-104);
* GELU erf / tanh with explicit f32 boundaries and narrow-type RNE
  quantisation (tests/test_gelu.py:35-66);
* FP16 / BF16 RNE quantisation of tensor-core operands
  (tests/test_tensor_cores.py:38-44);
* the comparison: ``np.isclose(actual, ref, rtol, atol, equal_nan=False)``
  with matching shapes, scalar outputs as one-element buffers, exact compare
  for zero-tolerance integer outputs (tools/check_compiler.py:187-231).

Parity is pinned: ``tests/test_oracle.py`` checks these functions against
every golden ``expected.npz`` the reference ships for the hot path
(copied to ``tests/golden/packages`` by ``tests/golden/make_golden.py``).
"""
from __future__ import annotations

import math

import numpy as np

DTYPES = {"f32": np.float32, "f16": np.float16, "f64": np.float64, "i32": np.int32,
          "bf16": np.float32, "i64": np.int64, "u32": np.uint32, "u8": np.uint8}


# ---------------------------------------------------------------- inputs

def input_array(arg: dict, seed_offset: int = 0, pattern: str = "normal") -> np.ndarray:
    """Seeded input for one meta.json argument (tools/check_compiler.py:124-143).

    ``bf16`` arguments are returned as float32 values already rounded to bf16.
    """
    kind = arg["dtype"]
    dtype = DTYPES[kind]
    shape = tuple(arg.get("shape") or [1])
    if "data" in arg:
        out = np.asarray(arg["data"], dtype=np.float64 if kind == "bf16" else dtype).reshape(shape)
        return quantize(out, "bf16") if kind == "bf16" else out
    seed = int(arg.get("seed", 0)) + seed_offset
    rng = np.random.default_rng(seed)
    if pattern == "zeros":
        result = np.zeros(shape)
    elif pattern == "ones":
        result = np.ones(shape)
    elif pattern == "alternating":
        result = (np.arange(math.prod(shape)).reshape(shape) % 2 * 2 - 1) * (1 + seed % 3)
    elif pattern == "wide":
        result = rng.standard_normal(shape) * 8
    else:
        result = rng.standard_normal(shape)
    if kind == "bf16":
        return quantize(np.asarray(result, np.float32), "bf16")
    return np.asarray(result, dtype=dtype)


def uniform(n: int, seed: int) -> np.ndarray:
    """U[-1, 1] fp32 input of the whole-array sum configuration."""
    return np.random.default_rng(seed).uniform(-1.0, 1.0, n).astype(np.float32)


def normal(shape, seed: int, mean: float = 0.0, std: float = 1.0, dtype=np.float32) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(shape) * std + mean).astype(dtype)


# ---------------------------------------------------------------- rounding

def quantize(values, kind: str) -> np.ndarray:
    """Host RNE conversion to ``kind`` returned as float32 (tests/test_gelu.py:35-48)."""
    values = np.asarray(values, np.float32)
    with np.errstate(all="ignore"):
        if kind == "f32":
            return values.copy()
        if kind == "f16":
            return values.astype(np.float16).astype(np.float32)
        if kind == "bf16":
            words = values.view(np.uint32)
            rounded = words + np.uint32(32767) + ((words >> 16) & np.uint32(1))
            result = ((rounded >> 16) << 16).view(np.float32)
            return np.where(np.isnan(values), np.float32(np.nan), result)
    raise ValueError(f"unsupported oracle type {kind}")


def to_bf16_bits(values) -> np.ndarray:
    """float32 values -> uint16 bf16 words (RNE)."""
    q = quantize(values, "bf16")
    return (q.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(words) -> np.ndarray:
    return (np.asarray(words, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- pointwise

def add(x0, x1):
    return [(x0 + x1)]


def axpb(a, b, x):
    """b + a * x in float32 (expressions_open p02: x * 2.0 + 1.0)."""
    return [(x * np.float32(a) + np.float32(b)).astype(np.float32)]


def relumul(x, y):
    return [(np.maximum(x, 0) * y).astype(np.float32)]


def gelu(values, approximate: str = "none", kind: str = "f32") -> np.ndarray:
    """GELU formula oracle (tests/test_gelu.py:51-66), f32 boundaries, quantised I/O."""
    x = quantize(values, kind)
    f = np.float32
    with np.errstate(all="ignore"):
        if approximate == "none":
            scaled = x / f(math.sqrt(2.0))
            gate = np.asarray([math.erf(float(v)) for v in scaled.ravel()], np.float32).reshape(x.shape)
        elif approximate == "tanh":
            cube = (x * x) * x
            scaled = f(math.sqrt(2.0 / math.pi)) * (x + f(0.044715) * cube)
            gate = np.asarray([math.tanh(float(v)) for v in scaled.ravel()], np.float32).reshape(x.shape)
        else:
            raise ValueError(approximate)
        return quantize((f(0.5) * x) * (f(1.0) + gate), kind)


def classify(values) -> np.ndarray:
    """Exceptional-value flags (tests/test_gelu.py:165-168)."""
    values = np.asarray(values, np.float32)
    return np.stack((np.isnan(values), np.isposinf(values), np.isneginf(values),
                     values == 0, (values == 0) & np.signbit(values),
                     np.isfinite(values)), axis=1).astype(np.int32)


def exceptional_inputs() -> np.ndarray:
    """NaNs, infinities, signed zeros, subnormal and tanh-branch boundaries (tests/test_gelu.py:142-156)."""
    return np.asarray([
        0x00000000, 0x80000000, 0x7f800000, 0xff800000, 0x7fc00000, 0xffc12345,
        0x7f800001, 0xff800001, 0x00000001, 0x80000001, 0x007fffff, 0x807fffff,
        0x00800000, 0x80800000, 0x7f7fffff, 0xff7fffff, 0x3f800000, 0xbf800000,
        0x33800000, 0xb3800000, 0x3e7fffff, 0xbe7fffff, 0x3e800000, 0xbe800000,
        0x3e800001, 0xbe800001, 0x477fe000, 0xc77fe000, 0x477ff000, 0xc77ff000,
        0x7f7f0000, 0xff7f0000, 0x3e9f0000, 0xbe9f0000, 0x3e9f8000, 0xbe9f8000,
        0x3ea00000,
    ], np.uint32).view(np.float32)


def gelu_finite_inputs() -> np.ndarray:
    """Finite GELU sweep with a partial final CTA (tests/test_gelu.py:69-76)."""
    rng = np.random.default_rng(260029)
    return np.concatenate((
        np.linspace(-9, 9, 193, dtype=np.float32),
        rng.uniform(-7, 7, 64).astype(np.float32),
        np.asarray([0, -0.0, 2**-24, -2**-24, 2**-14, -2**-14, 0.25, -0.25, 1, -1, 3, -3,
                    12, -12, 20, -20], np.float32),
    ))


# ---------------------------------------------------------------- reductions and rows

def sum_(x):
    return [np.asarray(np.asarray(x).astype(np.float64).sum(), np.float32)]


def mean(x, count=None):
    x = np.asarray(x).astype(np.float64)
    n = float(count) if count is not None else x.size
    return [np.asarray(x.sum() / n, np.float32)]


def rowsum(x):
    return [x.astype(np.float64).sum(-1).astype(np.float32)]


def rmsnorm(x, w, eps: float = 1e-5, count: float | None = None):
    """x / sqrt(mean(x^2) + eps) * w (expressions_open f01), mean over ``count``."""
    x64 = x.astype(np.float64)
    n = float(count) if count is not None else x.shape[-1]
    ms = (x64 ** 2).sum(-1, keepdims=True) / n
    return [(x / np.sqrt(ms + eps) * w).astype(np.float32)]


def softmax(x, axis: int = -1):
    """Float64 max-subtracted softmax (expressions_open.py:27-30, f02)."""
    x = x.astype(np.float64)
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return [(e / e.sum(axis=axis, keepdims=True)).astype(np.float32)]


def l2norm(x):
    return [(x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True))).astype(np.float32)]


# ---------------------------------------------------------------- tensor cores

def gemm(a, b, b_layout: str = "kn", epilogue: str = "none", ab: str = "f16", out: str = "f32",
         bias=None, transpose_out: bool = False):
    """float64 matmul of the quantised operands, optional bias and GELU, quantised output.

    Operands are quantised to ``ab`` (tests/test_tensor_cores.py:38-44; a no-op
    for f32); the product is float64 (expressions_open.py:66-73), rounded to
    f32 as the accumulator; a bias is added in f32 (the IR's
    ``add(acc, bias[col])``, examples/phase9/generated/phase9_bias_gelu_gemm);
    the epilogue is the GELU formula of tests/test_gelu.py:51-66 or max(., 0)
    (the tensor fixtures' bias + ReLU, tests/test_tensor_cores.py:129-135);
    ``transpose_out`` stores C transposed.
    """
    a = quantize(a, ab).astype(np.float64)
    b = quantize(b, ab).astype(np.float64)
    if b_layout == "nk":
        b = np.swapaxes(b, -1, -2)
    with np.errstate(all="ignore"):
        c = (a @ b).astype(np.float32)
        if bias is not None:
            c = (c + np.asarray(bias, np.float32)).astype(np.float32)
    if epilogue == "gelu_erf":
        c = gelu(c, "none", "f32").reshape(c.shape)
    elif epilogue == "gelu_tanh":
        c = gelu(c, "tanh", "f32").reshape(c.shape)
    elif epilogue == "relu":
        c = np.maximum(c, np.float32(0))
    elif epilogue != "none":
        raise ValueError(epilogue)
    if transpose_out:
        c = np.ascontiguousarray(np.swapaxes(c, -1, -2))
    return [quantize(c, out) if out != "f32" else c]


def gemm_chain_f16(x, y, z, ab: str = "f16", y_layout: str = "kn", z_layout: str = "kn"):
    """(q(q(x) @ q(y)) @ q(z)): the C -> A fragment repack of two tensor-core
    products (tests/test_tensor_cores.py:169-171); "nk" operands are stored
    transposed."""
    y = np.swapaxes(y, -1, -2) if y_layout == "nk" else y
    z = np.swapaxes(z, -1, -2) if z_layout == "nk" else z
    xy = quantize(x, ab).astype(np.float64) @ quantize(y, ab).astype(np.float64)
    return [(quantize(xy, ab).astype(np.float64) @ quantize(z, ab).astype(np.float64)).astype(np.float32)]


def sdpa(q, k, v, scale: float):
    """softmax(scale * q k^T) v in float64 per leading index (expressions_open.py:92-104)."""
    q64, k64, v64 = (np.asarray(t, np.float64) for t in (q, k, v))
    s = np.einsum("...qd,...kd->...qk", q64, k64) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return [np.einsum("...qk,...kd->...qd", p, v64)]


def attention_kt(q, kt, v, divisor: float):
    """Reference attention with K pre-transposed (expressions_open a01/a02)."""
    s = (q.astype(np.float64) @ kt.astype(np.float64)) / divisor
    return [(softmax(s)[0].astype(np.float64) @ v.astype(np.float64)).astype(np.float32)]


def attention_f32(q, kt, v, scale: float, mode: str = "div", epilogue: str = "none"):
    """FP32 attention of the IR class: softmax(score(q @ kt)) @ v, then GELU.

    q [..., s_q, d], kt [..., d, s_kv], v [..., s_kv, dv] (expressions_open.py:92-104
    takes kt pre-transposed).  The score is dot * c ("mul"), dot * f32(1/c)
    ("mul_recip", the IR's reciprocal-then-multiply) or dot / c ("div"), in
    float64 after the f32 reciprocal; the result is rounded to f32 before the
    GELU of tests/test_gelu.py:51-66.
    """
    q64, kt64, v64 = (np.asarray(t, np.float64) for t in (q, kt, v))
    dot = q64 @ kt64
    c = np.float32(scale)
    if mode == "mul":
        s = dot * np.float64(c)
    elif mode == "mul_recip":
        s = dot * np.float64(np.float32(1.0) / c)
    elif mode == "div":
        s = dot / np.float64(c)
    else:
        raise ValueError(mode)
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    out = (p @ v64).astype(np.float32)
    if epilogue == "gelu_erf":
        out = gelu(out, "none", "f32").reshape(out.shape)
    elif epilogue == "gelu_tanh":
        out = gelu(out, "tanh", "f32").reshape(out.shape)
    elif epilogue != "none":
        raise ValueError(epilogue)
    return [out]


# ---------------------------------------------------------------- plans

def evaluate(plan: dict, arrays: dict, ir=None) -> dict:
    """Reference outputs of one launch plan from named input arrays.

    Pointwise-program plans are checked against their IR (``ir``: the
    package's kernel.ir.json), which oracle/pointwise_ir.py evaluates; plans
    with an epilogue program against oracle/staged_ir.py.
    """
    op = plan["op"]
    if plan["params"].get("block"):
        # a block program: the block oracle runs the IR the same way
        if ir is None:
            raise ValueError("block-program plans are evaluated from their IR: pass ir=")
        from oracle.staged_ir import evaluate as evaluate_staged
        return evaluate_staged(ir, arrays)
    if "post" in plan["params"]:
        # a staged matmul storing an expression of its accumulators: the block oracle
        if ir is None:
            raise ValueError("plans with an epilogue program are evaluated from their IR: pass ir=")
        from oracle.staged_ir import evaluate as evaluate_staged
        return evaluate_staged(ir, arrays)
    if op == "pointwise":
        if ir is None:
            raise ValueError("pointwise plans are evaluated from their IR: pass ir=")
        if plan["params"].get("lanes"):
            from oracle.fragment_ir import evaluate as evaluate_fragments
            return evaluate_fragments(ir, arrays)
        from oracle.pointwise_ir import evaluate as evaluate_ir
        return evaluate_ir(ir, arrays)
    bind = plan["bind"]
    p = plan["params"]
    g = lambda role: arrays[bind[role]]  # noqa: E731
    s = lambda role: float(np.asarray(arrays[bind[role]]).ravel()[0])  # noqa: E731
    if op == "add_f32":
        out = add(g("x0"), g("x1"))
    elif op == "axpb_f32":
        out = axpb(s("a"), s("b"), g("x"))
    elif op == "relumul_f32":
        out = relumul(g("x"), g("y"))
    elif op == "gelu":
        x = g("x")
        out = [gelu(x.astype(np.float32), p["approximate"], plan["dtypes"]["io"]).reshape(x.shape)]
    elif op == "sum_f32":
        out = sum_(g("x"))
    elif op == "mean_f32":
        out = mean(g("x"), s("count"))
    elif op == "rowsum_f32":
        out = rowsum(g("x"))
    elif op == "rmsnorm_f32":
        out = rmsnorm(g("x"), g("w"), s("eps"), s("count"))
    elif op == "softmax_f32":
        out = softmax(g("x"))
    elif op == "l2norm_f32":
        out = l2norm(g("x"))
    elif op == "attention_tile_f16q":
        out = attention_tile_f16(g("q"), g("kt"), g("v"))
    elif op == "rowdot_f32":
        x = np.asarray(g("x"), np.float32)
        fx = x if p["activation"] == "none" else gelu(x, "none" if p["activation"] == "gelu_erf" else "tanh",
                                                      "f32").reshape(x.shape)
        out = [(np.asarray(g("y"), np.float64) * fx.astype(np.float64)).sum(-1).astype(np.float32)]
    elif op == "gemm":
        bias = g("bias") if "bias" in bind else None
        out = gemm(g("a"), g("b"), p["b_layout"], p["epilogue"], plan["dtypes"]["ab"], plan["dtypes"]["c"],
                   bias, p.get("transpose_out", False))
    elif op == "gemm_mixed":
        bias = g("bias") if "bias" in bind else None
        out = gemm(g("a"), g("b"), p["b_layout"], p["epilogue"], plan["dtypes"]["mma"], plan["dtypes"]["c"],
                   bias, p["transpose"])
    elif op == "gemm_chain":
        out = gemm_chain_f16(g("x"), g("y"), g("z"), plan["dtypes"]["mma"], p["y_layout"], p["z_layout"])
        if plan["dtypes"]["c"] != "f32":
            out = [quantize(out[0], plan["dtypes"]["c"])]
    elif op == "attention_f32":
        shape = lambda a, tail: np.asarray(a).reshape((p["bh"],) + tail)  # noqa: E731
        out = attention_f32(shape(g("q"), (p["s_q"], p["d"])), shape(g("kt"), (p["d"], p["s_kv"])),
                            shape(g("v"), (p["s_kv"], p["dv"])), s("scale"), p["scale_mode"], p["epilogue"])
        out = [out[0].reshape((p["s_q"], p["dv"])) if p["bh"] == 1 else out[0]]
    else:
        raise ValueError(f"no oracle for {op}")
    key = next(bind[r] for r in ("out", "c", "o") if r in bind)
    return {key: out[0]}


def compare(actual, reference, rtol: float, atol: float) -> dict:
    """One comparison row with the reference harness semantics (check_compiler.py:187-231)."""
    actual = np.asarray(actual)
    reference = np.asarray(reference)
    if actual.shape != reference.shape:
        if actual.size == reference.size == 1:
            actual = actual.reshape(reference.shape)
        else:
            raise ValueError(f"shape {actual.shape} != reference {reference.shape}")
    if reference.dtype.kind in "iu" and rtol == atol == 0:
        good = actual.astype(object) == reference.astype(object)
        delta = np.asarray(np.abs(actual.astype(object) - reference.astype(object)), np.float64)
    else:
        good = np.isclose(actual.astype(np.float64), reference.astype(np.float64),
                          rtol=rtol, atol=atol, equal_nan=False)
        delta = np.abs(actual.astype(np.float64) - reference.astype(np.float64))
    finite = delta[np.isfinite(delta)]
    row = {"pass": bool(np.all(good)), "elements": int(actual.size),
           "mismatches": int(np.count_nonzero(~np.asarray(good, bool))),
           "max_abs_error": float(finite.max()) if finite.size else None}
    if not row["pass"]:
        idx = tuple(np.argwhere(~np.asarray(good, bool))[0]) if actual.shape else ()
        row["first_failure"] = {"index": [int(i) for i in idx], "actual": float(actual[idx]),
                                "expected": float(reference[idx])}
    return row


def attention_tile_f16(q, kt, v):
    """Fragment attention tile oracle (tests/test_fragment_rows.py:196-203).

    f16-quantised operands, f32 scores, float64 softmax, weights rounded to
    f16 before the second product (FragmentRepack semantics).
    """
    q, kt, v = (quantize(x, "f16").astype(np.float64) for x in (q, kt, v))
    scores = (q @ kt).astype(np.float32)
    shifted = scores.astype(np.float64) - np.max(scores, axis=1, keepdims=True)
    weights = np.exp(shifted)
    weights = (weights / np.sum(weights, axis=1, keepdims=True)).astype(np.float32)
    rounded = quantize(weights, "f16").astype(np.float64)
    return [(rounded @ v).astype(np.float32)]


def sdpa_f16(q, k, v, scale: float):
    """f16 SDPA reference: float64 softmax of f16 inputs, f16-rounded weights, f16 output.

    Matches the FragmentRepack rounding of the reference's f16 attention tile
    (P is rounded to f16 before the PV product) and returns float32 values of
    the f16 output.
    """
    q64, k64, v64 = (quantize(t, "f16").astype(np.float64) for t in (q, k, v))
    s = np.einsum("...qd,...kd->...qk", q64, k64) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return [quantize(np.einsum("...qk,...kd->...qd", p, v64).astype(np.float32), "f16")]
