"""Pointwise programs: straight-line scalar Tile bodies compiled to a register
program that one CUDA kernel (csrc/pointwise.cu) runs per tile point.

A Tile whose body is Load / Let / Assign / Select / Write over its axes,
with affine indices, is an elementwise computation of any op mix the
reference admits.  The fixed kernels (add, scale-shift, relu*mul, GELU)
cover the common classes at full bandwidth; everything else in this family
(several outputs per point, bit casts and classifications, f16/bf16 compute,
comparisons and selects) compiles here.

The compiler follows the reference's scalar lowering rule by rule
(ptx_backend.py:406-1177): literal rounding (:406-438), conversions
(:470-537), C type promotion (:618-630), comparisons with unordered `!=`
(:650-663), per-node f16/bf16 rounding of binary operators (:665-716) and of
IR statements (:981-984), and the composite operations' exact sequences of
separately rounded f32 steps — exp as ex2.approx(x log2 e) (:1062-1068),
tanh by odd polynomial or exponential formula (:1090-1119), erf by
Abramowitz-Stegun 7.1.26 (:1141-1169), GELU (:1122-1140), sigmoid/silu
(:1170-1176).  The result is a list of primitive register operations; the
kernel executes each with the PTX instruction the reference emits for it.

Types: f32, f16, bf16 (held widened in f32 registers), s32 and pred (held
as 0/1 words).  Indices must be affine in the Tile axes; every output
element must be written exactly once.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field

import numpy as np

from .ir import CompileError, KernelPackage, Node, dtype_name, static_extent

# ---------------------------------------------------------------- instruction set
# Opcodes shared with csrc/pointwise.cu (LC_PW_* in include/lazyb200.h).
OPCODES = [
    "MOV", "CONST",
    "LD_F32", "LD_F16", "LD_BF16", "LD_S32",
    "ST_F32", "ST_F16", "ST_BF16", "ST_S32",
    "FADD", "FSUB", "FMUL", "FDIV", "FFMA", "FNEG", "FABS", "FMAX", "FMIN", "FSQRT",
    "FFLOOR", "FCEIL", "FTRUNC", "FRINT", "FEX2", "FLG2", "FSIN", "FCOS", "FCOPYSIGN",
    "RND_F16", "RND_BF16", "F2I", "I2F", "I2H", "I2BF",
    "IADD", "ISUB", "IMUL", "IDIV", "IREM", "ISHL", "ISHR", "IAND", "IOR", "IXOR", "INOT",
    "INEG", "IABS", "IMAX", "IMIN", "IPOPC",
    "FEQ", "FNE", "FLT", "FLE", "FGT", "FGE",
    "IEQ", "INE", "ILT", "ILE", "IGT", "IGE",
    "PAND", "POR", "SEL",
    # lane programs (fragment algebra, lazy_compiler_b200/fragment_vm.py)
    "COORD", "LDX_F32", "LDX_F16", "LDX_BF16", "LDX_S32", "STX_F32", "STX_F16", "STX_BF16", "STX_S32",
    "STX_ADD_F32", "SHFL_XOR", "PACK_F16X2", "PACK_BF16X2", "MMA_F16", "MMA_BF16",
    "FREM",
    # row programs (lazy_compiler_b200/rowprog.py)
    "STATE", "PARTIAL", "PARTNER", "SETP",
    # serial programs (lazy_compiler_b200/serial.py)
    "LOOPB", "LOOPE",
    # block programs (lazy_compiler_b200/blockprog.py)
    "BRA", "BRZ", "SLB", "SLE", "LDS", "STS", "BAR", "WSYNC", "TID",
]
OP = {name: i for i, name in enumerate(OPCODES)}

MAX_CODE = 2048
MAX_CONST = 128
MAX_FORMS = 32
MAX_BUFFERS = 16
MAX_AXES = 8
MAX_REGS = 128

_TYPES = {"float": "f32", "int": "s32", "i32": "s32", "__half": "f16", "half": "f16",
          "__nv_bfloat16": "bf16", "bool": "pred"}
_FLOATS = ("f32", "f16", "bf16")
_SUPPORTED = ("f32", "f16", "bf16", "s32", "pred")
_STORAGE = {"f32": "F32", "f16": "F16", "bf16": "BF16", "s32": "S32"}


def vm_type(dt) -> str:
    name = dtype_name(dt) if isinstance(dt, Node) else str(dt)
    name = _TYPES.get(name, name)
    if name not in _SUPPORTED:
        raise CompileError(f"pointwise programs do not support type {name}")
    return name


def f32_word(x: float) -> int:
    """Bits of x rounded once to binary32 (round to nearest even, overflow to inf)."""
    try:
        return struct.unpack("<I", struct.pack("<f", float(x)))[0]
    except OverflowError:
        return struct.unpack("<I", struct.pack("<f", math.copysign(math.inf, x)))[0]


def int_to_f32_word(x: int) -> int:
    """An integer rounded once to binary32 (exact for any size, ties to even)."""
    m = abs(x)
    shift = max(0, m.bit_length() - 24)
    q, r = divmod(m, 1 << shift)
    if shift and (r > (1 << (shift - 1)) or (r == (1 << (shift - 1)) and q & 1)):
        q += 1
    value = math.inf if (q << shift).bit_length() > 128 else math.ldexp(float(q), shift)
    return f32_word(-value if x < 0 else value)


@dataclass(frozen=True)
class Val:
    reg: int
    type: str


@dataclass
class Form:
    buffer: int
    dtype: str
    base: int
    coef: tuple


@dataclass
class Program:
    """A compiled pointwise program (the plan's ``params["program"]``)."""
    code: list = field(default_factory=list)       # (op, dst, a, b, c, aux)
    consts: list = field(default_factory=list)     # 32-bit words
    forms: list = field(default_factory=list)      # Form
    buffers: list = field(default_factory=list)    # buffer names by slot
    extents: tuple = ()
    n_regs: int = 0
    sizes: list = field(default_factory=list)      # elements of each buffer slot
    loops: list = field(default_factory=list)      # extents of the runtime loops (serial programs)

    def to_json(self) -> dict:
        return {"code": [list(c) for c in self.code], "consts": list(self.consts),
                "forms": [{"buffer": f.buffer, "dtype": f.dtype, "base": f.base, "coef": list(f.coef)}
                          for f in self.forms],
                "buffers": list(self.buffers), "extents": list(self.extents), "n_regs": self.n_regs,
                "sizes": list(self.sizes), "loops": list(self.loops)}


class PointwiseCompiler:
    """Lowers one pointwise Tile body to register operations (see the module docstring)."""

    def __init__(self, pkg: KernelPackage, tile: Node):
        self.setup(pkg, [a.name for a in tile.axes], tuple(static_extent(a.extent) for a in tile.axes))

    def setup(self, pkg: KernelPackage, axes: list, extents: tuple) -> None:
        self.pkg = pkg
        self.axes = axes
        self.extents = extents
        if not 1 <= len(self.axes) <= MAX_AXES:
            raise CompileError("pointwise Tiles take one to four axes")
        if any(e <= 0 for e in self.extents):
            raise CompileError("pointwise Tile with an empty axis")
        self.code: list = []          # (op, dst, a, b, c, aux) with virtual registers
        self.consts: dict = {}
        self.forms: list = []
        self.form_index: dict = {}
        self.slots: dict = {}
        self.env: dict = {}
        self.nvreg = 0
        self.writes: list = []        # (buffer, form index) for coverage

    # ------------------------------------------------------------ emission
    def new(self, dt: str) -> Val:
        self.nvreg += 1
        return Val(self.nvreg - 1, dt)

    _IMPURE = ("LD_", "ST_", "LDX_", "STX_", "SHFL_XOR", "MMA_", "PARTIAL", "PARTNER", "SETP", "LOOP")

    def emit(self, op: str, dt: str | None, *srcs: Val, aux: int = 0) -> Val | None:
        # a pure operation on SSA values already computed is reused (fixed
        # registers are mutable, so operations reading them are not)
        key = None
        if dt is not None and not op.startswith(self._IMPURE) and all(s.reg >= 0 for s in srcs):
            key = (op, dt, tuple(s.reg for s in srcs), aux)
            memo = self.__dict__.setdefault("_memo", {})
            if key in memo:
                return memo[key]
        dst = self.new(dt) if dt is not None else None
        regs = [s.reg for s in srcs] + [0] * (3 - len(srcs))
        self.code.append((OP[op], dst.reg if dst else 0, *regs, aux, len(srcs), dst is not None))
        if key is not None:
            self._memo[key] = dst
        return dst

    def const_word(self, word: int, dt: str) -> Val:
        if word not in self.consts:
            if len(self.consts) >= MAX_CONST:
                raise CompileError("pointwise program has too many constants")
            self.consts[word] = len(self.consts)
        return self.emit("CONST", dt, aux=self.consts[word])

    # ------------------------------------------------------------ values
    def literal(self, x, dt: str = "s32") -> Val:
        dt = vm_type(dt)
        if dt == "f32":
            word = int_to_f32_word(x) if isinstance(x, int) and not isinstance(x, bool) else f32_word(x)
            return self.const_word(word, "f32")
        if dt in ("f16", "bf16"):
            return self.convert(self.literal(x, "f32"), dt)
        if dt == "pred":
            return self.const_word(1 if x else 0, "pred")
        number = int(x) % (1 << 32)
        return self.const_word(number, "s32")

    def convert(self, v: Val, dt: str) -> Val:
        dt = vm_type(dt)
        s = v.type
        if s == dt:
            return v
        if dt == "pred":
            return self.compare("ne", v, self.literal(0, s))
        if s == "pred":
            if dt == "s32":
                return self.emit("SEL", "s32", v, self.literal(1, "s32"), self.literal(0, "s32"))
            one = self.literal(1.0, "f32")
            zero = self.literal(0.0, "f32")
            return Val(self.emit("SEL", "f32", v, one, zero).reg, dt)   # 1 and 0 are exact in every float type
        if s in _FLOATS and dt in _FLOATS:
            if dt == "f32":
                return Val(v.reg, "f32")                                 # widening is exact
            return self.emit("RND_F16" if dt == "f16" else "RND_BF16", dt, v)
        if s in _FLOATS and dt == "s32":
            return self.emit("F2I", "s32", v)                            # cvt.rzi.s32
        if s == "s32":
            return self.emit({"f32": "I2F", "f16": "I2H", "bf16": "I2BF"}[dt], dt, v)
        raise CompileError(f"conversion {s} -> {dt} is not supported")

    @staticmethod
    def common_type(a: str, b: str) -> str:
        for t in ("f32", "f16", "bf16"):
            if t in (a, b):
                return t
        if a == b == "pred":
            return "pred"
        return "s32"

    def compare(self, op: str, a: Val, b: Val) -> Val:
        dt = self.common_type(a.type, b.type)
        if dt == "bf16":
            dt = "f32"                 # exact expansion preserves every value
        a, b = self.convert(a, dt), self.convert(b, dt)
        if dt == "pred":
            dt = "s32"
            a, b = Val(a.reg, "s32"), Val(b.reg, "s32")
        prefix = "F" if dt in _FLOATS else "I"
        return self.emit(prefix + op.upper(), "pred", a, b)     # FNE is unordered (true for NaN)

    def binary(self, op: str, a: Val, b: Val, dt: str | None = None) -> Val:
        if op in ("&&", "||"):
            return self.emit("PAND" if op == "&&" else "POR", "pred", self.convert(a, "pred"),
                             self.convert(b, "pred"))
        cmp = {"<": "lt", "<=": "le", ">": "gt", ">=": "ge", "==": "eq", "!=": "ne"}
        if op in cmp:
            return self.compare(cmp[op], a, b)
        if op in ("<<", ">>") and dt is None:
            if a.type not in ("s32", "pred") or b.type not in ("s32", "pred"):
                raise CompileError(f"shift operator {op!r} requires integer operands")
            dt = "s32"
        dt = dt or self.common_type(a.type, b.type)
        if dt == "pred":
            dt = "s32"
        if dt in _FLOATS and op not in ("+", "-", "*", "/"):
            raise CompileError(f"binary operator {op!r} is unsupported for {dt} operands")
        if dt in ("f16", "bf16"):
            return self.convert(self.binary(op, self.convert(self.convert(a, dt), "f32"),
                                            self.convert(self.convert(b, dt), "f32")), dt)
        a, b = self.convert(a, dt), self.convert(b, dt)
        if dt == "f32":
            return self.emit({"+": "FADD", "-": "FSUB", "*": "FMUL", "/": "FDIV"}[op], "f32", a, b)
        ops = {"+": "IADD", "-": "ISUB", "*": "IMUL", "/": "IDIV", "%": "IREM", "&": "IAND", "|": "IOR",
               "^": "IXOR", "<<": "ISHL", ">>": "ISHR"}
        if op not in ops:
            raise CompileError(f"binary operator {op!r} is not supported")
        return self.emit(ops[op], "s32", a, b)

    def select(self, p: Val, a: Val, b: Val, dt: str | None = None) -> Val:
        dt = dt or self.common_type(a.type, b.type)
        if dt == "pred":
            r = self.select(p, self.convert(a, "s32"), self.convert(b, "s32"))
            return self.convert(r, "pred")
        a, b = self.convert(a, dt), self.convert(b, dt)
        return self.emit("SEL", dt, self.convert(p, "pred"), a, b)

    # ------------------------------------------------------------ operations
    ALIASES = {"sum": "add", "prod": "multiply", "sub": "subtract", "mul": "multiply", "neg": "negative",
               "exp_fast": "exp", "true_divide": "divide", "amax": "maximum", "max": "maximum",
               "min": "minimum", "absolute": "abs", "pow": "power"}
    UNARY_ANY = ("copy", "pad", "logical_not")
    COMPARE = {"equal": "eq", "not_equal": "ne", "less": "lt", "less_equal": "le", "greater": "gt",
               "greater_equal": "ge"}

    def operation(self, name: str, args: list, dt: str) -> Val:
        dt = vm_type(dt)
        name = self.ALIASES.get(name, name)
        if name in ("copy", "pad"):
            return self.convert(args[0], dt)
        if name == "bitcast":
            src = args[0]
            if {src.type, dt} - {"f32", "s32"}:
                raise CompileError(f"bitcast {src.type} -> {dt} is not supported")
            return Val(self.emit("MOV", dt, src).reg, dt) if src.type != dt else src
        if name == "where":
            return self.select(args[0], args[1], args[2], dt)
        if name in self.COMPARE:
            return self.convert(self.compare(self.COMPARE[name], args[0], args[1]), dt)
        if name == "logical_not" or (name == "bitwise_not" and dt in ("f32", "pred")):
            return self.convert(self.compare("eq", args[0], self.literal(0, args[0].type)), dt)
        if name in ("logical_and", "logical_or") or (name in ("bitwise_and", "bitwise_or")
                                                     and dt in ("f32", "pred")):
            return self.convert(self.binary("&&" if name.endswith("and") else "||", *args), dt)
        if dt in ("f16", "bf16"):
            return self.convert(self.operation(name, [self.convert(a, "f32") for a in args], "f32"), dt)
        if dt == "pred":
            raise CompileError(f"elementwise {name!r} is unsupported for pred")
        args = [self.convert(a, dt) for a in args]
        binary = {"add": "+", "subtract": "-", "multiply": "*", "divide": "/", "bitwise_and": "&",
                  "bitwise_or": "|", "bitwise_xor": "^", "left_shift": "<<", "right_shift": ">>"}
        if dt == "s32":
            return self.int_operation(name, args, binary)
        if name == "floor_divide":
            return self.emit("FFLOOR", "f32", self.binary("/", *args))
        if name in ("mod", "remainder"):
            # floor remainder: the exact |x| mod |y| with x's sign, then y added
            # when the signs differ, a zero result taking y's sign; NaN for a
            # non-finite x, a NaN or zero y (ptx_backend.py:840-892)
            return self.emit("FREM", "f32", *args)
        if name in binary:
            return self.binary(binary[name], *args, dt="f32")
        x = args[0]
        simple = {"maximum": "FMAX", "fmax": "FMAX", "minimum": "FMIN", "fmin": "FMIN", "negative": "FNEG",
                  "abs": "FABS", "sqrt": "FSQRT", "floor": "FFLOOR", "ceil": "FCEIL", "trunc": "FTRUNC",
                  "rint": "FRINT", "fma": "FFMA"}
        if name in simple:
            return self.emit(simple[name], "f32", *args)
        if name == "square":
            return self.binary("*", x, x)
        if name == "reciprocal":
            return self.binary("/", self.literal(1, "f32"), x)
        if name == "rsqrt":
            return self.binary("/", self.literal(1, "f32"), self.emit("FSQRT", "f32", x))
        if name == "relu":
            return self.emit("FMAX", "f32", x, self.literal(0, "f32"))
        if name in ("exp", "exp2"):
            y = x if name == "exp2" else self.binary("*", x, self.literal(math.log2(math.e), "f32"))
            return self.emit("FEX2", "f32", y)
        if name in ("log", "log2", "log10"):
            y = self.emit("FLG2", "f32", x)
            if name == "log2":
                return y
            return self.binary("*", y, self.literal(math.log(2) if name == "log" else math.log10(2), "f32"))
        if name == "sin":
            r = self.emit("FSIN", "f32", x)
            small = self.compare("lt", self.emit("FABS", "f32", x), self.literal(2.0 ** -12, "f32"))
            return self.select(small, x, r, "f32")
        if name == "cos":
            return self.emit("FCOS", "f32", x)
        if name == "tanh":
            return self.tanh(x)
        if name == "erf":
            return self.erf(x)
        if name == "gelu":
            gate = self.erf(self.binary("/", x, self.literal(math.sqrt(2.0), "f32")))
            return self.binary("*", self.binary("*", self.literal(0.5, "f32"), x),
                               self.binary("+", self.literal(1.0, "f32"), gate))
        if name == "gelu_tanh":
            cube = self.binary("*", self.binary("*", x, x), x)
            inner = self.binary("+", x, self.binary("*", self.literal(0.044715, "f32"), cube))
            gate = self.tanh(self.binary("*", self.literal(math.sqrt(2.0 / math.pi), "f32"), inner))
            return self.binary("*", self.binary("*", self.literal(0.5, "f32"), x),
                               self.binary("+", self.literal(1.0, "f32"), gate))
        if name in ("sigmoid", "silu"):
            den = self.binary("+", self.literal(1, "f32"), self.operation("exp", [self.emit("FNEG", "f32", x)], "f32"))
            return self.binary("/", x if name == "silu" else self.literal(1, "f32"), den)
        raise CompileError(f"elementwise {name!r} is not supported in pointwise programs")

    def int_operation(self, name: str, args: list, binary: dict) -> Val:
        if name in binary:
            return self.binary(binary[name], *args, dt="s32")
        a = args[0]
        if name in ("maximum", "fmax"):
            return self.emit("IMAX", "s32", *args)
        if name in ("minimum", "fmin"):
            return self.emit("IMIN", "s32", *args)
        if name == "negative":
            return self.emit("INEG", "s32", a)
        if name == "abs":
            return self.emit("IABS", "s32", a)
        if name == "square":
            return self.binary("*", a, a, dt="s32")
        if name == "bitwise_not":
            return self.emit("INOT", "s32", a)
        if name == "bitwise_count":
            return self.emit("IPOPC", "s32", self.emit("IABS", "s32", a))
        if name == "relu":
            return self.emit("IMAX", "s32", a, self.literal(0, "s32"))
        if name in ("floor_divide", "mod", "remainder"):
            b = args[1]
            q = self.binary("/", a, b, dt="s32")
            rem = self.binary("%", a, b, dt="s32")
            differ = self.compare("lt", self.binary("^", a, b, dt="s32"), self.literal(0, "s32"))
            fix = self.binary("&&", self.compare("ne", rem, self.literal(0, "s32")), differ)
            if name == "floor_divide":
                return self.binary("-", q, self.convert(fix, "s32"), dt="s32")
            return self.select(fix, self.binary("+", rem, b, dt="s32"), rem)
        raise CompileError(f"elementwise {name!r} is not supported for s32")

    def fma(self, a: Val, b: Val, c: Val) -> Val:
        return self.emit("FFMA", "f32", a, b, c)

    def tanh(self, x: Val) -> Val:
        """Odd Taylor polynomial for |x| <= 1/4, else (1 - e^{-2|x|}) / (1 + e^{-2|x|}), sign of x."""
        ax = self.emit("FABS", "f32", x)
        z = self.binary("*", x, x)
        poly = self.literal(-1382 / 155925, "f32")
        for coefficient in (62 / 2835, -17 / 315, 2 / 15, -1 / 3):
            poly = self.fma(poly, z, self.literal(coefficient, "f32"))
        small = self.emit("FCOPYSIGN", "f32", x, self.fma(self.binary("*", x, z), poly, x))
        tail = self.operation("exp", [self.binary("*", self.literal(-2, "f32"), ax)], "f32")
        magnitude = self.binary("/", self.binary("-", self.literal(1, "f32"), tail),
                                self.binary("+", self.literal(1, "f32"), tail))
        large = self.emit("FCOPYSIGN", "f32", x, magnitude)
        return self.select(self.compare("le", ax, self.literal(0.25, "f32")), small, large, "f32")

    def erf(self, x: Val) -> Val:
        """Abramowitz and Stegun 7.1.26, every step rounded separately, sign of x."""
        ax = self.emit("FABS", "f32", x)
        t = self.binary("/", self.literal(1, "f32"),
                        self.binary("+", self.literal(1, "f32"),
                                    self.binary("*", self.literal(0.3275911, "f32"), ax)))
        poly = self.literal(1.061405429, "f32")
        for coefficient in (-1.453152027, 1.421413741, -0.284496736, 0.254829592):
            poly = self.binary("+", self.binary("*", poly, t), self.literal(coefficient, "f32"))
        tail = self.binary("*", self.binary("*", poly, t),
                           self.operation("exp", [self.emit("FNEG", "f32", self.binary("*", ax, ax))], "f32"))
        return self.emit("FCOPYSIGN", "f32", x, self.binary("-", self.literal(1, "f32"), tail))

    # ------------------------------------------------------------ expressions and statements
    def lookup(self, name: str) -> Val:
        if name not in self.env:
            raise CompileError(f"unbound IR value {name!r}")
        return self.env[name]

    def expr(self, e) -> Val:
        if isinstance(e, bool):
            return self.literal(e, "pred")
        if isinstance(e, int):
            return self.literal(e, "s32")
        if isinstance(e, float):
            return self.literal(e, "f32")
        if isinstance(e, str):
            return self.lookup(e)
        if not isinstance(e, Node):
            raise CompileError(f"unsupported expression {e!r}")
        k = e.kind
        if k == "Var":
            if e.name not in self.env and e.name in self.axes:
                # a tile coordinate as a value: s32, as the reference binds its axes
                return self.emit("COORD", "s32", aux=self.axes.index(e.name))
            return self.lookup(e.name)
        if k == "Literal":
            return self.literal(e.value, e.get("dtype") or ("f32" if isinstance(e.value, float) else "s32"))
        if k == "BinaryExpr":
            return self.binary(e.op, self.expr(e.left), self.expr(e.right))
        if k == "CastExpr":
            return self.convert(self.expr(e.get("expr", e.get("value"))), e.dtype)
        if k == "FuncCallExpr":
            args = [self.expr(a) for a in e.args]
            return self.operation(e.name, args, args[0].type if args else "f32")
        if k == "TernaryExpr":
            p = self.convert(self.expr(e.cond), "pred")
            a, b = self.expr(e.if_true), self.expr(e.if_false)
            return self.select(p, a, b, self.common_type(a.type, b.type))
        raise CompileError(f"unsupported expression {k}")

    def assign_type(self, name: str, args: list) -> str:
        if args and all(a.type == args[0].type for a in args):
            return args[0].type
        return "f32"

    def affine(self, e) -> dict:
        """{axis: coefficient, 1: constant} of an index expression, or CompileError."""
        if isinstance(e, bool):
            raise CompileError("boolean index")
        if isinstance(e, int):
            return {1: e}
        if isinstance(e, Node):
            if e.kind == "Literal" and isinstance(e.value, int) and not isinstance(e.value, bool):
                return {1: e.value}
            if e.kind == "Var" and e.name in self.axes:
                return {e.name: 1}
            if e.kind == "BinaryExpr" and e.op in ("+", "-", "*"):
                l, r = self.affine(e.left), self.affine(e.right)
                if e.op == "*":
                    if set(l) == {1}:
                        return {k: v * l[1] for k, v in r.items()}
                    if set(r) == {1}:
                        return {k: v * r[1] for k, v in l.items()}
                    raise CompileError("non-affine index product")
                sign = 1 if e.op == "+" else -1
                out = dict(l)
                for k, v in r.items():
                    out[k] = out.get(k, 0) + sign * v
                return out
        raise CompileError(f"pointwise index {e!r} is not affine in the tile axes")

    def form(self, buffer: str, index: tuple, lane: int) -> int:
        buf = self.pkg.buffers.get(buffer)
        if buf is None:
            raise CompileError(f"unknown buffer {buffer}")
        shape = tuple(buf.shape) or (1,)
        total: dict = {}
        strides = [1] * len(index) if len(index) == 1 or (len(index) > 1 and len(index) != len(shape)) else \
            [math.prod(shape[d + 1:]) for d in range(len(index))]
        try:
            terms = [(self.affine(i), st) for i, st in zip(index, strides)]
        except CompileError:
            # a row-major split of one axis (x[a // c, a % c]) flattens back to the axis
            terms = [(self.flat_affine(index, strides), 1)]
        for aff, stride in terms:
            for k, v in aff.items():
                total[k] = total.get(k, 0) + v * stride
        base = total.pop(1, 0) + lane
        coef = tuple(total.get(a, 0) for a in self.axes)
        size = math.prod(shape)
        lo = base + sum(min(0, c * (e - 1)) for c, e in zip(coef, self.extents))
        hi = base + sum(max(0, c * (e - 1)) for c, e in zip(coef, self.extents))
        if lo < 0 or hi >= size:
            raise CompileError(f"index of {buffer} leaves the buffer")
        if buffer not in self.slots:
            if len(self.slots) >= MAX_BUFFERS:
                raise CompileError("pointwise program uses too many buffers")
            self.slots[buffer] = len(self.slots)
        key = (buffer, base, coef)
        if key not in self.form_index:
            if len(self.forms) >= MAX_FORMS:
                raise CompileError("pointwise program has too many distinct indices")
            self.form_index[key] = len(self.forms)
            self.forms.append(Form(self.slots[buffer], vm_type(buf.dtype), base, coef))
        return self.form_index[key]

    def flat_affine(self, index: tuple, strides: list) -> dict:
        """The flattened offset of an index with div / mod terms, when the terms
        recombine (c * (x // c) + x % c == x) into an affine form of the axes."""
        from .recognize import _aff, _aff_add, _aff_scale, _Eval
        ev = _Eval(self.pkg)
        total = _aff({})
        for i, stride in zip(index, strides):
            if not isinstance(i, Node):
                raise CompileError(f"pointwise index {i!r} is not affine in the tile axes")
            total = _aff_add(total, _aff_scale(ev.index(i), stride))
        active = getattr(self, "active", {})
        out: dict = {}
        for term, coef in total:
            if term == 1:
                out[1] = out.get(1, 0) + coef
            elif isinstance(term, str) and term in active:
                out[active[term]] = out.get(active[term], 0) + coef
            elif isinstance(term, str) and term in self.axes:
                out[term] = out.get(term, 0) + coef
            else:
                raise CompileError("pointwise index is not affine in the tile axes")
        return out

    def statement(self, s: Node) -> None:
        k = s.kind
        if k == "Load":
            buf = self.pkg.buffers.get(s.input)
            if buf is None:
                raise CompileError(f"Load from unknown buffer {s.input}")
            dt = vm_type(buf.dtype)
            for lane, name in enumerate(s.names):
                f = self.form(s.input, tuple(s.index), lane)
                self.env[name] = self.emit("LD_" + _STORAGE[dt], dt, aux=f)
        elif k == "Let":
            v = self.expr(s.value)
            self.env[s.name] = self.convert(v, s.get("dtype") or v.type)
        elif k == "Assign":
            op = s.op.name if isinstance(s.op, Node) else str(s.op)
            args = [self.lookup(a) if isinstance(a, str) else self.expr(a) for a in s.args]
            dt = s.get("dtype")
            self.env[s.name] = self.operation(op, args, vm_type(dt) if dt is not None else
                                              self.assign_type(op, args))
        elif k == "Select":
            branches = list(s.branches)
            if not branches:
                raise CompileError("Select requires at least one branch")
            value = self.convert(self.lookup(branches[-1].value), "f32")
            for br in reversed(branches[:-1]):
                value = self.select(self.expr(br.select), self.convert(self.lookup(br.value), "f32"), value)
            self.env[s.name] = value
        elif k == "Write":
            buf = self.pkg.buffers.get(s.output)
            if buf is None or buf.role != "output":
                raise CompileError("pointwise programs write the kernel's outputs only")
            if s.get("atomic") or s.get("swizzle", "NONE") not in (None, "NONE"):
                raise CompileError("pointwise writes are plain stores")
            dt = vm_type(buf.dtype)
            if dt == "pred":
                raise CompileError("predicate outputs are not supported")
            for lane, name in enumerate(s.values):
                f = self.form(s.output, tuple(s.index), lane)
                v = self.convert(self.lookup(name), dt)
                self.emit("ST_" + _STORAGE[dt], None, v, aux=f)
                self.writes.append((s.output, f))
        else:
            raise CompileError(f"{k} is not part of a pointwise program")

    # ------------------------------------------------------------ finishing
    def allocate(self, extend: dict | None = None) -> list:
        """Map virtual registers to physical ones (linear scan).

        Register ids >= 0 are virtual; -1 - p names fixed physical register p
        (the fragment registers of lane programs and the accumulators of
        serial programs, below ``n_fixed``), which virtual registers never
        share.  ``extend`` keeps registers allocated up to a later pc (values
        a loop's back edge reads again).
        """
        base = getattr(self, "n_fixed", 0)
        last: dict = {}
        for pc, (op, dst, a, b, c, aux, nsrc, has_dst) in enumerate(self.code):
            for r in (a, b, c)[:nsrc]:
                if r >= 0:
                    last[r] = pc
        for r, pc in (extend or {}).items():
            last[r] = max(last.get(r, pc), pc)
        free: list = []
        phys: dict = {}
        top = base
        out = []
        for pc, (op, dst, a, b, c, aux, nsrc, has_dst) in enumerate(self.code):
            srcs = [-1 - r if r < 0 else phys[r] for r in (a, b, c)[:nsrc]]
            for r in set((a, b, c)[:nsrc]):
                if r >= 0 and last.get(r) == pc:
                    free.append(phys[r])
            d = 0
            if has_dst:
                if dst < 0:
                    d = -1 - dst
                else:
                    if free:
                        d = free.pop()
                    else:
                        d = top
                        top += 1
                    phys[dst] = d
                    if dst not in last:
                        free.append(d)
            srcs += [0] * (3 - len(srcs))
            out.append((op, d, *srcs, aux))
        if top > MAX_REGS:
            raise CompileError(f"program needs {top} registers (at most {MAX_REGS})")
        return out, top

    def coverage(self) -> str:
        outs = {b for b, _ in self.writes}
        if len(outs) != 1:
            raise CompileError("pointwise programs must write one output")
        out = outs.pop()
        size = math.prod(self.pkg.buffers[out].shape or (1,))
        points = math.prod(self.extents)
        if points * len(self.writes) != size:
            raise CompileError(f"writes cover {points * len(self.writes)} elements of {out} ({size})")
        forms = [self.forms[f] for _, f in self.writes]
        if points * len(forms) <= (1 << 24):
            grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for e in self.extents], indexing="ij")
            seen = np.zeros(size, np.int64)
            for f in forms:
                flat = f.base + sum(c * g for c, g in zip(f.coef, grids))
                np.add.at(seen, np.asarray(flat).ravel(), 1)
            if np.any(seen != 1):
                raise CompileError("pointwise writes do not cover the output exactly once")
            return out
        # Large tiles: the writes must share one stride pattern and their
        # offsets must be an arithmetic run; then the (stride, extent) pairs of
        # the axes and of the run must number the output in mixed radix.
        if len({f.coef for f in forms}) != 1:
            raise CompileError("large pointwise tiles must write with one stride pattern")
        bases = sorted(f.base for f in forms)
        run = bases[1] - bases[0] if len(bases) > 1 else 1
        if bases != [bases[0] + run * j for j in range(len(bases))] or bases[0] != 0:
            raise CompileError("pointwise write offsets are not a dense run from element 0")
        dims = sorted([(c, e) for c, e in zip(forms[0].coef, self.extents) if e > 1] + [(run, len(bases))])
        step = 1
        for stride, extent in dims:
            if extent == 1:
                continue
            if stride != step:
                raise CompileError("pointwise writes do not cover the output densely")
            step *= extent
        return out

    def compile(self, body: tuple) -> Program:
        for s in body:
            self.statement(s)
        if not self.writes:
            raise CompileError("pointwise program writes nothing")
        self.coverage()
        code, nregs = self.allocate()
        if len(code) > MAX_CODE:
            raise CompileError(f"pointwise program has {len(code)} operations (at most {MAX_CODE})")
        consts = [0] * len(self.consts)
        for word, i in self.consts.items():
            consts[i] = word
        return Program(code, consts, self.forms, list(self.slots), self.extents, nregs,
                       [math.prod(self.pkg.buffers[b].shape or (1,)) for b in self.slots])


def compile_pointwise(pkg: KernelPackage, tile: Node):
    """Plan of a pointwise Tile compiled to a register program."""
    from .recognize import _plan
    comp = PointwiseCompiler(pkg, tile)
    prog = comp.compile(tuple(tile.body))
    out = {b for b, _ in comp.writes}.pop()
    bind = {f"buf{i}": name for i, name in enumerate(prog.buffers)}
    return _plan(pkg, "pointwise", "lc_pointwise", bind,
                 {"program": prog.to_json(), "out": out, "points": math.prod(prog.extents)},
                 {name: pkg.buffers[name].dtype for name in prog.buffers})
