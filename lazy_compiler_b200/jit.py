"""Native block programs: a block program's register code translated to CUDA
C and compiled for sm_100a with NVRTC, so it runs at the speed of a
hand-written kernel instead of through the interpreter.

The translation is one C statement per operation, with the program's
registers as local variables (the interpreter keeps them in an indexed
array, which lives in local memory), branches and loops as gotos, and every
operation's arithmetic exactly the interpreter's (csrc/pointwise.cu,
``exec_range``): the same intrinsics, the same clamped loads, bounds-checked
stores and bounded loops, so the native kernel computes bit for bit what
the interpreter computes.  The library validates the program (the same
checks as ``lc_blockprog``) before it launches the compiled kernel
(``lc_jit_blockprog``).

Programs with an operation this translation does not cover run through the
interpreter; so does every program when NVRTC is unavailable or when
``LC_JIT=0``.
"""
from __future__ import annotations

import hashlib
import os
import re
import threading

from .pointwise import OPCODES

KERNEL = "lc_jit_block"
POINT_KERNEL = "lc_jit_point"
ROWS_KERNEL = "lc_jit_rows"

_PREAMBLE = r"""
typedef unsigned int u32;
typedef long long i64;
struct JitArgs { void *buffers[16]; i64 blocks; };
__device__ __forceinline__ float f(u32 w) { return __uint_as_float(w); }
__device__ __forceinline__ u32 w(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float ex2a(float x) { float y; asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ float lg2a(float x) { float y; asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ float sina(float x) { float y; asm("sin.approx.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ float cosa(float x) { float y; asm("cos.approx.f32 %0, %1;" : "=f"(y) : "f"(x)); return y; }
__device__ __forceinline__ unsigned short to_h(float x) { unsigned short h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(x)); return h; }
__device__ __forceinline__ float from_h(unsigned short h) { float x; asm("cvt.f32.f16 %0, %1;" : "=f"(x) : "h"(h)); return x; }
__device__ __forceinline__ unsigned short to_bf(float x) { unsigned short h; asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(h) : "f"(x)); return h; }
__device__ __forceinline__ float from_bf(unsigned short h) { return __uint_as_float(((u32)h) << 16); }
__device__ __forceinline__ float i2h(int v) { unsigned short h; asm("cvt.rn.f16.s32 %0, %1;" : "=h"(h) : "r"(v)); return from_h(h); }
__device__ __forceinline__ i64 clampi(i64 at, i64 size) { return at < 0 ? 0 : (at >= size ? size - 1 : at); }
__device__ __forceinline__ float frem_floor(float xv, float yv) {
  float rv = __int_as_float(0x7fc00000);
  if (isfinite(xv) && !isnan(yv) && yv != 0.0f) {
    rv = fmodf(xv, yv);
    if (rv != 0.0f && ((xv < 0.0f) != (yv < 0.0f))) rv = __fadd_rn(rv, yv);
    if (rv == 0.0f) rv = copysignf(0.0f, yv);
  }
  return rv;
}
"""

_UNARY_F = {"FNEG": "A ^ 0x80000000u", "FABS": "A & 0x7fffffffu", "FSQRT": "w(__fsqrt_rn(f(A)))",
            "FFLOOR": "w(floorf(f(A)))", "FCEIL": "w(ceilf(f(A)))", "FTRUNC": "w(truncf(f(A)))",
            "FRINT": "w(rintf(f(A)))", "FEX2": "w(ex2a(f(A)))", "FLG2": "w(lg2a(f(A)))", "FSIN": "w(sina(f(A)))",
            "FCOS": "w(cosa(f(A)))", "RND_F16": "w(from_h(to_h(f(A))))", "RND_BF16": "w(from_bf(to_bf(f(A))))",
            "F2I": "(u32)__float2int_rz(f(A))", "I2F": "w(__int2float_rn((int)A))", "I2H": "w(i2h((int)A))",
            "INOT": "~A", "INEG": "0u - A", "IABS": "((int)A < 0 ? 0u - A : A)", "IPOPC": "(u32)__popc(A)",
            "MOV": "A"}
_BINARY = {"FADD": "w(__fadd_rn(f(A), f(B)))", "FSUB": "w(__fsub_rn(f(A), f(B)))",
           "FMUL": "w(__fmul_rn(f(A), f(B)))", "FDIV": "w(__fdiv_rn(f(A), f(B)))",
           "FMAX": "w(fmaxf(f(A), f(B)))", "FMIN": "w(fminf(f(A), f(B)))",
           "FCOPYSIGN": "((B & 0x7fffffffu) | (A & 0x80000000u))",
           "IADD": "A + B", "ISUB": "A - B", "IMUL": "A * B",
           "IDIV": "((int)B == 0 ? 0u : ((int)B == -1 ? 0u - A : (u32)((int)A / (int)B)))",
           "IREM": "(((int)B == 0 || (int)B == -1) ? ((int)B == 0 ? A : 0u) : (u32)((int)A % (int)B))",
           "ISHL": "(B >= 32u ? 0u : A << B)", "ISHR": "(u32)((int)A >> (B >= 32u ? 31u : B))",
           "IAND": "A & B", "IOR": "A | B", "IXOR": "A ^ B", "IMAX": "(u32)max((int)A, (int)B)",
           "IMIN": "(u32)min((int)A, (int)B)", "FEQ": "(u32)(f(A) == f(B))", "FNE": "(u32)!(f(A) == f(B))",
           "FLT": "(u32)(f(A) < f(B))", "FLE": "(u32)(f(A) <= f(B))", "FGT": "(u32)(f(A) > f(B))",
           "FGE": "(u32)(f(A) >= f(B))", "IEQ": "(u32)((int)A == (int)B)", "INE": "(u32)((int)A != (int)B)",
           "ILT": "(u32)((int)A < (int)B)", "ILE": "(u32)((int)A <= (int)B)", "IGT": "(u32)((int)A > (int)B)",
           "IGE": "(u32)((int)A >= (int)B)", "PAND": "(u32)((A != 0u) & (B != 0u))",
           "POR": "(u32)((A != 0u) | (B != 0u))", "FREM": "w(frem_floor(f(A), f(B)))"}
_TERNARY = {"FFMA": "w(__fmaf_rn(f(A), f(B), f(C)))", "SEL": "(A != 0u ? B : C)"}


class Untranslatable(Exception):
    """The program uses an operation the translation does not cover."""


def block_source(prog: dict, layout: dict) -> str:
    """CUDA C of a block program (raises Untranslatable)."""
    code = prog["code"]
    n_regs = max(1, prog["n_regs"])
    extents = [int(e) for e in prog["extents"]]
    loops = [int(e) for e in prog.get("loops", [])]
    n_axes = len(extents)
    nb, threads = layout["n_block_axes"], layout["threads"]
    sizes = [int(s) for s in prog["sizes"]]
    consts = [int(c) & 0xFFFFFFFF for c in prog["consts"]]
    smem = layout["smem"]
    lines = [f"extern \"C\" __global__ void __launch_bounds__({threads}) {KERNEL}(const __grid_constant__ JitArgs p) {{",
             "  extern __shared__ u32 smem[];",
             "  // lanes of this warp that exist (a CTA may be one partial warp)",
             "  const u32 lanes = blockDim.x - (threadIdx.x & ~31u) >= 32u ? 0xffffffffu"
             " : ((1u << (blockDim.x - (threadIdx.x & ~31u))) - 1u);"]
    lines.append("  u32 " + ", ".join(f"r{i} = 0u" for i in range(n_regs)) + ";")
    lines.append("  i64 " + ", ".join(f"x{d} = 0" for d in range(n_axes + len(loops))) + ";")
    lines.append("  for (i64 blk = blockIdx.x; blk < p.blocks; blk += gridDim.x) {")
    lines.append("    i64 rest = threadIdx.x;")
    for d in range(n_axes - 1, nb - 1, -1):
        lines.append(f"    x{d} = rest % {extents[d]}; rest /= {extents[d]};")
    lines.append("    rest = blk;")
    for d in range(nb - 1, -1, -1):
        lines.append(f"    x{d} = rest % {extents[d]}; rest /= {extents[d]};")
    lines += _statements(prog, smem)
    lines.append(f"  L{len(code)}: ;")
    lines.append("    __syncthreads();")
    lines.append("  }")
    lines.append("}")
    return _PREAMBLE + "\n".join(lines) + "\n"


def _statements(prog: dict, smem: list, begin: int = 0, end: int | None = None) -> list:
    """One labelled C statement per operation of [begin, end) (raises Untranslatable)."""
    code = prog["code"]
    n_axes = len(prog["extents"])
    loops = [int(e) for e in prog.get("loops", [])]
    sizes = [int(x) for x in prog["sizes"]]
    consts = [int(c) & 0xFFFFFFFF for c in prog["consts"]]
    forms = prog.get("forms", [])
    lines = []
    for pc in range(begin, len(code) if end is None else end):
        op, dst, a, b, c, aux = code[pc]
        name = OPCODES[op]
        A, B, C = f"r{a}", f"r{b}", f"r{c}"

        def sub(t):
            # operand names in the templates are the single letters A, B, C
            return re.sub(r"\b([ABC])\b", lambda m: {"A": A, "B": B, "C": C}[m.group(1)], t)

        stmt = None
        if name == "CONST":
            stmt = f"r{dst} = {consts[aux]}u;"
        elif name in _UNARY_F:
            stmt = f"r{dst} = {sub(_UNARY_F[name])};"
        elif name in _BINARY:
            stmt = f"r{dst} = {sub(_BINARY[name])};"
        elif name in _TERNARY:
            stmt = f"r{dst} = {sub(_TERNARY[name])};"
        elif name == "COORD":
            stmt = f"r{dst} = (u32)x{aux};"
        elif name == "TID":
            stmt = f"r{dst} = threadIdx.x;"
        elif name.startswith("LDX_"):
            at = f"clampi((i64)(int){A}, {sizes[aux]}LL)"
            if name == "LDX_F16":
                stmt = f"r{dst} = w(from_h(((const unsigned short *)p.buffers[{aux}])[{at}]));"
            elif name == "LDX_BF16":
                stmt = f"r{dst} = w(from_bf(((const unsigned short *)p.buffers[{aux}])[{at}]));"
            else:
                stmt = f"r{dst} = ((const u32 *)p.buffers[{aux}])[{at}];"
        elif name.startswith("STX_"):
            cond = f"{C} != 0u && (i64)(int){A} >= 0 && (i64)(int){A} < {sizes[aux]}LL"
            at = f"(i64)(int){A}"
            if name == "STX_F16":
                body = f"((unsigned short *)p.buffers[{aux}])[{at}] = to_h(f({B}));"
            elif name == "STX_BF16":
                body = f"((unsigned short *)p.buffers[{aux}])[{at}] = to_bf(f({B}));"
            elif name == "STX_ADD_F32":
                body = f"atomicAdd(((float *)p.buffers[{aux}]) + {at}, f({B}));"
            else:
                body = f"((u32 *)p.buffers[{aux}])[{at}] = {B};"
            stmt = f"if ({cond}) {{ {body} }}"
        elif name == "SHFL_XOR":
            stmt = f"__syncwarp(lanes); r{dst} = __shfl_xor_sync(lanes, {A}, {aux});"
        elif name == "LDS":
            off, size = smem[aux]
            stmt = f"r{dst} = smem[{off} + clampi((i64)(int){A}, {size}LL)];"
        elif name == "STS":
            off, size = smem[aux]
            stmt = f"if ((i64)(int){A} >= 0 && (i64)(int){A} < {size}LL) smem[{off} + (int){A}] = {B};"
        elif name == "BAR":
            stmt = "__syncthreads();"
        elif name == "WSYNC":
            stmt = "__syncwarp(lanes);"
        elif name == "BRA":
            stmt = f"goto L{aux};"
        elif name == "BRZ":
            stmt = f"if ({A} == 0u) goto L{aux};"
        elif name in ("SLB", "SLE"):
            d = n_axes + (aux & 15)
            other = aux >> 4
            limit = f"min((i64)(int){B}, {loops[aux & 15]}LL)"
            if name == "SLB":
                stmt = f"x{d} = (i64)(int){A}; if (x{d} < 0 || x{d} >= {limit}) goto L{other + 1};"
            else:
                stmt = f"x{d} += ((int){A} < 1 ? 1 : (int){A}); if (x{d} < {limit}) goto L{other + 1};"
        elif name.startswith(("LD_", "ST_")):
            fm = forms[aux]
            at = " + ".join([f"{int(fm['base'])}LL"] + [f"{int(k)}LL * x{d}" for d, k in enumerate(fm["coef"]) if int(k)])
            ptr = f"p.buffers[{fm['buffer']}]"
            stmt = {"LD_F32": f"r{dst} = ((const u32 *){ptr})[{at}];",
                    "LD_S32": f"r{dst} = ((const u32 *){ptr})[{at}];",
                    "LD_F16": f"r{dst} = w(from_h(((const unsigned short *){ptr})[{at}]));",
                    "LD_BF16": f"r{dst} = w(from_bf(((const unsigned short *){ptr})[{at}]));",
                    "ST_F32": f"((u32 *){ptr})[{at}] = {A};", "ST_S32": f"((u32 *){ptr})[{at}] = {A};",
                    "ST_F16": f"((unsigned short *){ptr})[{at}] = to_h(f({A}));",
                    "ST_BF16": f"((unsigned short *){ptr})[{at}] = to_bf(f({A}));"}[name]
        elif name == "STATE":
            stmt = f"r{dst} = w(st{aux});"
        elif name == "PARTIAL":
            stmt = f"r{dst} = w(pa{aux});"
        elif name == "PARTNER":
            stmt = f"r{dst} = w(pn{aux});"
        elif name == "SETP":
            stmt = f"pa{aux} = f({A});"
        elif name in ("LOOPB", "LOOPE"):
            d = n_axes + (aux & 15)
            other = aux >> 4
            limit = f"min((i64)(int){A}, {loops[aux & 15]}LL)"
            if name == "LOOPB":
                stmt = f"x{d} = 0; if ({limit} <= 0) goto L{other + 1};"
            else:
                stmt = f"if (++x{d} < {limit}) goto L{other + 1};"
        if stmt is None:
            raise Untranslatable(name)
        lines.append(f"  L{pc}: {stmt}")
    return lines


def rows_source(prog: dict, layout: dict) -> str:
    """CUDA C of a row program: one CTA of the Tile's threads per row, the
    passes, the lane butterfly, the halving tree and the final operations
    as the interpreter's rowprog kernel runs them (raises Untranslatable)."""
    extents = [int(e) for e in prog["extents"]]
    R = len(extents) - 1
    cols = extents[R]
    n_regs = max(1, prog["n_regs"])
    n_states = len(layout["state_pass"])
    ns = max(1, n_states)
    threads = int(layout["threads"])
    L = [f"extern \"C\" __global__ void __launch_bounds__({threads}) {ROWS_KERNEL}(const __grid_constant__ JitArgs p) {{",
         f"  __shared__ float warp_part[32][{ns}];",
         f"  __shared__ float combined[{ns}];",
         "  u32 " + ", ".join(f"r{i} = 0u" for i in range(n_regs)) + ";",
         "  i64 " + ", ".join(f"x{d} = 0" for d in range(R + 1)) + ";",
         "  float " + ", ".join(f"st{k} = 0.0f, pa{k} = 0.0f, pn{k} = 0.0f" for k in range(ns)) + ";",
         "  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;",
         "  for (i64 row = blockIdx.x; row < p.blocks; row += gridDim.x) {",
         "    i64 rest = row;"]
    for d in range(R - 1, -1, -1):
        L.append(f"    x{d} = rest % {extents[d]}; rest /= {extents[d]};")
    for pss, (b, e) in enumerate(layout["passes"]):
        slots = [k for k, ps in enumerate(layout["state_pass"]) if ps == pss]
        for k in slots:
            L.append(f"    pa{k} = __uint_as_float({int(layout['state_init'][k]) & 0xFFFFFFFF}u);")
        L.append(f"    for (i64 c = threadIdx.x; c < {cols}; c += blockDim.x) {{")
        L.append(f"      x{R} = c;")
        L += ["    " + t for t in _statements(prog, [], b, e)]
        L.append(f"    }}")
        L.append(f"    x{R} = 0;")
        if not slots:
            continue
        wb, we = layout["warp"][pss]
        tb, te = layout["tree"][pss]
        L.append("    for (int o = 16; o > 0; o >>= 1) {")
        for k in slots:
            L.append(f"      pn{k} = __shfl_xor_sync(0xffffffffu, pa{k}, o);")
        L += ["    " + t for t in _statements(prog, [], wb, we)]
        L.append("    }")
        L.append("    if (lane == 0) { " + " ".join(f"warp_part[warp][{k}] = pa{k};" for k in slots) + " }")
        L.append("    __syncthreads();")
        L.append("    if (threadIdx.x == 0) {")
        L.append("      for (int d = nwarps >> 1; d > 0; d >>= 1)")
        L.append("        for (int i = 0; i < d; ++i) {")
        L.append("          " + " ".join(f"pa{k} = warp_part[i][{k}]; pn{k} = warp_part[i + d][{k}];" for k in slots))
        L += ["      " + t for t in _statements(prog, [], tb, te)]
        L.append("          " + " ".join(f"warp_part[i][{k}] = pa{k};" for k in slots))
        L.append("        }")
        L.append("      " + " ".join(f"combined[{k}] = warp_part[0][{k}];" for k in slots))
        L.append("    }")
        L.append("    __syncthreads();")
        L.append("    " + " ".join(f"st{k} = combined[{k}];" for k in slots))
        L.append("    __syncthreads();")
    fb, fe = layout["final"]
    L.append("    if (threadIdx.x == 0) {")
    L += ["    " + t for t in _statements(prog, [], fb, fe)]
    L.append("    }")
    L.append("  }")
    L.append("}")
    return _PREAMBLE + "\n".join(L) + "\n"


def point_source(prog: dict) -> str:
    """CUDA C of a pointwise or serial program: one point per thread, grid-stride
    (raises Untranslatable; lane programs, whose warps exchange registers,
    stay with the interpreter)."""
    if any(OPCODES[c[0]] in ("SHFL_XOR", "MMA_F16", "MMA_BF16", "PACK_F16X2", "PACK_BF16X2") for c in prog["code"]):
        raise Untranslatable("lane operations")
    extents = [int(e) for e in prog["extents"]]
    loops = [int(e) for e in prog.get("loops", [])]
    n_axes = len(extents)
    n_regs = max(1, prog["n_regs"])
    lines = [f"extern \"C\" __global__ void __launch_bounds__(256) {POINT_KERNEL}(const __grid_constant__ JitArgs p) {{"]
    lines.append("  u32 " + ", ".join(f"r{i} = 0u" for i in range(n_regs)) + ";")
    lines.append("  i64 " + ", ".join(f"x{d} = 0" for d in range(n_axes + len(loops))) + ";")
    lines.append("  for (i64 gid = (i64)blockIdx.x * blockDim.x + threadIdx.x; gid < p.blocks;"
                 " gid += (i64)gridDim.x * blockDim.x) {")
    lines.append("    i64 rest = gid;")
    for d in range(n_axes - 1, -1, -1):
        lines.append(f"    x{d} = rest % {extents[d]}; rest /= {extents[d]};")
    lines += _statements(prog, [])
    lines.append(f"  L{len(prog['code'])}: ;")
    lines.append("  }")
    lines.append("}")
    return _PREAMBLE + "\n".join(lines) + "\n"


_cache: dict = {}
_lock = threading.Lock()


def enabled() -> bool:
    return os.environ.get("LC_JIT", "1") != "0"


def compile_cubin(source: str) -> bytes:
    """sm_100a cubin of ``source`` (cached by the source's hash)."""
    key = hashlib.sha256(source.encode()).hexdigest()
    with _lock:
        if key in _cache:
            return _cache[key]
    from cuda.bindings import nvrtc

    err, program = nvrtc.nvrtcCreateProgram(source.encode(), b"block.cu", 0, [], [])
    if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
        raise RuntimeError(f"nvrtcCreateProgram: {err}")
    try:
        opts = [b"--gpu-architecture=sm_100a", b"--std=c++17", b"-default-device"]
        (err,) = nvrtc.nvrtcCompileProgram(program, len(opts), opts)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            _, size = nvrtc.nvrtcGetProgramLogSize(program)
            log = b" " * size
            nvrtc.nvrtcGetProgramLog(program, log)
            raise RuntimeError(f"NVRTC failed: {log.decode(errors='replace')[:2000]}")
        _, size = nvrtc.nvrtcGetCUBINSize(program)
        cubin = b" " * size
        (err,) = nvrtc.nvrtcGetCUBIN(program, cubin)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            raise RuntimeError(f"nvrtcGetCUBIN: {err}")
    finally:
        nvrtc.nvrtcDestroyProgram(program)
    with _lock:
        _cache[key] = cubin
    return cubin


def point_cubin(prog: dict) -> bytes | None:
    """The compiled native kernel of a pointwise or serial program, or None."""
    if not enabled():
        return None
    try:
        return compile_cubin(point_source(prog))
    except (Untranslatable, ImportError, RuntimeError):
        return None      # the interpreter runs it


def rows_cubin(prog: dict, layout: dict) -> bytes | None:
    """The compiled native kernel of a row program, or None (interpreter)."""
    if not enabled():
        return None
    try:
        return compile_cubin(rows_source(prog, layout))
    except (Untranslatable, ImportError, RuntimeError):
        return None      # the interpreter runs it


def block_cubin(prog: dict, layout: dict) -> bytes | None:
    """The compiled native kernel of a block program, or None (interpreter)."""
    if not enabled():
        return None
    try:
        return compile_cubin(block_source(prog, layout))
    except (Untranslatable, ImportError, RuntimeError):
        return None      # the interpreter runs it
