"""Recognition of one-warp tensor-fragment programs by exact interpretation.

The reference lowers RegFragment / LdmatrixLoad / MmaSyncPtx / FragmentRepack
/ RegStore to the per-lane registers of one warp (ptx_tensor.py:164-477),
after any shared-memory staging the program does with Load/Write fill loops
or cp.async copies (ptx_backend.py:1241-1270, 1455-1490).  This module runs
such a program once on the host, not on values but on provenance:

* every element of an A or B fragment holds the id of the buffer element it
  was gathered from, found through the same address arithmetic the
  reference emits: ``ldm`` row strides, the shared-memory XOR swizzles, the
  ldmatrix lane-to-row maps, the clamped M/N guard and the zero-filled K
  tail of global gathers;
* every C fragment holds the list of (A, B) fragment pairs multiplied into
  it;
* a FragmentRepack makes an A fragment whose elements are C elements of an
  earlier product (an intermediate matrix);
* every RegStore records, for each output element it writes, the C element,
  the epilogue and the store's flags.

The program is accepted only if every output element is written exactly
once, every written element's terms multiply A[r, k] by B[k, n] for the row
r and column n its address implies, over k = 0 .. K-1 exactly once, with
both operands rounded to the MMA type.  It then becomes one of two plans:

    out = epilogue(Q(A) Q(B) [+ bias]) [stored transposed]     op "gemm_mixed"
    out = Q(Q(X) Q(Y)) Q(Z)                                    op "gemm_chain"

Loops are unrolled, so only programs of at most ``MAX_STEPS`` interpreted
statements are taken here; large tiled GEMMs go through the structural
recogniser.  A zero-padded operand element multiplied by a non-finite one
gives NaN in the reference but counts as a zero term here (padding only
meets finite data in these programs' valid outputs).
"""
from __future__ import annotations

import math
import re
from dataclasses import dataclass, field

import numpy as np

from .ir import CompileError, KernelPackage, Node, static_extent

MAX_STEPS = 20000
SHAPE = (16, 8, 16)
_SWIZZLE_MASK = {"B32": 1, "B64": 3, "B128": 7}
_CTYPES = {"__half": "f16", "half": "f16", "__nv_bfloat16": "bf16", "float": "f32", "f16": "f16",
           "bf16": "bf16", "f32": "f32"}
_LEAF_SHIFT = 40
_LANES = np.arange(32, dtype=np.int64)


def _dt(value) -> str:
    if isinstance(value, Node):
        return str(value.get("name"))
    return str(value)


# ---------------------------------------------------------------- index arithmetic

def _tdiv(a, b):
    """C integer division (truncation toward zero) on ints or int64 arrays."""
    if np.any(np.asarray(b) == 0):
        raise CompileError("integer division by zero in an index")
    q = np.abs(a) // np.abs(b)
    out = np.where((np.asarray(a) < 0) ^ (np.asarray(b) < 0), -q, q)
    return out if out.ndim else int(out)


def _tmod(a, b):
    return a - b * _tdiv(a, b)


_BIN = {"+": lambda a, b: a + b, "-": lambda a, b: a - b, "*": lambda a, b: a * b,
        "/": _tdiv, "%": _tmod, "<<": lambda a, b: a << b, ">>": lambda a, b: a >> b,
        "&": lambda a, b: a & b, "|": lambda a, b: a | b, "^": lambda a, b: a ^ b}


def ival(e, env: dict):
    """Integer value of an index expression; per-lane values are int64 arrays of 32."""
    if isinstance(e, bool):
        raise CompileError("boolean used as an index")
    if isinstance(e, (int, np.integer)):
        return int(e)
    if isinstance(e, Node):
        if e.kind == "Literal":
            v = e.value
            if isinstance(v, bool) or not isinstance(v, int):
                raise CompileError(f"non-integer index literal {v!r}")
            return v
        if e.kind == "Var":
            if e.name not in env:
                raise CompileError(f"index variable {e.name!r} is not bound")
            return env[e.name]
        if e.kind == "BinaryExpr" and e.op in _BIN:
            return _BIN[e.op](ival(e.left, env), ival(e.right, env))
    raise CompileError(f"unsupported index expression {e!r}")


def uniform(v, what: str) -> int:
    """A value every lane agrees on (fragment operations are warp-collective)."""
    if isinstance(v, np.ndarray):
        if v.size == 0 or np.any(v != v.flat[0]):
            raise CompileError(f"{what} differs between the lanes of the warp")
        return int(v.flat[0])
    return int(v)


def swizzle(index, mode: str):
    """The reference's shared-memory XOR swizzle on element indices (ptx_backend.py:1244-1254)."""
    if mode in (None, "NONE"):
        return index
    base, _, shift = str(mode).partition("@")
    if base not in _SWIZZLE_MASK:
        raise CompileError(f"unsupported shared swizzle {mode}")
    bits = (index >> (int(shift) if shift else 6)) & _SWIZZLE_MASK[base]
    return index ^ (bits << 3)


# ---------------------------------------------------------------- program state

@dataclass
class Smem:
    name: str
    shape: tuple
    dtype: str
    align: int
    leaf: np.ndarray            # element id per physical element, -1 unset
    pending: np.ndarray         # cp.async group number not yet waited for, -1 none
    dirty: bool = False         # written since the last barrier


@dataclass
class CVal:
    """A C fragment: sum over terms of A (16 x 16 ids) times B (16 x 8 ids)."""
    terms: list = field(default_factory=list)   # (A ids, B ids, mma type)


@dataclass(eq=False)
class Virtual:
    """An intermediate made by FragmentRepack: 16 x 16 elements of two C fragments."""
    halves: tuple            # (CVal, CVal): columns 0..7 and 8..15
    dtype: str               # rounding applied to every element
    info: dict | None = None  # its place in the product it came from, once verified


@dataclass
class Fragment:
    role: str
    dtype: str
    members: list


@dataclass
class StoreRecord:
    flats: np.ndarray        # output flat index per written element
    i: np.ndarray            # fragment row (0..15)
    j: np.ndarray            # fragment column (0..7)
    cval: CVal
    epilogue: object
    atomic: bool


class FragmentInterpreter:
    """Runs a one-warp fragment program on element provenance."""

    def __init__(self, pkg: KernelPackage, tile: Node):
        self.pkg = pkg
        self.sources: list = []          # leaf source number -> buffer name or Virtual
        self.source_no: dict = {}
        self.smem: dict = {}
        self.frags: dict = {}
        self.env: dict = {}
        self.values: dict = {}           # scalar name -> per-lane leaf ids (int64[32])
        self.stores: list = []
        self.steps = 0
        self.cp_group = 0                # number of committed cp.async groups
        self.cp_open: list = []          # copies issued since the last commit
        if not is_single_warp(pkg, tile):
            raise CompileError("fragment programs must run as one 32-lane warp in one block")
        self.lane = tile.axes[0].name
        self.env[self.lane] = _LANES.copy()

    # ------------------------------------------------------------ leaves
    def src_no(self, src) -> int:
        key = id(src) if isinstance(src, Virtual) else src
        if key not in self.source_no:
            self.source_no[key] = len(self.sources)
            self.sources.append(src)
        return self.source_no[key]

    def leaf(self, src, flat):
        return (np.int64(self.src_no(src)) << _LEAF_SHIFT) | np.asarray(flat, np.int64)

    # ------------------------------------------------------------ statements
    def run(self, stmts, mask=None) -> None:
        for s in stmts:
            self.stmt(s, mask)

    def stmt(self, s: Node, mask) -> None:
        self.steps += 1
        if self.steps > MAX_STEPS:
            raise CompileError("fragment program too long to interpret")
        k = s.kind
        handler = getattr(self, "do_" + k, None)
        if handler is None:
            raise CompileError(f"{k} is not supported in a tensor-fragment program")
        handler(s, mask)

    def warp_op(self, s: Node, mask) -> None:
        if mask is not None and not np.all(mask):
            raise CompileError(f"{s.kind} under lane-divergent control")

    def do_Smem(self, s, mask):
        shape = tuple(int(x) for x in s.extents)
        dtype = _CTYPES.get(str(s.dtype))
        if dtype is None:
            raise CompileError(f"shared buffer type {s.dtype} is not supported")
        size = math.prod(shape)
        self.smem[s.name] = Smem(s.name, shape, dtype, int(s.get("align") or 0),
                                 np.full(size, -1, np.int64), np.full(size, -1, np.int64))

    def do_Sync(self, s, mask):
        self.warp_op(s, mask)
        for sm in self.smem.values():
            sm.dirty = False

    def loop_range(self, s):
        env = self.env
        start = ival(s.start, env) if s.kind == "StridedLoop" and s.get("start") is not None else 0
        step = ival(s.step, env) if s.kind == "StridedLoop" and s.get("step") is not None else 1
        end = s.get("end") if s.kind == "StridedLoop" else None
        bound = ival(end, env) if end is not None else static_extent(s.axis.extent)
        step = uniform(step, "loop step")
        if step <= 0:
            raise CompileError("loop step must be positive")
        return start, step, bound

    def do_StridedLoop(self, s, mask):
        start, step, bound = self.loop_range(s)
        name = s.axis.name
        saved = self.env.get(name)
        if s.kind == "StridedLoop" and s.get("end") is not None:
            self.env[name + "_end"] = bound
        if isinstance(start, np.ndarray) or isinstance(bound, np.ndarray):
            start = np.broadcast_to(np.asarray(start, np.int64), (32,))
            bound = np.broadcast_to(np.asarray(bound, np.int64), (32,))
            it = 0
            while True:
                value = start + it * step
                live = value < bound
                if mask is not None:
                    live &= mask
                if not live.any():
                    break
                self.env[name] = value
                self.run(s.body, live)
                it += 1
                if it > MAX_STEPS:
                    raise CompileError("loop too long to interpret")
        else:
            if (bound - start + step - 1) // step > MAX_STEPS:
                raise CompileError("loop too long to interpret")
            for value in range(start, bound, step):
                self.env[name] = value
                self.run(s.body, mask)
        if saved is None:
            self.env.pop(name, None)
        else:
            self.env[name] = saved

    do_Loop = do_StridedLoop

    def flat_index(self, shape: tuple, index: tuple, env=None):
        env = self.env if env is None else env
        vals = [ival(e, env) for e in index]
        if len(vals) == 1:
            return vals[0]
        if len(vals) != len(shape):
            raise CompileError(f"index rank {len(vals)} does not match shape {list(shape)}")
        total = 0
        for i, v in enumerate(vals):
            total = total + v * math.prod(shape[i + 1:])
        return total

    def do_Load(self, s, mask):
        if len(s.names) != 1:
            raise CompileError("vector loads are not supported in fragment programs")
        buf = self.pkg.buffers.get(s.input)
        if buf is None:
            raise CompileError(f"load from unknown buffer {s.input}")
        if buf.dtype not in ("f32", "f16", "bf16") or _dt(s.get("dtype")) not in ("f32", buf.dtype):
            raise CompileError("fill loads must read f32, f16 or bf16 without narrowing")
        flat = np.broadcast_to(np.asarray(self.flat_index(buf.shape, s.index), np.int64), (32,))
        live = np.ones(32, bool) if mask is None else mask
        size = math.prod(buf.shape) if buf.shape else 1
        if np.any(live & ((flat < 0) | (flat >= size))):
            raise CompileError(f"load from {s.input} outside the buffer")
        self.values[s.names[0]] = (np.where(live, self.leaf(s.input, np.clip(flat, 0, size - 1)), -1),
                                   buf.dtype)

    def do_Write(self, s, mask):
        sm = self.smem.get(s.output)
        if sm is None:
            raise CompileError("fragment programs may only write shared memory outside RegStore")
        if s.get("atomic") or len(s.values) != 1:
            raise CompileError("shared fills must write one element without atomics")
        name = s.values[0]
        if name not in self.values:
            raise CompileError(f"shared fill writes {name!r}, which is not a loaded element")
        leaves, src_dtype = self.values[name]
        vdt = _dt(s.get("value_dtype")) if s.get("value_dtype") is not None else sm.dtype
        if vdt != sm.dtype:
            raise CompileError("shared fill converts to another type than the buffer's")
        flat = np.broadcast_to(np.asarray(self.flat_index(sm.shape, s.index), np.int64), (32,))
        phys = swizzle(flat, s.get("swizzle"))
        live = np.ones(32, bool) if mask is None else mask
        if np.any(live & ((phys < 0) | (phys >= sm.leaf.size))):
            raise CompileError(f"write to {sm.name} outside the buffer")
        idx = phys[live]
        if len(np.unique(idx)) != len(idx):
            raise CompileError("two lanes write one shared element")
        sm.leaf[idx] = leaves[live]
        sm.pending[idx] = -1
        sm.dirty = True

    def do_CpAsyncCopy(self, s, mask):
        sm = self.smem.get(s.smem)
        buf = self.pkg.buffers.get(s.src)
        if sm is None or buf is None:
            raise CompileError("cp.async must copy a global buffer into shared memory")
        if buf.dtype != sm.dtype:
            raise CompileError("cp.async copies bytes: source and shared types must match")
        size = {"f32": 4, "f16": 2, "bf16": 2}[sm.dtype]
        nbytes = int(s.nbytes)
        if nbytes not in (4, 8, 16) or nbytes % size:
            raise CompileError(f"invalid cp.async size {nbytes}")
        dst = np.broadcast_to(np.asarray(self.flat_index(sm.shape, s.smem_index), np.int64), (32,))
        if s.get("lane_index") is not None:
            li = s.lane_index
            dst = dst + np.asarray(ival(li[0], self.env), np.int64) * sm.shape[-1] + ival(li[1], self.env)
        phys = swizzle(dst, s.get("swizzle"))
        src = np.broadcast_to(np.asarray(self.flat_index(buf.shape, s.src_index), np.int64), (32,))
        live = np.ones(32, bool) if mask is None else mask
        count = nbytes // size
        gsize = math.prod(buf.shape) if buf.shape else 1
        for e in range(count):
            p, g = phys[live] + e, src[live] + e
            if np.any((p < 0) | (p >= sm.leaf.size)) or np.any((g < 0) | (g >= gsize)):
                raise CompileError("cp.async outside its buffers")
            self.cp_open.append((sm, p.copy(), self.leaf(s.src, g)))

    def do_CpAsyncCommit(self, s, mask):
        self.warp_op(s, mask)
        group = self.cp_group
        for sm, p, leaves in self.cp_open:
            sm.pending[p] = group
            sm.leaf[p] = leaves
        self.cp_open = []
        self.cp_group += 1

    def do_CpAsyncWait(self, s, mask):
        self.warp_op(s, mask)
        allowed = int(s.group)
        done_below = self.cp_group - allowed  # groups numbered below this are complete
        for sm in self.smem.values():
            finished = (sm.pending >= 0) & (sm.pending < done_below)
            if finished.any():
                sm.pending[finished] = -1
                sm.dirty = True

    # ------------------------------------------------------------ fragments
    def ref(self, text: str, role: str | None = None):
        m = re.fullmatch(r"([A-Za-z_$][\w$]*)(?:\[([A-Za-z_$][\w$]*|[0-9]+)\])?", str(text))
        if m is None:
            raise CompileError(f"unsupported fragment reference {text!r}")
        stem, sub = m.groups()
        frag = self.frags.get(stem)
        if frag is None:
            raise CompileError(f"undeclared fragment {stem!r}")
        if role is not None and frag.role != role:
            raise CompileError(f"fragment {stem!r} must have role {role}")
        if sub is None:
            if len(frag.members) != 1:
                raise CompileError(f"fragment family {stem!r} needs a subscript")
            return frag, 0
        idx = int(sub) if sub.isdecimal() else uniform(ival(Node("Var", (("name", sub),)), self.env),
                                                        "fragment subscript")
        if not 0 <= idx < len(frag.members):
            raise CompileError(f"fragment index {idx} outside {stem!r}")
        return frag, idx

    def do_RegFragment(self, s, mask):
        self.warp_op(s, mask)
        if tuple(s.shape) != SHAPE:
            raise CompileError(f"fragment shape {s.shape} is not m16n8k16")
        if s.get("fragment_layout", "m16n8k16") not in (None, "m16n8k16"):
            raise CompileError("only the m16n8k16 fragment layout is supported")
        dtype = _dt(s.dtype)
        if s.role == "c" and dtype != "f32" or s.role in ("a", "b") and dtype not in ("f16", "bf16") \
                or s.role not in ("a", "b", "c"):
            raise CompileError("fragments must be f16/bf16 A/B or f32 C")
        count = int(s.get("count") or 1)
        if not 1 <= count <= 64:
            raise CompileError("fragment family count must be 1..64")
        self.frags[s.name] = Fragment(s.role, dtype,
                                      [CVal() if s.role == "c" else None for _ in range(count)])

    def do_LdmatrixLoad(self, s, mask):
        self.warp_op(s, mask)
        if s.role not in ("a", "b") or (s.role == "a" and s.get("b_trans")):
            raise CompileError("invalid tensor operand role or orientation")
        if s.get("byte_slab") or s.get("scale_buffer") is not None or s.get("scale_index") \
                or s.get("scale_ldm"):
            raise CompileError("byte or block-scaled tensor loads are not supported")
        if s.get("fragment_layout", "m16n8k16") not in (None, "m16n8k16"):
            raise CompileError("only the m16n8k16 fragment layout is supported")
        frag, idx = self.ref(s.frag, s.role)
        if s.get("staged"):
            ids = self.shared_gather(s, frag)
        else:
            ids = (self.global_gather(s, frag),)
        frag.members[idx] = ids[0]
        if len(ids) == 2:
            pair, pidx = self.ref(s.pair_frag, "b")
            if pair.dtype != frag.dtype:
                raise CompileError("paired fragments must share a type")
            pair.members[pidx] = ids[1]

    def global_gather(self, s, frag) -> np.ndarray:
        buf = self.pkg.buffers.get(s.src_buffer)
        if buf is None or s.src_buffer in self.smem:
            raise CompileError("unstaged tensor loads must read a global buffer")
        if s.get("swizzle", "NONE") not in (None, "NONE") or s.get("pair_frag") is not None:
            raise CompileError("global tensor loads take no swizzle or paired fragment")
        if buf.dtype not in ("f16", "bf16", "f32"):
            raise CompileError(f"tensor loads from {buf.dtype} buffers are not supported")
        ldm = int(s.get("ldm") or buf.shape[-1])
        if ldm <= 0:
            raise CompileError("tensor load row stride must be positive")
        base = uniform(self.flat_index(buf.shape, s.src_index), "fragment base")
        if s.role == "a":
            mn, k = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")   # [m, k]
        else:
            k, mn = np.meshgrid(np.arange(16), np.arange(8), indexing="ij")    # [k, n]
        valid = np.ones(mn.shape, bool)
        if s.get("gmem_guard") is not None:
            g0, g1 = (uniform(ival(e, self.env), "guard") for e in s.gmem_guard)
            rem = g1 - g0
            if rem <= 0:
                valid[:] = False
            mn = np.minimum(mn, max(rem - 1, 0))
        if s.get("k_zero") is not None:
            k0, k1 = (uniform(ival(e, self.env), "guard") for e in s.k_zero)
            valid &= k < (k1 - k0)
        row, col = (mn, k) if s.role == "a" or s.get("b_trans") else (k, mn)
        flat = base + row * ldm + col
        size = math.prod(buf.shape)
        if np.any(valid & ((flat < 0) | (flat >= size))):
            raise CompileError(f"tensor load from {s.src_buffer} outside the buffer")
        return np.where(valid, self.leaf(s.src_buffer, np.clip(flat, 0, size - 1)), -1)

    def shared_gather(self, s, frag) -> tuple:
        sm = self.smem.get(s.src_buffer)
        if sm is None:
            raise CompileError("staged tensor loads must read shared memory")
        if sm.dtype != frag.dtype:
            raise CompileError("ldmatrix needs shared storage of the fragment's type")
        if s.get("gmem_guard") is not None or s.get("k_zero") is not None:
            raise CompileError("staged tensor loads take no guards")
        ldm = int(s.get("ldm") or sm.shape[-1])
        if ldm % 8 or sm.align < 16:
            raise CompileError("ldmatrix needs 16-byte aligned rows")
        if sm.dirty:
            raise CompileError(f"{sm.name} is read before a barrier orders its fill")
        base = uniform(self.flat_index(sm.shape, s.src_index), "fragment base")
        mode = s.get("swizzle")
        b_trans = bool(s.get("b_trans"))
        paired = s.get("pair_frag") is not None
        if paired and s.role != "b":
            raise CompileError("paired ldmatrix loads two B fragments")

        def read(logical_row_start, inner):
            # one ldmatrix row: 8 contiguous elements at the swizzled row address
            start = swizzle(np.asarray(logical_row_start, np.int64), mode)
            if np.any(start % 8):
                raise CompileError("ldmatrix row address is not 16-byte aligned")
            phys = start + inner
            if np.any((phys < 0) | (phys >= sm.leaf.size)):
                raise CompileError(f"ldmatrix outside {sm.name}")
            if np.any(sm.pending[phys] >= 0):
                raise CompileError(f"{sm.name} is read before its cp.async completes")
            ids = sm.leaf[phys]
            if np.any(ids < 0):
                raise CompileError(f"ldmatrix reads elements of {sm.name} nothing wrote")
            return ids

        if s.role == "a":
            i, kk = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
            return (read(base + i * ldm + (kk // 8) * 8, kk % 8),)
        kk, j = np.meshgrid(np.arange(16), np.arange(8), indexing="ij")
        if not b_trans:       # B stored [k, n]: ldmatrix.trans over k rows
            first = read(base + kk * ldm, j)
            return (first, read(base + kk * ldm + 8, j)) if paired else (first,)
        first = read(base + j * ldm + (kk // 8) * 8, kk % 8)   # B stored [n, k]
        if paired:
            return first, read(base + (j + 8) * ldm + (kk // 8) * 8, kk % 8)
        return (first,)

    def do_MmaSyncPtx(self, s, mask):
        self.warp_op(s, mask)
        if tuple(s.shape) != SHAPE or s.ab_dtype not in ("f16", "bf16") or s.c_dtype != "f32":
            raise CompileError("MMA must be m16n8k16 with f16/bf16 operands and f32 accumulation")
        if s.get("b_row_major") or s.get("sfa_frag") is not None or s.get("sfb_frag") is not None:
            raise CompileError("row-major B and block-scaled MMA forms are not supported")
        a, ai = self.ref(s.a_frag, "a")
        b, bi = self.ref(s.b_frag, "b")
        c, ci = self.ref(s.c_frag, "c")
        if a.dtype != s.ab_dtype or b.dtype != s.ab_dtype:
            raise CompileError("MMA type disagrees with its fragments")
        av, bv = a.members[ai], b.members[bi]
        if av is None or bv is None:
            raise CompileError("MMA reads a fragment nothing loaded")
        c.members[ci] = CVal(c.members[ci].terms + [(av, bv, s.ab_dtype)])

    def do_FragmentRepack(self, s, mask):
        self.warp_op(s, mask)
        if int(s.get("part") or 0) != 0 or len(s.srcs) != 2 or s.ab_dtype not in ("f16", "bf16"):
            raise CompileError("repack takes two C fragments into a 16-bit A fragment")
        frag, idx = self.ref(s.frag, "a")
        if frag.dtype != s.ab_dtype:
            raise CompileError("repack type disagrees with its A fragment")
        halves = tuple(self.ref(src, "c") for src in s.srcs)
        v = Virtual(tuple(f.members[i] for f, i in halves), s.ab_dtype)
        i, j = np.meshgrid(np.arange(16), np.arange(16), indexing="ij")
        frag.members[idx] = self.leaf(v, i * 16 + j)

    def do_RegStore(self, s, mask):
        self.warp_op(s, mask)
        if tuple(s.shape) != SHAPE or s.get("volta_interleaved") or s.get("extra_frags"):
            raise CompileError("fragment stores must be plain m16n8k16 stores")
        if s.get("swizzle", "NONE") not in (None, "NONE"):
            raise CompileError("swizzled global stores are not supported")
        if tuple(s.get("fragment_index") or (0, 0)) != (0, 0) and s.get("fragment_layout") not in (None, "m16n8k16"):
            raise CompileError("only the m16n8k16 fragment layout is supported")
        buf = self.pkg.buffers.get(s.dst_buffer)
        if buf is None or s.dst_buffer in self.smem or buf.role != "output":
            raise CompileError("fragment stores must write the kernel's output")
        if buf.dtype not in ("f32", "f16", "bf16"):
            raise CompileError("tensor outputs must be f32, f16 or bf16")
        if s.get("atomic") and buf.dtype != "f32":
            raise CompileError("atomic tensor stores need an f32 output")
        frag, idx = self.ref(s.frag, "c")
        shape = buf.shape
        rd, cd = s.get("row_dim"), s.get("col_dim")
        for dim in (rd, cd):
            if dim is not None and not 0 <= dim < len(shape):
                raise CompileError("tensor output dimension outside its buffer rank")
        row_stride = int(s.get("ldm") or 0) or (math.prod(shape[rd + 1:]) if rd is not None else shape[-1])
        col_stride = math.prod(shape[cd + 1:]) if cd is not None else 1
        base = uniform(self.flat_index(shape, s.dst_index), "store base")
        i, j = np.meshgrid(np.arange(16), np.arange(8), indexing="ij")
        keep = np.ones(i.shape, bool)
        for guard, off in ((s.get("m_guard"), i), (s.get("n_guard"), j)):
            if guard is not None:
                g0, g1 = (uniform(ival(e, self.env), "store guard") for e in guard)
                keep &= g0 + off < g1
        flats = base + i * row_stride + j * col_stride
        size = math.prod(shape)
        if np.any(keep & ((flats < 0) | (flats >= size))):
            raise CompileError(f"fragment store outside {s.dst_buffer}")
        self.stores.append((s.dst_buffer, StoreRecord(flats[keep], i[keep], j[keep], frag.members[idx],
                                                      s.get("epilogue"), bool(s.get("atomic")))))


# ---------------------------------------------------------------- verification

def _decode(interp: FragmentInterpreter, ids: np.ndarray):
    src = ids >> _LEAF_SHIFT
    flat = ids & ((np.int64(1) << _LEAF_SHIFT) - 1)
    return src, flat


@dataclass
class Contraction:
    a_src: object            # buffer name or Virtual
    b_src: str
    rows: np.ndarray         # A row per element
    cols: np.ndarray         # B column per element
    k: int
    b_layout: str
    mma: str


def _operand_rows(interp, src, flat, role, layout=None):
    """(row, k) of A leaves or (k, n) of B leaves."""
    if isinstance(src, Virtual):
        info = _virtual_info(interp, src)
        return info["rows"][flat], info["cols"][flat], info["n"]
    buf = interp.pkg.buffers[src]
    if len(buf.shape) != 2:
        raise CompileError("GEMM operands must be matrices")
    r, c = np.divmod(flat, buf.shape[1])
    if role == "a":
        return r, c, buf.shape[1]
    if layout == "kn":
        return r, c, buf.shape[0]
    return c, r, buf.shape[1]


def contraction(interp: FragmentInterpreter, cval: CVal, i: np.ndarray, j: np.ndarray) -> Contraction:
    """The GEMM the C elements (i, j) of `cval` compute, or CompileError."""
    if not cval.terms:
        raise CompileError("a stored fragment holds no product")
    mmas = {t for _, _, t in cval.terms}
    if len(mmas) != 1:
        raise CompileError("one fragment mixes f16 and bf16 products")
    A = np.stack([a for a, _, _ in cval.terms])            # [P, 16, 16]
    B = np.stack([b for _, b, _ in cval.terms])            # [P, 16, 8]
    a = A[:, i, :].transpose(1, 0, 2).reshape(len(i), -1)  # [E, P*16]
    b = B[:, :, j].transpose(2, 0, 1).reshape(len(j), -1)
    live = (a >= 0) & (b >= 0)
    if not live.any(axis=1).all():
        raise CompileError("a stored element has no product term")
    a_src, a_flat = _decode(interp, a[live])
    b_src, b_flat = _decode(interp, b[live])
    if len(np.unique(a_src)) != 1 or len(np.unique(b_src)) != 1:
        raise CompileError("a fragment multiplies elements of several buffers")
    asrc = interp.sources[int(a_src[0])]
    bsrc = interp.sources[int(b_src[0])]
    if isinstance(bsrc, Virtual):
        raise CompileError("repacked fragments may only be A operands")
    ar, ak, ka = _operand_rows(interp, asrc, a_flat, "a")
    counts = live.sum(axis=1)
    elem = np.repeat(np.arange(len(i)), counts)
    for layout in ("kn", "nk"):
        bk, bn, kb = _operand_rows(interp, bsrc, b_flat, "b", layout)
        if ka != kb or not np.array_equal(ak, bk):
            continue
        rows = np.full(len(i), -1, np.int64)
        cols = np.full(len(i), -1, np.int64)
        rows[elem] = ar
        cols[elem] = bn
        if not (np.array_equal(rows[elem], ar) and np.array_equal(cols[elem], bn)):
            continue
        # every element: K terms, k = 0 .. K-1 each once
        if not np.all(counts == ka):
            continue
        order = np.lexsort((ak, elem))
        if not np.array_equal(ak[order], np.tile(np.arange(ka), len(i))):
            continue
        return Contraction(asrc, bsrc, rows, cols, ka, layout, mmas.pop())
    raise CompileError("a stored fragment is not a full row-by-column contraction")


def _virtual_info(interp: FragmentInterpreter, v: Virtual) -> dict:
    """Map the 256 elements of a repacked fragment to (row, column) of one product T = X Y."""
    if v.info is not None:
        return v.info
    i, j = np.meshgrid(np.arange(16), np.arange(8), indexing="ij")
    i, j = i.ravel(), j.ravel()
    parts = [contraction(interp, half, i, j) for half in v.halves]
    first = parts[0]
    for p in parts[1:]:
        if (p.a_src, p.b_src, p.k, p.b_layout, p.mma) != (first.a_src, first.b_src, first.k, first.b_layout,
                                                         first.mma):
            raise CompileError("a repacked fragment joins different products")
    if isinstance(first.a_src, Virtual):
        raise CompileError("nested fragment repacks are not supported")
    rows = np.empty(256, np.int64)
    cols = np.empty(256, np.int64)
    for h, p in enumerate(parts):
        flat = i * 16 + j + 8 * h
        rows[flat], cols[flat] = p.rows, p.cols
    ybuf = interp.pkg.buffers[first.b_src]
    n = ybuf.shape[1] if first.b_layout == "kn" else ybuf.shape[0]
    v.info = {"rows": rows, "cols": cols, "n": n, "product": first}
    return v.info


def _epilogue(pkg: KernelPackage, lam) -> tuple[str, tuple | None]:
    """Classify a RegStore epilogue lambda: (activation, (bias buffer, index) or None)."""
    if lam is None:
        return "none", None
    from .recognize import _Eval, _match, V, op, _strip_casts
    from .recognize_f32 import strip_epilogue, _drop_copies
    params = list(lam.params)
    if not params:
        raise CompileError("epilogue takes no accumulator")
    ev = _Eval(pkg)
    ev.smem = set()
    ev.env[params[0]] = ("acc", "__acc")
    loads = {}
    for st in lam.body:
        if st.kind == "Load":
            if len(st.names) != 1:
                raise CompileError("epilogue loads must be scalar")
            loads[st.names[0]] = (st.input, tuple(st.index))
            ev.env[st.names[0]] = ("bias", st.names[0])
        elif st.kind in ("Assign", "Select"):
            for d in (st.get("dtype"),):
                if d is not None and _dt(d) != "f32":
                    raise CompileError("epilogue arithmetic must be f32")
            ev.stmt(st)
        else:
            raise CompileError(f"unsupported epilogue statement {st.kind}")
    (result,) = lam.results
    expr, _ = _strip_casts(ev.env[result])
    expr = _drop_copies(expr)
    act = "none"
    if isinstance(expr, tuple) and expr[:2] == ("op", "relu") and len(expr) == 3:
        act, inner = "relu", expr[2]
    else:
        b = _match(op("maximum", V("x"), V("zero", lambda e: e == ("lit", 0.0))), expr, {})
        if b:
            act, inner = "relu", b["x"]
        else:
            act, inner = strip_epilogue(pkg, expr)
    inner = _drop_copies(inner)
    if inner == ("acc", "__acc"):
        return act, None
    b = _match(op("add", V("acc", lambda e: e == ("acc", "__acc")),
                  V("bias", lambda e: isinstance(e, tuple) and e[:1] == ("bias",))), inner, {})
    if not b:
        raise CompileError("epilogue is not acc, acc + bias[col], then identity, GELU or ReLU")
    buf, index = loads[b["bias"][1]]
    bb = pkg.buffers.get(buf)
    if bb is None or bb.dtype != "f32" or len(bb.shape) != 1:
        raise CompileError("epilogue bias must be an f32 vector")
    return act, (buf, index)


def _bias_ok(index: tuple, coords: list, rec: StoreRecord, cols: np.ndarray) -> bool:
    """Does the bias index read bias[n] for every stored element?

    The reference binds the epilogue's coordinate parameters to the element's
    row and column inside its fragment (ptx_tensor.py:436-438), not in the
    output, so a bias indexed by them is bias[n] only for fragments stored at
    column 0; that is checked element by element.
    """
    env = {"__M__": rec.i.astype(np.int64), "__N__": rec.j.astype(np.int64)}
    for name in coords:
        if name not in env:
            raise CompileError(f"unbound epilogue coordinate {name!r}")
    if len(index) != 1:
        return False
    got = np.broadcast_to(np.asarray(ival(index[0], env), np.int64), cols.shape)
    return np.array_equal(got, cols)


def is_single_warp(pkg: KernelPackage, tile: Node) -> bool:
    """A Tile over one 32-lane axis launched as one warp in one block."""
    axes = tuple(tile.axes)
    meta = pkg.kernel_meta
    block = [int(x) for x in meta.get("block", [0])]
    grid = [int(x) for x in meta.get("grid", [0])]
    return (len(axes) == 1 and static_extent(axes[0].extent) == 32 and block[:1] == [32]
            and all(x == 1 for x in block[1:]) and all(x == 1 for x in grid))


def recognise_fragment_tile(pkg: KernelPackage, tile: Node):
    """Plan of a one-warp fragment program (see the module docstring)."""
    from .recognize import _plan
    interp = FragmentInterpreter(pkg, tile)
    interp.run(tile.body)
    if not interp.stores:
        raise CompileError("fragment program stores nothing")
    outs = {name for name, _ in interp.stores}
    if len(outs) != 1:
        raise CompileError("fragment program must store one output")
    out = outs.pop()
    obuf = pkg.buffers[out]
    if len(obuf.shape) != 2:
        raise CompileError("fragment program output must be a matrix")
    recs = [r for _, r in interp.stores]
    atomic = {r.atomic for r in recs}
    if len(atomic) != 1:
        raise CompileError("fragment stores mix atomic and plain stores")
    atomic = atomic.pop()
    if atomic and out not in pkg.kernel_meta.get("zero_outputs", []):
        raise CompileError("atomic fragment stores need the output in zero_outputs")
    size = math.prod(obuf.shape)
    written = np.bincount(np.concatenate([r.flats for r in recs]), minlength=size)
    if np.any(written != 1):
        raise CompileError("fragment stores do not write every output element exactly once")
    # one contraction per store record, all the same product
    sig = None
    epis = set()
    trans_forms = set()
    for r in recs:
        con = contraction(interp, r.cval, r.i, r.j)
        key = (id(con.a_src) if isinstance(con.a_src, Virtual) else con.a_src, con.b_src, con.k,
               con.b_layout, con.mma)
        if isinstance(con.a_src, Virtual):
            info = _virtual_info(interp, con.a_src)
            key = ("chain", info["product"].a_src, info["product"].b_src, info["product"].k,
                   info["product"].b_layout, info["n"], con.b_src, con.k, con.b_layout, con.mma)
        if sig is not None and key != sig[0]:
            raise CompileError("fragments store different products")
        sig = (key, con)
        epi = _epilogue(pkg, r.epilogue)
        if epi[1] is not None:
            coords = list(r.epilogue.params[1:])
            if not _bias_ok(epi[1][1], coords, r, con.cols):
                raise CompileError("epilogue bias is not indexed by the output column")
            epi = (epi[0], epi[1][0])
        epis.add(epi)
        plain = con.rows * obuf.shape[1] + con.cols
        trans = con.cols * obuf.shape[1] + con.rows
        forms = set()
        if np.array_equal(r.flats, plain):
            forms.add(False)
        if np.array_equal(r.flats, trans):
            forms.add(True)
        if not forms:
            raise CompileError("fragment stores do not place C[r, n] at its row and column")
        trans_forms.add(frozenset(forms))
    if len(epis) != 1:
        raise CompileError("fragments use different epilogues")
    act, bias = epis.pop()
    common = frozenset.intersection(*trans_forms)
    if not common:
        raise CompileError("fragment stores mix plain and transposed layouts")
    transposed = False if False in common else True
    key, con = sig
    if isinstance(con.a_src, Virtual):
        if act != "none" or bias is not None or atomic or transposed:
            raise CompileError("chained products take no epilogue or store variant")
        info = _virtual_info(interp, con.a_src)
        inner = info["product"]
        x, y, z = inner.a_src, inner.b_src, con.b_src
        xs, ys, zs = (pkg.buffers[n].shape for n in (x, y, z))
        m, k = xs
        n1 = info["n"]
        n2 = zs[1] if con.b_layout == "kn" else zs[0]
        if tuple(obuf.shape) != (m, n2) or con.k != n1 or inner.k != k or inner.mma != con.mma \
                or info["rows"].max() >= m:
            raise CompileError("chained product shapes are inconsistent")
        return _plan(pkg, "gemm_chain", "lc_gemm_chain", {"x": x, "y": y, "z": z, "c": out},
                     {"m": m, "k": k, "n1": n1, "n2": n2, "y_layout": inner.b_layout,
                      "z_layout": con.b_layout},
                     {"mma": con.mma, "x": pkg.buffers[x].dtype, "y": pkg.buffers[y].dtype,
                      "z": pkg.buffers[z].dtype, "c": obuf.dtype})
    a, b = con.a_src, con.b_src
    sa, sb = pkg.buffers[a].shape, pkg.buffers[b].shape
    m, k = sa
    n = sb[1] if con.b_layout == "kn" else sb[0]
    want = (n, m) if transposed else (m, n)
    if tuple(obuf.shape) != want or con.k != k:
        raise CompileError(f"GEMM shapes {sa} x {sb} -> {obuf.shape} are inconsistent")
    bind = {"a": a, "b": b, "c": out}
    if bias is not None:
        if tuple(pkg.buffers[bias].shape) != (n,):
            raise CompileError("epilogue bias length differs from N")
        bind["bias"] = bias
    return _plan(pkg, "gemm_mixed", "lc_gemm_mixed", bind,
                 {"m": m, "n": n, "k": k, "b_layout": con.b_layout, "epilogue": act,
                  "transpose": transposed, "accumulate": atomic},
                 {"mma": con.mma, "a": pkg.buffers[a].dtype, "b": pkg.buffers[b].dtype, "c": obuf.dtype})
