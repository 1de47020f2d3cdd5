"""A numpy interpreter of compiled pointwise programs — test infrastructure.

Runs the register program of a ``pointwise`` plan on the CPU, one numpy
array per register over all tile points, so the CPU suite can check the
program compiler's typing and lowering against the IR oracle without a GPU.
The approximate PTX instructions (ex2/lg2/sin/cos.approx) are replaced by
accurate numpy functions; everything else is bit-exact IEEE arithmetic.
"""
import numpy as np

from lazy_compiler_b200.pointwise import OPCODES

_NP = {"f32": np.float32, "f16": np.float16, "bf16": np.float32, "s32": np.int32}


def _f(w):
    return w.view(np.float32)


def _w(x):
    return np.asarray(x, np.float32).view(np.uint32)


def _bf16(x):
    bits = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32)
    return np.where(np.isnan(x), np.float32(np.nan), out)


def _half(words, bf16):
    """The f32 values of the low and high 16-bit halves of packed words."""
    lo, hi = words & np.uint32(0xFFFF), words >> 16
    if bf16:
        return (lo << 16).view(np.float32), (hi << 16).view(np.float32)
    return (lo.astype(np.uint16).view(np.float16).astype(np.float32),
            hi.astype(np.uint16).view(np.float16).astype(np.float32))


def _mma(r, dst, a, b, c, bf16, n):
    """mma.sync m16n8k16 per warp of 32 points: fragments gathered into
    matrices, the product in float64 rounded once to f32 (the tensor core's
    f32 accumulation agrees to the packages' tolerances)."""
    lane = np.arange(n) % 32
    g, t = lane // 4, lane % 4
    for w0 in range(0, n, 32):
        sl = slice(w0, w0 + 32)
        A = np.zeros((16, 16))
        B = np.zeros((16, 8))
        C = np.zeros((16, 8))
        for i in range(4):
            lo, hi = _half(r[a + i][sl], bf16)
            rows = g[sl] + (8 if i & 1 else 0)
            cols = 2 * t[sl] + (8 if i & 2 else 0)
            A[rows, cols], A[rows, cols + 1] = lo, hi
        for i in range(2):
            lo, hi = _half(r[b + i][sl], bf16)
            k = 2 * t[sl] + (8 if i else 0)
            B[k, g[sl]], B[k + 1, g[sl]] = lo, hi
        for e in range(4):
            C[g[sl] + (8 if e >= 2 else 0), 2 * t[sl] + (e & 1)] = _f(r[c + e][sl])
        D = (A @ B + C).astype(np.float32)
        for e in range(4):
            r.setdefault(dst + e, np.zeros(n, np.uint32))
            r[dst + e] = r[dst + e].copy()
            r[dst + e][sl] = _w(D[g[sl] + (8 if e >= 2 else 0), 2 * t[sl] + (e & 1)])


def run(prog: dict, arrays: dict, coords=None, states=None, partials=None, partners=None, mask=None,
        outs=None) -> dict:
    """Run a program (or one range of it: ``prog["code"]``) over every point.

    ``coords`` overrides the points (one coordinate array per axis);
    ``states`` / ``partials`` / ``partners`` map state slots to per-point
    arrays for row programs (SETP writes ``partials`` in place); ``mask``
    limits stores and SETP to some points; ``outs`` collects outputs across
    calls."""
    if coords is None:
        ext = prog["extents"]
        grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for e in ext], indexing="ij")
        coords = [g.ravel() for g in grids]
    n = coords[0].size
    live = np.ones(n, bool) if mask is None else mask
    bufs = []
    for name, size in zip(prog["buffers"], prog["sizes"]):
        if name in arrays:
            a = np.asarray(arrays[name]).ravel()
            bufs.append(a.astype(np.float32) if a.dtype == np.float16 else a.copy())
        else:
            bufs.append(None)
    outs = {} if outs is None else outs
    r = {}
    consts = np.asarray(prog["consts"], np.uint64).astype(np.uint32)
    with np.errstate(all="ignore"):
        code = prog["code"]
        loops = list(prog.get("loops", []))
        coords = list(coords) + [np.zeros(n, np.int64) for _ in loops]   # loop counters follow the axes
        n_axes = len(coords) - len(loops)
        pc = -1
        while pc + 1 < len(code):
            pc += 1
            op, dst, a, b, c, aux = code[pc]
            if OPCODES[op] in ("LOOPB", "LOOPE"):
                d = n_axes + (aux & 15)
                limit = min(int(r[a].view(np.int32)[0]), loops[aux & 15])
                if OPCODES[op] == "LOOPB":
                    coords[d] = np.zeros(n, np.int64)
                    if limit <= 0:
                        pc = aux >> 4
                else:
                    coords[d] = coords[d] + 1
                    if coords[d][0] < limit:
                        pc = aux >> 4
                continue
            _step(prog, code[pc], r, coords, bufs, outs, consts, n, live, states, partials, partners)
    return outs



def _step(prog, entry, r, coords, bufs, outs, consts, n, live, states, partials, partners):
    """One operation (not a loop or branch) over every point; stores and SETP only where ``live``."""
    op, dst, a, b, c, aux = entry
    name = OPCODES[op]
    A, B, C = r.get(a), r.get(b), r.get(c)
    if name.startswith(("LD_", "ST_")):
        f = prog["forms"][aux]
        at = f["base"] + sum(k * x for k, x in zip(f["coef"], coords))
        slot = f["buffer"]
        if name.startswith("LD_"):
            v = bufs[slot][at]
            r[dst] = v.astype(np.int32).view(np.uint32) if name == "LD_S32" else _w(v.astype(np.float32))
        else:
            bname = prog["buffers"][slot]
            if bname not in outs:
                outs[bname] = np.full(prog["sizes"][slot], np.nan if name != "ST_S32" else 0,
                                      np.float32 if name != "ST_S32" else np.int32)
            val = A.view(np.int32) if name == "ST_S32" else _f(A)
            if name == "ST_F16":
                val = val.astype(np.float16).astype(np.float32)
            elif name == "ST_BF16":
                val = _bf16(val)
            outs[bname][at[live]] = val[live]
        return
    fa, fb, fc = (_f(x) if x is not None else None for x in (A, B, C))
    ia, ib = (x.view(np.int32).astype(np.int64) if x is not None else None for x in (A, B))
    if name == "MOV":
        out = A
    elif name == "CONST":
        out = np.full(n, consts[aux], np.uint32)
    elif name in ("FADD", "FSUB", "FMUL", "FDIV"):
        out = _w({"FADD": fa + fb, "FSUB": fa - fb, "FMUL": fa * fb, "FDIV": fa / fb}[name])
    elif name == "FFMA":
        out = _w((fa.astype(np.float64) * fb + fc.astype(np.float64)).astype(np.float32))
    elif name == "FNEG":
        out = A ^ np.uint32(0x80000000)
    elif name == "FABS":
        out = A & np.uint32(0x7FFFFFFF)
    elif name in ("FMAX", "FMIN"):
        out = _w(np.fmax(fa, fb) if name == "FMAX" else np.fmin(fa, fb))
    elif name in ("FSQRT", "FFLOOR", "FCEIL", "FTRUNC", "FRINT"):
        fn = {"FSQRT": np.sqrt, "FFLOOR": np.floor, "FCEIL": np.ceil, "FTRUNC": np.trunc,
              "FRINT": np.rint}[name]
        out = _w(fn(fa))
    elif name in ("FEX2", "FLG2", "FSIN", "FCOS"):
        fn = {"FEX2": np.exp2, "FLG2": np.log2, "FSIN": np.sin, "FCOS": np.cos}[name]
        out = _w(fn(fa.astype(np.float64)).astype(np.float32))
    elif name == "FCOPYSIGN":
        out = (B & np.uint32(0x7FFFFFFF)) | (A & np.uint32(0x80000000))
    elif name == "RND_F16":
        out = _w(fa.astype(np.float16).astype(np.float32))
    elif name == "RND_BF16":
        out = _w(_bf16(fa))
    elif name == "F2I":
        x = np.nan_to_num(np.trunc(fa.astype(np.float64)), nan=0.0, posinf=2.0 ** 31, neginf=-2.0 ** 31)
        out = np.clip(x, -2 ** 31, 2 ** 31 - 1).astype(np.int32).view(np.uint32)
    elif name in ("I2F", "I2H", "I2BF"):
        x = ia.astype(np.float64)
        if name == "I2F":
            out = _w(x.astype(np.float32))
        elif name == "I2H":
            out = _w(x.astype(np.float16).astype(np.float32))
        else:
            m, e = np.frexp(x)
            out = _w(np.ldexp(np.rint(np.ldexp(m, 8)), e - 8).astype(np.float32))
    elif name.startswith("I") and name not in ("IEQ", "INE", "ILT", "ILE", "IGT", "IGE"):
        safe = np.where(ib == 0, 1, ib) if ib is not None else None
        q = np.where(ib == 0, 0, np.trunc(ia / safe)).astype(np.int64) if ib is not None else None
        res = {"IADD": lambda: ia + ib, "ISUB": lambda: ia - ib, "IMUL": lambda: ia * ib,
               "IDIV": lambda: q, "IREM": lambda: np.where(ib == 0, ia, ia - safe * q),
               "ISHL": lambda: np.where((ib & 0xFFFFFFFF) >= 32, 0, ia << np.clip(ib, 0, 31)),
               "ISHR": lambda: ia >> np.clip(ib & 0xFFFFFFFF, 0, 31), "IAND": lambda: ia & ib,
               "IOR": lambda: ia | ib, "IXOR": lambda: ia ^ ib, "INOT": lambda: ~ia, "INEG": lambda: -ia,
               "IABS": lambda: np.abs(ia), "IMAX": lambda: np.maximum(ia, ib),
               "IMIN": lambda: np.minimum(ia, ib),
               "IPOPC": lambda: np.asarray([bin(int(v) & 0xFFFFFFFF).count("1") for v in ia])}[name]()
        out = (np.asarray(res, np.int64) % (1 << 32)).astype(np.uint32)
    elif name in ("FEQ", "FNE", "FLT", "FLE", "FGT", "FGE"):
        res = {"FEQ": fa == fb, "FNE": ~(fa == fb), "FLT": fa < fb, "FLE": fa <= fb, "FGT": fa > fb,
               "FGE": fa >= fb}[name]
        out = res.astype(np.uint32)
    elif name in ("IEQ", "INE", "ILT", "ILE", "IGT", "IGE"):
        res = {"IEQ": ia == ib, "INE": ia != ib, "ILT": ia < ib, "ILE": ia <= ib, "IGT": ia > ib,
               "IGE": ia >= ib}[name]
        out = res.astype(np.uint32)
    elif name in ("PAND", "POR"):
        out = (((A != 0) & (B != 0)) if name == "PAND" else ((A != 0) | (B != 0))).astype(np.uint32)
    elif name == "SEL":
        out = np.where(A != 0, B, C)
    elif name == "COORD":
        out = coords[aux].astype(np.int64).astype(np.uint32)
    elif name.startswith("LDX_"):
        data = bufs[aux]
        at = np.clip(ia, 0, data.size - 1)
        v = data[at]
        out = v.astype(np.int32).view(np.uint32) if name == "LDX_S32" else _w(v.astype(np.float32))
    elif name.startswith("STX_"):
        bname = prog["buffers"][aux]
        if bname not in outs:
            outs[bname] = np.full(prog["sizes"][aux], np.nan if name != "STX_S32" else 0,
                                  np.float32 if name != "STX_S32" else np.int32)
        live = (C != 0) & (ia >= 0) & (ia < prog["sizes"][aux]) & live
        val = B.view(np.int32) if name == "STX_S32" else _f(B)
        if name == "STX_F16":
            val = val.astype(np.float16).astype(np.float32)
        elif name == "STX_BF16":
            val = _bf16(val)
        if name == "STX_ADD_F32":
            base = np.nan_to_num(outs[bname], nan=0.0)   # the runner zeroes atomic outputs
            for k in np.nonzero(live)[0]:
                base[ia[k]] += val[k]
            outs[bname] = base
        else:
            outs[bname][ia[live]] = val[live]
        return
    elif name == "SHFL_XOR":
        out = A[np.arange(n) ^ aux]
    elif name in ("PACK_F16X2", "PACK_BF16X2"):
        if name == "PACK_F16X2":
            lo = fa.astype(np.float16).view(np.uint16).astype(np.uint32)
            hi = fb.astype(np.float16).view(np.uint16).astype(np.uint32)
        else:
            lo = _bf16(fa).view(np.uint32) >> 16
            hi = _bf16(fb).view(np.uint32) >> 16
        out = (hi << 16) | lo
    elif name == "STATE":
        out = _w(np.broadcast_to(np.asarray(states[aux], np.float32), (n,)))
    elif name == "PARTIAL":
        out = _w(np.asarray(partials[aux], np.float32))
    elif name == "PARTNER":
        out = _w(np.asarray(partners[aux], np.float32))
    elif name == "SETP":
        partials[aux] = np.where(live, _f(A), partials[aux]).astype(np.float32)
        return
    elif name == "FREM":
        r0 = np.fmod(fa, fb)
        adjust = (r0 != 0) & ((fa < 0) != (fb < 0))
        r0 = np.where(adjust, (r0 + fb).astype(np.float32), r0)
        r0 = np.where(r0 == 0, np.copysign(np.float32(0), fb), r0)
        r0 = np.where(~np.isfinite(fa) | np.isnan(fb) | (fb == 0), np.float32(np.nan), r0)
        out = _w(r0.astype(np.float32))
    elif name in ("MMA_F16", "MMA_BF16"):
        _mma(r, dst, a, b, c, name == "MMA_BF16", n)
        return
    else:
        raise ValueError(name)
    r[dst] = np.asarray(out, np.uint32)

def assert_faithful(ir, rtol=1e-5, atol=1e-6):
    """The lane program compiled from ``ir`` computes what the fragment oracle
    computes on the package's inputs (unwritten elements stay NaN in both)."""
    import json

    from lazy_compiler_b200.compiler import compile_file
    from oracle import expressions as O
    from oracle import fragment_ir

    plan = compile_file(ir)
    assert plan["op"] == "pointwise" and plan["params"].get("lanes"), plan["op"]
    meta = json.loads((ir.parent / "meta.json").read_text())
    arrays = {a["name"]: O.input_array(a, 0) for a in meta["kernels"][0]["args"] if not a.get("output")}
    ref = fragment_ir.evaluate(ir, arrays)
    got = run(plan["params"]["program"], arrays)
    for key, value in ref.items():
        np.testing.assert_allclose(got[key].reshape(value.shape), value, rtol=rtol, atol=atol, equal_nan=True)
    return plan


def run_rows(prog: dict, layout: dict, arrays: dict, block: int | None = None) -> dict:
    """A row program on the CPU, as its schedule runs it: every thread of the
    Tile's ``threads``-wide CTA folds its strided columns into its partials in
    column order; the partials combine through the warp operations at each
    level of a lane butterfly (xor 16 ... 1), then lane 0 of each warp through
    the tree operations pairwise, halving (warp i with warp i + d); the final
    operations run once per row."""
    block = block or layout.get("threads", 128)
    *row_ext, cols = prog["extents"]
    rows = int(np.prod(row_ext))
    states, outs = {}, {}
    grids = np.meshgrid(*[np.arange(e, dtype=np.int64) for e in row_ext], indexing="ij")
    row_coords = [g.ravel() for g in grids]
    r_coords = [np.repeat(rc, block) for rc in row_coords]
    t_idx = np.tile(np.arange(block, dtype=np.int64), rows)
    per_row = row_coords + [np.zeros(rows, np.int64)]
    lanes = np.arange(rows * block, dtype=np.int64)

    def sub(b, e):
        return dict(prog, code=prog["code"][b:e])

    for p, (b, e) in enumerate(layout["passes"]):
        slots = [k for k, ps in enumerate(layout["state_pass"]) if ps == p]
        partials = {k: np.full(rows * block, np.uint32(layout["state_init"][k]), np.uint32).view(np.float32)
                    for k in slots}
        wide = {k: np.repeat(np.asarray(v, np.float32), block) for k, v in states.items()}
        for it in range(-(-cols // block)):
            c = it * block + t_idx
            run(sub(b, e), arrays, coords=r_coords + [np.minimum(c, cols - 1)], states=wide, partials=partials,
                mask=c < cols, outs=outs)
        if slots:
            wb, we = layout["warp"][p]
            for o in (16, 8, 4, 2, 1):
                partner = {k: partials[k][lanes ^ o] for k in slots}
                run(sub(wb, we), arrays, coords=r_coords + [np.zeros(rows * block, np.int64)], states=wide,
                    partials=partials, partners=partner, outs=outs)
            tb, te = layout["tree"][p]
            nwarps = block // 32
            part = {k: partials[k].reshape(rows, block)[:, ::32].copy() for k in slots}
            d = nwarps // 2
            while d:
                for i in range(d):
                    own = {k: part[k][:, i].copy() for k in slots}
                    other = {k: part[k][:, i + d] for k in slots}
                    run(sub(tb, te), arrays, coords=per_row, states=states, partials=own, partners=other, outs=outs)
                    for k in slots:
                        part[k][:, i] = own[k]
                d //= 2
            states.update({k: part[k][:, 0].copy() for k in slots})
    fb, fe = layout["final"]
    run(sub(fb, fe), arrays, coords=per_row, states=states, partials={}, outs=outs)
    return outs


def run_block(prog: dict, layout: dict, arrays: dict) -> dict:
    """A block program on the CPU: every thread of every block in lockstep,
    one operation at a time, with an active mask for control flow (forward
    branches park the threads that jump until the target; a loop repeats its
    body for the threads still in range), per-block shared arrays (filled
    with NaN, so a read of an element nothing wrote shows in the result) and
    barriers as no-ops (lockstep already orders every access)."""
    ext = [int(e) for e in prog["extents"]]
    nb, T = layout["n_block_axes"], layout["threads"]
    blocks = int(np.prod(ext[:nb])) if nb else 1
    n = blocks * T
    blk = np.repeat(np.arange(blocks, dtype=np.int64), T)
    tid = np.tile(np.arange(T, dtype=np.int64), blocks)
    coords = []
    for values, axes in ((blk, ext[:nb]), (tid, ext[nb:])):
        rest, parts = values.copy(), []
        for e in reversed(axes):
            parts.append(rest % e)
            rest //= e
        coords += list(reversed(parts))
    loops = list(prog.get("loops", []))
    n_axes = len(coords)
    coords += [np.zeros(n, np.int64) for _ in loops]
    words = max([off + size for off, size in layout["smem"]] + [1])
    smem = np.full((blocks, words), np.float32(np.nan)).view(np.uint32)
    bufs = []
    for name, size in zip(prog["buffers"], prog["sizes"]):
        if name in arrays:
            a = np.asarray(arrays[name]).ravel()
            bufs.append(a.astype(np.float32) if a.dtype == np.float16 else a.copy())
        else:
            bufs.append(None)
    outs: dict = {}
    r: dict = {}
    consts = np.asarray(prog["consts"], np.uint64).astype(np.uint32)
    code = prog["code"]
    active = np.ones(n, bool)
    pending: dict = {}
    no_value = ("ST_", "STX_", "SETP")
    pc = 0
    with np.errstate(all="ignore"):
        while pc < len(code):
            if pc in pending:
                active = active | pending.pop(pc)
            op, dst, a, b, c, aux = code[pc]
            name = OPCODES[op]
            ia = r[a].view(np.int32).astype(np.int64) if a in r else np.zeros(n, np.int64)
            if name == "BRA":
                pending[aux] = pending.get(aux, np.zeros(n, bool)) | active
                active = np.zeros(n, bool)
            elif name == "BRZ":
                jump = active & (r[a] == 0)
                pending[aux] = pending.get(aux, np.zeros(n, bool)) | jump
                active = active & ~jump
            elif name == "SLB":
                d, end = n_axes + (aux & 15), aux >> 4
                limit = np.minimum(r[b].view(np.int32).astype(np.int64), loops[aux & 15])
                coords[d] = np.where(active, ia, coords[d])
                out = active & ((ia < 0) | (ia >= limit))
                pending[end + 1] = pending.get(end + 1, np.zeros(n, bool)) | out
                active = active & ~out
            elif name == "SLE":
                d, begin = n_axes + (aux & 15), aux >> 4
                limit = np.minimum(r[b].view(np.int32).astype(np.int64), loops[aux & 15])
                coords[d] = np.where(active, coords[d] + np.maximum(ia, 1), coords[d])
                again = active & (coords[d] < limit)
                pending[pc + 1] = pending.get(pc + 1, np.zeros(n, bool)) | (active & ~again)
                if again.any():
                    active = again
                    pc = begin + 1
                    continue
                active = np.zeros(n, bool)
            elif name in ("LDS", "STS"):
                off, size = layout["smem"][aux]
                if name == "LDS":
                    at = np.clip(ia, 0, size - 1)
                    value = smem[blk, off + at]
                    r[dst] = np.where(active, value, r.get(dst, np.zeros(n, np.uint32)))
                else:
                    ok = active & (ia >= 0) & (ia < size)
                    smem[blk[ok], off + ia[ok]] = r[b][ok]
            elif name == "TID":
                r[dst] = np.where(active, tid.astype(np.uint32), r.get(dst, np.zeros(n, np.uint32)))
            elif name in ("BAR", "WSYNC"):
                pass
            elif name in ("LOOPB", "LOOPE"):
                raise ValueError("counted loops are not part of block programs")
            else:
                old = r.get(dst)
                _step(prog, code[pc], r, coords, bufs, outs, consts, n, active, None, None, None)
                if not name.startswith(no_value):
                    r[dst] = np.where(active, r[dst], old if old is not None else np.zeros(n, np.uint32))
            pc += 1
    return outs
