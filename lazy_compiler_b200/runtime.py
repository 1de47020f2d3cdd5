"""ctypes bindings of ``liblazyb200.so`` and the plan launcher.

This is the "thin Python ctypes C-ABI layer" of the drop-in boundary: it
takes the launch plan printed by ``compile.py`` and a mapping from meta.json
argument names to device pointers, and calls the C-ABI entry point the plan
names.  It plays the part of the reference's CUDA-driver launcher
(tools/check_compiler.py:291-422 ``CudaDriver.run``: module load,
cuLaunchKernel with `.u64` pointers in ``arg_order``), minus the PTX JIT:
the kernels are prebuilt for sm_100a.

There is no CPU fallback.  If the library is missing, :func:`library` raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "liblazyb200.so"

LC_F32, LC_F16, LC_BF16 = 0, 1, 2
DTYPE_CODES = {"f32": LC_F32, "f16": LC_F16, "bf16": LC_BF16}
EPILOGUES = {"none": 0, "gelu_erf": 1, "gelu_tanh": 2, "relu": 3}
LC_GEMM_TRANSPOSE_C, LC_GEMM_ACCUMULATE = 1, 2
B_LAYOUTS = {"kn": 0, "nk": 1}
SCALE_MODES = {"mul": 0, "mul_recip": 1, "div": 2}
STATUS = {0: "LC_OK", -1: "LC_ERR_INVALID", -2: "LC_ERR_ALIGN", -3: "LC_ERR_CUDA",
          -4: "LC_ERR_TIMEOUT", -5: "LC_ERR_UNSUPPORTED", -6: "LC_ERR_NOMEM"}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int
# name -> argument types (all return int status)
SIGNATURES = {
    "lc_version": [],
    "lc_last_error": [ctypes.c_char_p, ctypes.c_size_t],
    "lc_add_f32": [_P, _P, _P, _I64, _P],
    "lc_axpb_f32": [_P, _P, _P, _P, _I64, _P],
    "lc_relumul_f32": [_P, _P, _P, _I64, _P],
    "lc_gelu": [_INT, _INT, _P, _P, _I64, _P],
    "lc_sum_f32": [_P, _P, _I64, _P],
    "lc_mean_f32": [_P, _P, _P, _I64, _P],
    "lc_sum_f32_noalloc": [_P, _P, _I64, _P],
    "lc_sum_partial_f32": [_P, _I64, _P, _P],
    "lc_sum_finalize": [_P, _P, _P, _P],
    "lc_peer_mailbox": [ctypes.POINTER(_P), ctypes.c_char_p],
    "lc_peer_open": [ctypes.c_char_p, ctypes.POINTER(_P)],
    "lc_peer_close": [_P],
    "lc_peer_reset": [_P],
    "lc_sum_peer_f32": [_P, _I64, _P, _P, ctypes.POINTER(_P), _INT, _INT, _P],
    "lc_rowsum_f32": [_P, _P, _I64, _I64, _P],
    "lc_rmsnorm_f32": [_P, _P, _P, _P, _P, _I64, _I64, _P],
    "lc_softmax_f32": [_P, _P, _I64, _I64, _P],
    "lc_l2norm_f32": [_P, _P, _I64, _I64, _P],
    "lc_rowdot_f32": [_INT, _P, _P, _P, _I64, _I64, _P],
    "lc_gemm": [_INT, _INT, _INT, _INT, _P, _P, _P, _I64, _I64, _I64, _P],
    "lc_gemm_ex": [_INT, _INT, _INT, _INT, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "lc_gemm_path": [_INT, _INT, _P, _P, _I64, _I64, _I64],
    "lc_gemm_f32_dot2": [_INT, _INT, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "lc_attention_f32_dot2": [_INT, _INT, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "lc_pointwise": [_P, _P, _P],
    "lc_rowprog": [_P, _P, _P, _P],
    "lc_blockprog": [_P, _P, _P, _P],
    "lc_jit_blockprog": [_P, ctypes.c_size_t, _P, _P, _P, _P],
    "lc_jit_pointwise": [_P, ctypes.c_size_t, _P, _P, _P],
    "lc_jit_rowprog": [_P, ctypes.c_size_t, _P, _P, _P, _P],
    "lc_gemm_mixed": [_INT, _INT, _INT, _INT, _INT, _INT, _INT, _P, _P, _P, _P, _I64, _I64, _I64, _P],
    "lc_gemm_chain": [_INT, _INT, _INT, _INT, _INT, _INT, _INT, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P],
    "lc_attention_f32": [_INT, _INT, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "lc_attention_tile_f16q": [_P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _P],
    "lc_device_status": [_P],
    "lc_selftest_bounded_wait": [_I64, _P],
    "lc_sdpa_f16": [_P, _P, _P, _P, _I64, _I64, _I64, _I64, ctypes.c_float, _P],
    "lc_sdpa_path": [_P, _P, _P, _P, _I64, _I64, _I64],
}

# pointwise programs (include/lazyb200.h lc_pw_program)
LC_S32 = 3
STORAGE_CODES = {"f32": LC_F32, "f16": LC_F16, "bf16": LC_BF16, "s32": LC_S32}
PW_MAX_CODE, PW_MAX_CONST, PW_MAX_FORMS, PW_MAX_BUFFERS, PW_MAX_AXES = 2048, 128, 32, 16, 8


class PwForm(ctypes.Structure):
    _fields_ = [("base", ctypes.c_int64), ("coef", ctypes.c_int64 * PW_MAX_AXES),
                ("buffer", ctypes.c_int32), ("dtype", ctypes.c_int32)]


class PwProgram(ctypes.Structure):
    _fields_ = [("n_code", ctypes.c_int32), ("n_consts", ctypes.c_int32), ("n_forms", ctypes.c_int32),
                ("n_buffers", ctypes.c_int32), ("n_axes", ctypes.c_int32), ("n_regs", ctypes.c_int32),
                ("n_loops", ctypes.c_int32), ("reserved", ctypes.c_int32),
                ("extents", ctypes.c_int64 * PW_MAX_AXES), ("sizes", ctypes.c_int64 * PW_MAX_BUFFERS),
                ("code", (ctypes.c_uint32 * 2) * PW_MAX_CODE), ("consts", ctypes.c_uint32 * PW_MAX_CONST),
                ("forms", PwForm * PW_MAX_FORMS)]


def pw_program(prog: dict) -> PwProgram:
    """The C struct of a compiled pointwise program (a plan's ``params["program"]``)."""
    g = PwProgram()
    g.n_code, g.n_consts, g.n_forms = len(prog["code"]), len(prog["consts"]), len(prog["forms"])
    g.n_buffers, g.n_axes, g.n_regs = len(prog["buffers"]), len(prog["extents"]), max(1, prog["n_regs"])
    loops = prog.get("loops", [])
    g.n_loops = len(loops)
    for d, e in enumerate(list(prog["extents"]) + list(loops)):
        g.extents[d] = e
    for i, size in enumerate(prog["sizes"]):
        g.sizes[i] = size
    for i, (op, dst, a, b, c, aux) in enumerate(prog["code"]):
        g.code[i][0] = op | dst << 8 | a << 16 | b << 24
        g.code[i][1] = c | aux << 8
    for i, word in enumerate(prog["consts"]):
        g.consts[i] = word
    for i, f in enumerate(prog["forms"]):
        g.forms[i].base, g.forms[i].buffer, g.forms[i].dtype = f["base"], f["buffer"], STORAGE_CODES[f["dtype"]]
        for d, c in enumerate(f["coef"]):
            g.forms[i].coef[d] = c
    return g


RP_MAX_PASSES, RP_MAX_STATES = 4, 8


class RpLayout(ctypes.Structure):
    _fields_ = [("n_passes", ctypes.c_int32), ("n_states", ctypes.c_int32), ("final_begin", ctypes.c_int32),
                ("final_end", ctypes.c_int32), ("begin", ctypes.c_int32 * RP_MAX_PASSES),
                ("end", ctypes.c_int32 * RP_MAX_PASSES), ("warp_begin", ctypes.c_int32 * RP_MAX_PASSES),
                ("warp_end", ctypes.c_int32 * RP_MAX_PASSES), ("tree_begin", ctypes.c_int32 * RP_MAX_PASSES),
                ("tree_end", ctypes.c_int32 * RP_MAX_PASSES), ("state_init", ctypes.c_uint32 * RP_MAX_STATES),
                ("state_pass", ctypes.c_int32 * RP_MAX_STATES), ("threads", ctypes.c_int32)]


def rp_layout(layout: dict) -> RpLayout:
    """The C struct of a row program's layout (a plan's ``params["layout"]``)."""
    lay = RpLayout()
    lay.n_passes, lay.n_states = len(layout["passes"]), len(layout["state_pass"])
    lay.final_begin, lay.final_end = layout["final"]
    for i, ((b, e), (wb, we), (tb, te)) in enumerate(zip(layout["passes"], layout["warp"], layout["tree"])):
        lay.begin[i], lay.end[i] = b, e
        lay.warp_begin[i], lay.warp_end[i] = wb, we
        lay.tree_begin[i], lay.tree_end[i] = tb, te
    for k, (init, ps) in enumerate(zip(layout["state_init"], layout["state_pass"])):
        lay.state_init[k], lay.state_pass[k] = init, ps
    lay.threads = layout.get("threads", 256)
    return lay


BP_MAX_SMEM = 8


class BpLayout(ctypes.Structure):
    _fields_ = [("threads", ctypes.c_int32), ("n_block_axes", ctypes.c_int32), ("n_smem", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("smem_offset", ctypes.c_int32 * BP_MAX_SMEM),
                ("smem_size", ctypes.c_int32 * BP_MAX_SMEM)]


def bp_layout(layout: dict) -> BpLayout:
    """The C struct of a block program's layout (a plan's ``params["layout"]``)."""
    lay = BpLayout()
    lay.threads, lay.n_block_axes, lay.n_smem = layout["threads"], layout["n_block_axes"], len(layout["smem"])
    for i, (off, size) in enumerate(layout["smem"]):
        lay.smem_offset[i], lay.smem_size[i] = off, size
    return lay


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class LcError(RuntimeError):
    """A non-zero status from a C-ABI entry point."""

    def __init__(self, function: str, status: int, message: str):
        super().__init__(f"{function} returned {STATUS.get(status, status)}: {message}")
        self.function = function
        self.status = status
        self.message = message


def library() -> ctypes.CDLL:
    """Load ``liblazyb200.so`` once and bind every C-ABI signature.

    Raises ``RuntimeError`` when the library has not been built: the kernels
    are the only implementation.
    """
    global _lib
    with _lock:
        if _lib is None:
            if not LIBRARY_PATH.exists():
                raise RuntimeError(
                    f"{LIBRARY_PATH.name} is not built; run `python -m lazy_compiler_b200.build` "
                    "(there is no CPU fallback)")
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_int
            _lib = lib
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(512)
    library().lc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def call(name: str, *args) -> None:
    """Call one entry point and raise :class:`LcError` on a non-zero status."""
    status = getattr(library(), name)(*args)
    if status != 0:
        raise LcError(name, status, last_error())


_PREPARED: dict = {}


def _prepared(params: dict, build):
    """The C structs (and native module image) of a plan's program, built once
    per program: repeated launches of one plan skip rebuilding them."""
    key = id(params["program"])
    entry = _PREPARED.get(key)
    if entry is None or entry[0] is not params["program"]:
        entry = (params["program"], build())
        with _lock:
            if len(_PREPARED) >= 256:
                _PREPARED.pop(next(iter(_PREPARED)))
            _PREPARED[key] = entry
    return entry[1]


def _launch_point(params: dict, prog: dict, ptrs, s) -> None:
    """A pointwise or serial program: natively compiled when it can be, else interpreted."""
    def build():
        from . import jit
        cubin = jit.point_cubin(prog)
        image = ctypes.create_string_buffer(cubin, len(cubin)) if cubin is not None else None
        return pw_program(prog), None, image
    g, _, image = _prepared(params, build)
    if image is not None:
        call("lc_jit_pointwise", ctypes.cast(image, ctypes.c_void_p), len(image.raw),
             ctypes.c_void_p(ctypes.addressof(g)), ptrs, s)
    else:
        call("lc_pointwise", ctypes.c_void_p(ctypes.addressof(g)), ptrs, s)


def launch(plan: dict, pointers: dict, stream: int | None = None) -> None:
    """Launch the kernel a ``compile.py`` plan names.

    ``pointers`` maps meta.json argument names to device addresses (ints);
    ``stream`` is a cudaStream_t handle (``torch.cuda.current_stream().cuda_stream``)
    or ``None`` for the default stream.
    """
    b = plan["bind"]
    p = plan["params"]
    ptr = lambda role: ctypes.c_void_p(int(pointers[b[role]]))  # noqa: E731
    s = ctypes.c_void_p(stream or 0)
    op = plan["op"]
    if op == "add_f32":
        call("lc_add_f32", ptr("x0"), ptr("x1"), ptr("out"), p["n"], s)
    elif op == "axpb_f32":
        call("lc_axpb_f32", ptr("a"), ptr("b"), ptr("x"), ptr("out"), p["n"], s)
    elif op == "relumul_f32":
        call("lc_relumul_f32", ptr("x"), ptr("y"), ptr("out"), p["n"], s)
    elif op == "gelu":
        call("lc_gelu", DTYPE_CODES[plan["dtypes"]["io"]], 1 if p["approximate"] == "tanh" else 0,
             ptr("x"), ptr("out"), p["n"], s)
    elif op == "sum_f32":
        call("lc_sum_f32", ptr("x"), ptr("out"), p["n"], s)
    elif op == "mean_f32":
        call("lc_mean_f32", ptr("x"), ptr("count"), ptr("out"), p["n"], s)
    elif op == "rowsum_f32":
        call("lc_rowsum_f32", ptr("x"), ptr("out"), p["rows"], p["cols"], s)
    elif op == "rmsnorm_f32":
        call("lc_rmsnorm_f32", ptr("count"), ptr("eps"), ptr("x"), ptr("w"), ptr("out"),
             p["rows"], p["cols"], s)
    elif op == "softmax_f32":
        call("lc_softmax_f32", ptr("x"), ptr("out"), p["rows"], p["cols"], s)
    elif op == "l2norm_f32":
        call("lc_l2norm_f32", ptr("x"), ptr("out"), p["rows"], p["cols"], s)
    elif op == "rowdot_f32":
        call("lc_rowdot_f32", EPILOGUES[p["activation"]], ptr("x"), ptr("y"), ptr("out"), p["rows"],
             p["cols"], s)
    elif op == "gemm" and p.get("compensated"):
        bias = ptr("bias") if "bias" in b else ctypes.c_void_p(0)
        call("lc_gemm_f32_dot2", B_LAYOUTS[p["b_layout"]], EPILOGUES[p["epilogue"]], ptr("a"), ptr("b"), bias,
             ptr("c"), p["m"], p["n"], p["k"], s)
    elif op == "gemm":
        d = plan["dtypes"]
        bias = ptr("bias") if "bias" in b else ctypes.c_void_p(0)
        call("lc_gemm_ex", DTYPE_CODES[d["ab"]], DTYPE_CODES[d["c"]], B_LAYOUTS[p["b_layout"]],
             EPILOGUES[p["epilogue"]], ptr("a"), ptr("b"), bias, ptr("c"), p["m"], p["n"], p["k"], s)
    elif op == "pointwise":
        prog = p["program"]
        ptrs = (ctypes.c_void_p * PW_MAX_BUFFERS)(*[int(pointers[b[f"buf{i}"]]) for i in range(len(prog["buffers"]))])
        _launch_point(p, prog, ptrs, s)
    elif op == "rowprog":
        prog = p["program"]
        ptrs = (ctypes.c_void_p * PW_MAX_BUFFERS)(*[int(pointers[b[f"buf{i}"]]) for i in range(len(prog["buffers"]))])

        def build_rows():
            from . import jit
            cubin = jit.rows_cubin(prog, p["layout"])
            image = ctypes.create_string_buffer(cubin, len(cubin)) if cubin is not None else None
            return pw_program(prog), rp_layout(p["layout"]), image
        g, lay, image = _prepared(p, build_rows)
        if image is not None:
            call("lc_jit_rowprog", ctypes.cast(image, ctypes.c_void_p), len(image.raw),
                 ctypes.c_void_p(ctypes.addressof(g)), ctypes.c_void_p(ctypes.addressof(lay)), ptrs, s)
        else:
            call("lc_rowprog", ctypes.c_void_p(ctypes.addressof(g)), ctypes.c_void_p(ctypes.addressof(lay)), ptrs, s)
    elif op == "blockprog":
        prog = p["program"]
        ptrs = (ctypes.c_void_p * PW_MAX_BUFFERS)(*[int(pointers[b[f"buf{i}"]]) for i in range(len(prog["buffers"]))])

        def build():
            from . import jit
            cubin = jit.block_cubin(prog, p["layout"])
            image = ctypes.create_string_buffer(cubin, len(cubin)) if cubin is not None else None
            return pw_program(prog), bp_layout(p["layout"]), image
        g, lay, image = _prepared(p, build)
        if image is not None:
            call("lc_jit_blockprog", ctypes.cast(image, ctypes.c_void_p), len(image.raw),
                 ctypes.c_void_p(ctypes.addressof(g)), ctypes.c_void_p(ctypes.addressof(lay)), ptrs, s)
        else:
            call("lc_blockprog", ctypes.c_void_p(ctypes.addressof(g)), ctypes.c_void_p(ctypes.addressof(lay)), ptrs, s)
    elif op == "gemm_mixed":
        d = plan["dtypes"]
        bias = ptr("bias") if "bias" in b else ctypes.c_void_p(0)
        flags = (LC_GEMM_TRANSPOSE_C if p["transpose"] else 0) | (LC_GEMM_ACCUMULATE if p["accumulate"] else 0)
        call("lc_gemm_mixed", DTYPE_CODES[d["mma"]], DTYPE_CODES[d["a"]], DTYPE_CODES[d["b"]],
             DTYPE_CODES[d["c"]], B_LAYOUTS[p["b_layout"]], EPILOGUES[p["epilogue"]], flags, ptr("a"),
             ptr("b"), bias, ptr("c"), p["m"], p["n"], p["k"], s)
    elif op == "gemm_chain":
        d = plan["dtypes"]
        call("lc_gemm_chain", DTYPE_CODES[d["mma"]], DTYPE_CODES[d["x"]], DTYPE_CODES[d["y"]],
             DTYPE_CODES[d["z"]], DTYPE_CODES[d["c"]], B_LAYOUTS[p["y_layout"]], B_LAYOUTS[p["z_layout"]],
             ptr("x"), ptr("y"), ptr("z"), ptr("c"), p["m"], p["k"], p["n1"], p["n2"], s)
    elif op == "attention_f32":
        call("lc_attention_f32_dot2" if p.get("compensated") else "lc_attention_f32", SCALE_MODES[p["scale_mode"]], EPILOGUES[p["epilogue"]],
             ptr("scale"), ptr("q"), ptr("kt"), ptr("v"), ptr("o"), p["bh"], p["s_q"], p["s_kv"],
             p["d"], p["dv"], s)
    elif op == "attention_tile_f16q":
        call("lc_attention_tile_f16q", ptr("q"), ptr("kt"), ptr("v"), ptr("o"), p["bh"], p["s_q"], p["s_kv"],
             p["d"], p["dv"], s)
    elif op == "sdpa_f16":
        call("lc_sdpa_f16", ptr("q"), ptr("k"), ptr("v"), ptr("o"), p["bh"], p["s_q"], p["s_kv"],
             p["d"], ctypes.c_float(p["scale"]), s)
    else:
        raise ValueError(f"plan op {op!r} has no C-ABI entry point")
    if "post" in p:
        # an epilogue program over the result, in place, on the same stream
        post = p["post"]
        prog = post["program"]
        ptrs = (ctypes.c_void_p * PW_MAX_BUFFERS)(*[int(pointers[post["bind"][f"buf{i}"]])
                                                     for i in range(len(prog["buffers"]))])
        _launch_point(post, prog, ptrs, s)
