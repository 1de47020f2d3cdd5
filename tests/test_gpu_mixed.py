"""GPU parity of lc_gemm_mixed (operands stored as f32/f16/bf16, rounded to
the f16/bf16 MMA type) and lc_gemm_chain against the float64 oracle.

Tolerance (stated): the operands are rounded exactly like the oracle rounds
them, so the products are exact and only the f32 accumulation differs:
|C - C_ref| <= 8 K 2^-24 (|Q(A)| |Q(B)|) elementwise, plus one rounding of the
output type (2^-11 relative for f16, 2^-8 for bf16) and 2^-22 relative for
the epilogue's f32 arithmetic.  The chain's f32 intermediate can round to
the neighbouring 16-bit value where the two accumulation orders straddle a
rounding boundary, so the chain is checked elementwise at 2e-2 of the output
scale and, for at least 99% of the elements, at 1e-4.
"""
import ctypes

import numpy as np
import pytest

from lazy_compiler_b200 import runtime
from oracle import expressions as O

pytestmark = pytest.mark.gpu

CODES = runtime.DTYPE_CODES


def torch_():
    import torch
    return torch


def tdt(kind):
    torch = torch_()
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[kind]


def to_dev(a, kind):
    torch = torch_()
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to("cuda").to(tdt(kind))


def host(t):
    torch = torch_()
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def P(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def operands(m, n, k, layout, a_type, b_type, seed):
    rng = np.random.default_rng(seed)
    a = O.quantize(rng.standard_normal((m, k)).astype(np.float32), a_type)
    b = O.quantize(rng.standard_normal((k, n) if layout == "kn" else (n, k)).astype(np.float32), b_type)
    return a, b


def run_mixed(a, b, mma, a_type, b_type, c_type, layout, epi="none", bias=None, transpose=False,
              accumulate=False, c_init=None):
    torch = torch_()
    m, k = a.shape
    n = b.shape[1] if layout == "kn" else b.shape[0]
    ta, tb = to_dev(a, a_type), to_dev(b, b_type)
    tbias = to_dev(bias, "f32") if bias is not None else None
    shape = (n, m) if transpose else (m, n)
    if c_init is not None:
        c = to_dev(c_init, c_type)
    else:
        c = torch.full(shape, float("nan"), device="cuda", dtype=tdt(c_type))
    flags = (runtime.LC_GEMM_TRANSPOSE_C if transpose else 0) | (runtime.LC_GEMM_ACCUMULATE if accumulate else 0)
    runtime.call("lc_gemm_mixed", CODES[mma], CODES[a_type], CODES[b_type], CODES[c_type],
                 runtime.B_LAYOUTS[layout], runtime.EPILOGUES[epi], flags, P(ta), P(tb), P(tbias), P(c),
                 m, n, k, None)
    return host(c)


def check(got, a, b, layout, mma, c_type, epi="none", bias=None, transpose=False, base=None):
    ref = O.gemm(a, b, layout, epi, mma, "f32", bias, transpose)[0].astype(np.float64)
    qa = O.quantize(a, mma).astype(np.float64)
    qb = O.quantize(b, mma).astype(np.float64)
    bb = qb if layout == "kn" else qb.T
    mag = np.abs(qa) @ np.abs(bb)
    if transpose:
        mag = mag.T
    k = a.shape[1]
    bound = 8 * max(k, 1) * 2.0 ** -24 * mag + 2.0 ** -22 * np.abs(ref) + 1e-30
    if base is not None:
        ref = ref + base
        bound = bound + 2.0 ** -23 * np.abs(ref)
    if c_type != "f32":
        bound = bound + {"f16": 2.0 ** -11, "bf16": 2.0 ** -8}[c_type] * np.abs(ref) + 6e-8
    err = np.abs(got.astype(np.float64) - ref)
    assert np.isfinite(got).all()
    assert (err <= bound).all(), float((err - bound).max())


SMALL = [(1, 1, 1), (11, 7, 19), (16, 8, 16), (33, 47, 65), (64, 100, 3)]
LARGE = [(512, 384, 256), (1000, 520, 136)]   # at least 2^24 multiply-adds: the tcgen05 path


@pytest.mark.parametrize("m,n,k", SMALL + LARGE)
@pytest.mark.parametrize("mma", ["f16", "bf16"])
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_mixed_f32_operands(m, n, k, mma, layout, cuda_device):
    a, b = operands(m, n, k, layout, "f32", "f32", seed=m + n + k)
    got = run_mixed(a, b, mma, "f32", "f32", "f32", layout)
    check(got, a, b, layout, mma, "f32")


@pytest.mark.parametrize("a_type,b_type", [("f16", "f32"), ("f32", "bf16"), ("f16", "f16"), ("bf16", "f16")])
@pytest.mark.parametrize("m,n,k", [(33, 47, 65), (512, 384, 256)])
def test_mixed_storage_types(a_type, b_type, m, n, k, cuda_device):
    for mma in ("f16", "bf16"):
        a, b = operands(m, n, k, "kn", a_type, b_type, seed=5)
        got = run_mixed(a, b, mma, a_type, b_type, "f32", "kn")
        check(got, a, b, "kn", mma, "f32")


@pytest.mark.parametrize("m,n,k", [(11, 7, 19), (512, 384, 256)])
@pytest.mark.parametrize("epi", ["relu", "gelu_erf", "gelu_tanh", "none"])
@pytest.mark.parametrize("transpose", [False, True])
def test_mixed_store_variants(m, n, k, epi, transpose, cuda_device):
    a, b = operands(m, n, k, "kn", "f32", "f32", seed=3)
    bias = np.random.default_rng(4).standard_normal(n).astype(np.float32)
    got = run_mixed(a, b, "f16", "f32", "f32", "f32", "kn", epi, bias, transpose)
    check(got, a, b, "kn", "f16", "f32", epi, bias, transpose)


@pytest.mark.parametrize("c_type", ["f16", "bf16"])
def test_mixed_16bit_outputs(c_type, cuda_device):
    for m, n, k in [(33, 47, 65), (512, 384, 256)]:
        a, b = operands(m, n, k, "nk", "f32", "f32", seed=8)
        got = run_mixed(a, b, "bf16", "f32", "f32", c_type, "nk", transpose=True)
        check(got, a, b, "nk", "bf16", c_type, transpose=True)


@pytest.mark.parametrize("m,n,k", [(16, 8, 16), (512, 384, 256)])
def test_mixed_accumulate_adds_into_c(m, n, k, cuda_device):
    a, b = operands(m, n, k, "kn", "f32", "f32", seed=9)
    base = np.random.default_rng(10).standard_normal((m, n)).astype(np.float32)
    got = run_mixed(a, b, "f16", "f32", "f32", "f32", "kn", accumulate=True, c_init=base)
    check(got, a, b, "kn", "f16", "f32", base=base.astype(np.float64))
    zero = np.zeros((m, n), np.float32)
    got0 = run_mixed(a, b, "f16", "f32", "f32", "f32", "kn", accumulate=True, c_init=zero)
    check(got0, a, b, "kn", "f16", "f32")


def test_mixed_k_zero_is_epilogue_of_bias(cuda_device):
    torch = torch_()
    bias = to_dev(np.arange(5, dtype=np.float32) - 2, "f32")
    c = torch.full((3, 5), float("nan"), device="cuda")
    runtime.call("lc_gemm_mixed", CODES["f16"], CODES["f32"], CODES["f32"], CODES["f32"], 0,
                 runtime.EPILOGUES["relu"], 0, None, None, P(bias), P(c), 3, 5, 0, None)
    assert np.array_equal(host(c), np.tile(np.maximum(np.arange(5) - 2, 0).astype(np.float32), (3, 1)))


def test_mixed_bad_arguments(cuda_device):
    lib = runtime.library()
    args = (None, None, None, None, 4, 4, 4, None)
    assert lib.lc_gemm_mixed(CODES["f32"], 0, 0, 0, 0, 0, 0, *args) == -1                 # f32 MMA
    assert lib.lc_gemm_mixed(CODES["f16"], 0, 0, CODES["f16"], 0, 0, runtime.LC_GEMM_ACCUMULATE, *args) == -1
    assert lib.lc_gemm_mixed(CODES["f16"], 0, 0, 0, 0, 9, 0, *args) == -1                  # epilogue
    assert lib.lc_gemm_mixed(CODES["f16"], 0, 0, 0, 0, 0, 8, *args) == -1                  # flags
    assert lib.lc_gemm_mixed(CODES["f16"], 0, 0, 0, 0, 0, 0, *args) == -1                  # null buffers


# ---------------------------------------------------------------- chain

def run_chain(x, y, z, mma, y_layout="kn", z_layout="kn", c_type="f32"):
    torch = torch_()
    m, k = x.shape
    n1 = y.shape[1] if y_layout == "kn" else y.shape[0]
    n2 = z.shape[1] if z_layout == "kn" else z.shape[0]
    tx, ty, tz = to_dev(x, "f32"), to_dev(y, "f32"), to_dev(z, "f32")
    c = torch.full((m, n2), float("nan"), device="cuda", dtype=tdt(c_type))
    runtime.call("lc_gemm_chain", CODES[mma], CODES["f32"], CODES["f32"], CODES["f32"], CODES[c_type],
                 runtime.B_LAYOUTS[y_layout], runtime.B_LAYOUTS[z_layout], P(tx), P(ty), P(tz), P(c),
                 m, k, n1, n2, None)
    return host(c)


@pytest.mark.parametrize("m,k,n1,n2", [(16, 16, 16, 8), (37, 29, 41, 13), (512, 256, 384, 256)])
@pytest.mark.parametrize("mma", ["f16", "bf16"])
def test_chain(m, k, n1, n2, mma, cuda_device):
    rng = np.random.default_rng(m + k)
    x = rng.standard_normal((m, k)).astype(np.float32) / np.sqrt(k)
    y = rng.standard_normal((k, n1)).astype(np.float32)
    z = rng.standard_normal((n1, n2)).astype(np.float32) / np.sqrt(n1)
    got = run_chain(x, y, z, mma)
    ref = O.gemm_chain_f16(x, y, z, mma)[0]
    scale = float(np.abs(ref).max())
    assert np.allclose(got, ref, rtol=2e-2, atol=2e-2 * scale), float(np.abs(got - ref).max())
    # almost every element matches to f32 accumulation accuracy
    close = np.isclose(got, ref, rtol=1e-4, atol=1e-4 * scale)
    assert close.mean() > 0.99, close.mean()


def test_chain_transposed_operands(cuda_device):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((40, 24)).astype(np.float32)
    y = rng.standard_normal((32, 24)).astype(np.float32)      # [n1, k]
    z = rng.standard_normal((16, 32)).astype(np.float32)      # [n2, n1]
    got = run_chain(x, y, z, "f16", "nk", "nk")
    ref = O.gemm_chain_f16(x, y, z, "f16", "nk", "nk")[0]
    assert np.allclose(got, ref, rtol=2e-2, atol=2e-2 * float(np.abs(ref).max()))
