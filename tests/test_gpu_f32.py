"""GPU parity of the FP32 GEMM (lc_gemm with LC_F32 operands) and the FP32
attention (lc_attention_f32) against the float64 oracle.

Tolerances (stated):
* f32 GEMM: every element within the classic dot-product bound
  |C - C_ref| <= 8 K 2^-24 (|A| |B|) + 1e-30 — the f32 FMA chain needs
  K 2^-24 (|A| |B|); the bf16-split tensor-core path adds at most
  4 2^-24 |a b| per product (representation and dropped products), so 8 K
  leaves room for both — and the normwise relative error below 1e-5;
* f32 attention: isclose(rtol=1e-4, atol=1e-5) elementwise against the
  float64 softmax (the IR's own packages carry rtol 1e-3, atol 1e-4).
"""
import ctypes

import numpy as np
import pytest

from lazy_compiler_b200 import runtime
from oracle import expressions as O

pytestmark = pytest.mark.gpu


def torch_():
    import torch
    return torch


def P(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def dev(a):
    torch = torch_()
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda")


def gemm_f32(a, b, layout, epi="none", bias=None, m=None, n=None, k=None):
    torch = torch_()
    m = a.shape[0]
    k = a.shape[1]
    n = b.shape[1] if layout == "kn" else b.shape[0]
    ta, tb = dev(a), dev(b)
    tbias = dev(bias) if bias is not None else None
    c = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    runtime.call("lc_gemm_ex", runtime.LC_F32, runtime.LC_F32, runtime.B_LAYOUTS[layout],
                 runtime.EPILOGUES[epi], P(ta), P(tb), P(tbias), P(c), m, n, k, None)
    runtime.call("lc_device_status", None)
    path = runtime.library().lc_gemm_path(runtime.LC_F32, runtime.B_LAYOUTS[layout], P(ta), P(tb), m, n, k)
    return c.cpu().numpy(), path


def check_gemm(got, a, b, layout, epi="none", bias=None):
    ref = O.gemm(a, b, layout, epi, "f32", "f32", bias)[0].astype(np.float64)
    bb = b if layout == "kn" else b.T
    k = a.shape[1]
    mag = np.abs(a.astype(np.float64)) @ np.abs(bb.astype(np.float64))
    bound = 8 * max(k, 1) * 2.0 ** -24 * mag + 1e-30
    if bias is not None or epi != "none":
        bound = bound + 2.0 ** -23 * (np.abs(ref) + 1e-30) + 8 * max(k, 1) * 2.0 ** -24 * mag
    err = np.abs(got.astype(np.float64) - ref)
    assert np.isfinite(got).all()
    assert (err <= bound).all(), float((err - bound).max())
    norm = np.linalg.norm(got - ref) / (np.linalg.norm(ref) or 1.0)
    assert norm < 1e-5, norm


def operands(m, n, k, layout, seed=0):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n) if layout == "kn" else (n, k)).astype(np.float32)
    return a, b


SIMT = [(1, 1, 1), (7, 5, 3), (33, 47, 65), (64, 64, 64), (128, 64, 256), (130, 257, 19),
        (512, 512, 512), (1, 300, 1000), (300, 1, 9)]


@pytest.mark.parametrize("m,n,k", SIMT)
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_f32_gemm_simt(m, n, k, layout, cuda_device):
    a, b = operands(m, n, k, layout)
    got, path = gemm_f32(a, b, layout)
    assert path == 0
    check_gemm(got, a, b, layout)


def test_f32_gemm_split_k_across_shapes(cuda_device):
    """Split-K calls of different shapes share the library's partial-product buffer and stay exact."""
    for m, n, k, layout, seed in [(512, 512, 512, "kn", 1), (64, 64, 4096, "nk", 2), (128, 64, 256, "kn", 3),
                                  (512, 512, 512, "kn", 4), (1, 300, 1000, "kn", 5)]:
        a, b = operands(m, n, k, layout, seed=seed)
        got, path = gemm_f32(a, b, layout)
        assert path == 0
        check_gemm(got, a, b, layout)
        again, _ = gemm_f32(a, b, layout)
        assert np.array_equal(got, again)  # the fixed summation order makes it deterministic


@pytest.mark.parametrize("epi", ["gelu_erf", "gelu_tanh"])
def test_f32_gemm_bias_epilogue(epi, cuda_device):
    for m, n, k in [(33, 47, 65), (200, 100, 1500)]:  # the second splits the contraction
        a, b = operands(m, n, k, "kn", seed=3)
        bias = np.random.default_rng(4).standard_normal(n).astype(np.float32)
        got, _ = gemm_f32(a, b, "kn", epi, bias)
        check_gemm(got, a, b, "kn", epi, bias)


def test_f32_gemm_k_zero(cuda_device):
    a = np.zeros((5, 0), np.float32)
    b = np.zeros((0, 7), np.float32)
    torch = torch_()
    c = torch.full((5, 7), float("nan"), dtype=torch.float32, device="cuda")
    bias = dev(np.arange(7, dtype=np.float32))
    # k = 0: C = bias (an empty sum is 0); A and B may be null
    runtime.call("lc_gemm_ex", runtime.LC_F32, runtime.LC_F32, 0, 0, None, None, P(bias), P(c), 5, 7, 0, None)
    assert np.array_equal(c.cpu().numpy(), np.tile(np.arange(7, dtype=np.float32), (5, 1)))


SPLIT = [(1024, 1024, 1024, "kn"), (2048, 1536, 1024, "nk"), (1000, 2056, 1028, "kn"),
         (4096, 4096, 2048, "kn")]


@pytest.mark.parametrize("m,n,k,layout", SPLIT)
def test_f32_gemm_tensor_core_split(m, n, k, layout, cuda_device):
    a, b = operands(m, n, k, layout, seed=7)
    got, path = gemm_f32(a, b, layout)
    assert path in (1, 2)
    check_gemm(got, a, b, layout)


def test_f32_gemm_split_matches_simt_accuracy(cuda_device):
    """The bf16-split tensor-core path is f32-accurate: its normwise error against float64 is
    below 2e-6 and within 4x of the SIMT kernel's and of numpy's float32 matmul."""
    a, b = operands(1024, 1024, 1024, "kn", seed=11)
    got, path = gemm_f32(a, b, "kn")
    assert path in (1, 2)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    simt = np.zeros_like(ref)
    for r0 in range(0, 1024, 256):  # 256 x 1024 x 1024 is below the split threshold
        simt[r0:r0 + 256], p = gemm_f32(a[r0:r0 + 256], b, "kn")
        assert p == 0
    e_split = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    e_simt = np.linalg.norm(simt - ref) / np.linalg.norm(ref)
    e_np32 = np.linalg.norm((a @ b).astype(np.float64) - ref) / np.linalg.norm(ref)
    assert e_split < 2e-6, e_split
    assert e_split < 4 * max(e_simt, e_np32), (e_split, e_simt, e_np32)


@pytest.mark.parametrize("bad", [np.inf, -np.inf, np.nan, 3.3999e38])
def test_f32_gemm_split_nonfinite_falls_back(bad, cuda_device):
    """A value whose bf16 hi piece is not finite reruns the product in plain f32."""
    m = n = k = 1024
    a, b = operands(m, n, k, "kn", seed=5)
    a[17, 3] = bad
    if bad == 3.3999e38:
        b[3, :] = 1e-30  # keeps the products finite
    got, path = gemm_f32(a, b, "kn")
    assert path in (1, 2)
    with np.errstate(all="ignore"):
        ref = (a.astype(np.float64) @ b.astype(np.float64))
    other = np.ones(m, bool)
    other[17] = False
    assert np.isfinite(got[other]).all()
    if np.isfinite(bad):
        assert np.isfinite(got).all()
        assert np.allclose(got, ref, rtol=1e-4, atol=1e-3)
    else:
        assert np.array_equal(np.isnan(got[17]), np.isnan(ref[17]))
        assert np.array_equal(np.isinf(got[17]), np.isinf(ref[17]))


# ---------------------------------------------------------------- attention

def attention(q, kt, v, scale, mode, epi="none"):
    torch = torch_()
    bh, s_q, d = q.shape
    s_kv, dv = v.shape[1], v.shape[2]
    o = torch.full((bh, s_q, dv), float("nan"), dtype=torch.float32, device="cuda")
    c = dev(np.array([scale], np.float32))
    tq, tkt, tv = dev(q), dev(kt), dev(v)  # kept alive across the launch
    runtime.call("lc_attention_f32", runtime.SCALE_MODES[mode], runtime.EPILOGUES[epi], P(c),
                 P(tq), P(tkt), P(tv), P(o), bh, s_q, s_kv, d, dv, None)
    runtime.call("lc_device_status", None)
    return o.cpu().numpy()


ATT = [(1, 64, 64, 64, 64), (1, 128, 128, 32, 32), (1, 11, 37, 17, 13), (3, 100, 200, 128, 128),
       (2, 65, 1, 8, 100), (1, 300, 513, 96, 64), (1, 5, 9, 160, 33), (1, 7, 11, 32, 200)]


@pytest.mark.parametrize("bh,s_q,s_kv,d,dv", ATT)
@pytest.mark.parametrize("mode", ["mul", "mul_recip", "div"])
def test_attention_f32(bh, s_q, s_kv, d, dv, mode, cuda_device):
    rng = np.random.default_rng(bh * 1000 + s_q)
    q = rng.standard_normal((bh, s_q, d)).astype(np.float32)
    kt = rng.standard_normal((bh, d, s_kv)).astype(np.float32)
    v = rng.standard_normal((bh, s_kv, dv)).astype(np.float32)
    scale = {"mul": 0.125, "mul_recip": 8.0, "div": 5.656854}[mode]
    got = attention(q, kt, v, scale, mode)
    ref = O.attention_f32(q, kt, v, scale, mode)[0]
    assert np.isclose(got, ref, rtol=1e-4, atol=1e-5).all(), float(np.abs(got - ref).max())


@pytest.mark.parametrize("epi", ["gelu_erf", "gelu_tanh"])
def test_attention_f32_epilogue(epi, cuda_device):
    rng = np.random.default_rng(9)
    q = rng.standard_normal((2, 11, 17)).astype(np.float32)
    kt = rng.standard_normal((2, 17, 37)).astype(np.float32)
    v = rng.standard_normal((2, 37, 13)).astype(np.float32)
    got = attention(q, kt, v, 0.125, "mul", epi)
    ref = O.attention_f32(q, kt, v, 0.125, "mul", epi)[0]
    assert np.isclose(got, ref, rtol=1e-4, atol=1e-5).all()


def test_attention_f32_zero_keys_is_nan(cuda_device):
    """An empty softmax divides 0 by 0, as the reference's acc * (1/sum) does."""
    q = np.ones((1, 4, 8), np.float32)
    got = attention(q, np.zeros((1, 8, 0), np.float32), np.zeros((1, 0, 8), np.float32), 1.0, "mul")
    assert np.isnan(got).all()


def test_attention_f32_bad_arguments(cuda_device):
    lib = runtime.library()
    assert lib.lc_attention_f32(7, 0, None, None, None, None, None, 1, 1, 1, 1, 1, None) == -1
    assert lib.lc_attention_f32(0, 0, None, None, None, None, None, 1, 1, 1, 1, 1, None) == -1
    assert lib.lc_attention_f32(0, 0, None, None, None, None, None, 0, 5, 5, 5, 5, None) == 0
