"""GPU parity of lc_gemm (tcgen05 path and SIMT path) against the oracle.

Tolerance for f16/bf16 GEMM (stated): isclose(rtol=2e-2, atol=2e-2 * rms(ref))
elementwise, plus a normwise relative error bound.  With f32 output the
kernel accumulates in f32 over exactly quantised operands, so the normwise
error against the float64 oracle is also held to 1e-5.
"""
import ctypes

import numpy as np
import pytest

from conftest import golden, golden_meta
from lazy_compiler_b200 import runtime
from lazy_compiler_b200.runner import run_package
from oracle import expressions as O

pytestmark = pytest.mark.gpu

RTOL = 2e-2


def torch_():
    import torch
    return torch


def P(t):
    return ctypes.c_void_p(t.data_ptr())


TD = {"f16": "float16", "bf16": "bfloat16", "f32": "float32"}


def run_gemm(a, b, ab, out, layout, epi, m, n, k):
    torch = torch_()
    c = torch.full((m, n), float("nan"), dtype=getattr(torch, TD[out]), device="cuda")
    runtime.call("lc_gemm", runtime.DTYPE_CODES[ab], runtime.DTYPE_CODES[out], runtime.B_LAYOUTS[layout],
                 runtime.EPILOGUES[epi], P(a), P(b), P(c), m, n, k, None)
    runtime.call("lc_device_status", None)
    return c


def check(got, ref, out_kind, f32_norm=1e-5):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(got).all()
    rms = float(np.sqrt(np.mean(ref ** 2))) or 1.0
    assert np.isclose(got, ref, rtol=RTOL, atol=RTOL * rms).all()
    norm = np.linalg.norm(got - ref) / (np.linalg.norm(ref) or 1.0)
    bound = f32_norm if out_kind == "f32" else 5e-3
    assert norm < bound, norm


def operands(m, n, k, ab, layout, seed=0):
    torch = torch_()
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.standard_normal((k, n) if layout == "kn" else (n, k)) / np.sqrt(k)).astype(np.float32)
    dt = getattr(torch, TD[ab])
    ta, tb = torch.from_numpy(a).to("cuda", dt), torch.from_numpy(b).to("cuda", dt)
    return a, b, ta, tb


@pytest.mark.parametrize("name", ["phase9_half_gelu_gemm", "generated_tensor"])
def test_golden_tensor_packages(name, cuda_device):
    meta = golden_meta(name)
    out = run_package(golden(name))
    with np.load(golden(name) / "expected.npz") as z:
        for key in z.files:
            row = O.compare(out[key], z[key], meta["rtol"], meta["atol"])
            assert row["pass"], row


SMALL = [(1, 1, 1), (11, 19, 7), (17, 21, 33), (64, 64, 16), (5, 300, 40)]


@pytest.mark.parametrize("m,n,k", SMALL)
@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_simt_path(m, n, k, layout, cuda_device):
    a, b, ta, tb = operands(m, n, k, "f16", layout)
    assert runtime.library().lc_gemm_path(1, runtime.B_LAYOUTS[layout], P(ta), P(tb), m, n, k) == 0
    for epi in ("none", "gelu_erf", "gelu_tanh"):
        c = run_gemm(ta, tb, "f16", "f32", layout, epi, m, n, k)
        ref = O.gemm(a, b, layout, epi, "f16", "f32")[0]
        check(c.cpu().numpy(), ref, "f32", 1e-4)


TC = [(256, 256, 256), (128, 256, 512), (333, 520, 200), (1024, 1024, 1024), (640, 1280, 4096),
      (2000, 264, 136), (1024, 1024, 64), (1100, 1304, 520), (2048, 1536, 2048)]


@pytest.mark.parametrize("m,n,k,path", [(256, 256, 256, 1), (1024, 1024, 256, 2), (4096, 4096, 64, 2),
                                        (128, 8192, 1024, 1)])
def test_path_selection(m, n, k, path, cuda_device):
    _, _, ta, tb = operands(8, 8, 16, "f16", "kn")
    assert runtime.library().lc_gemm_path(1, 0, P(ta), P(tb), m, n, k) == path


@pytest.mark.parametrize("m,n,k", TC)
@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("ab", ["f16", "bf16"])
def test_tcgen05_path(m, n, k, layout, ab, cuda_device):
    a, b, ta, tb = operands(m, n, k, ab, layout, seed=m + n + k)
    assert runtime.library().lc_gemm_path(runtime.DTYPE_CODES[ab], runtime.B_LAYOUTS[layout],
                                          P(ta), P(tb), m, n, k) >= 1
    c = run_gemm(ta, tb, ab, "f32", layout, "none", m, n, k)
    ref = O.gemm(a, b, layout, "none", ab, "f32")[0]
    check(c.cpu().numpy(), ref, "f32")


@pytest.mark.parametrize("epi", ["gelu_erf", "gelu_tanh"])
@pytest.mark.parametrize("out", ["f32", "f16", "bf16"])
def test_tcgen05_epilogues_and_outputs(epi, out, cuda_device):
    m, n, k = 384, 512, 320
    a, b, ta, tb = operands(m, n, k, "f16", "kn", seed=3)
    c = run_gemm(ta, tb, "f16", out, "kn", epi, m, n, k)
    ref = O.gemm(a, b, "kn", epi, "f16", out)[0]
    check(c.float().cpu().numpy(), ref, out)


def test_tcgen05_unfused_output_types(cuda_device):
    m, n, k = 256, 384, 256
    a, b, ta, tb = operands(m, n, k, "bf16", "nk", seed=4)
    for out in ("f16", "bf16"):
        c = run_gemm(ta, tb, "bf16", out, "nk", "none", m, n, k)
        check(c.float().cpu().numpy(), O.gemm(a, b, "nk", "none", "bf16", out)[0], out)


def test_tcgen05_repeated_calls_are_identical(cuda_device):
    m, n, k = 512, 768, 1024
    _, _, ta, tb = operands(m, n, k, "f16", "kn", seed=5)
    c1 = run_gemm(ta, tb, "f16", "f32", "kn", "none", m, n, k)
    c2 = run_gemm(ta, tb, "f16", "f32", "kn", "none", m, n, k)
    assert torch_().equal(c1, c2)


@pytest.mark.parametrize("cfg", [("f16", 8192, 8192, 8192), ("bf16", 4096, 16384, 2048)])
def test_config_size_against_torch_fp32_and_sampled_oracle(cfg, cuda_device):
    """The GEMM configurations at full size: A,B ~ N(0, 1/sqrt(K)), f32 output."""
    torch = torch_()
    ab, m, n, k = cfg
    g = torch.Generator(device="cuda").manual_seed(11)
    dt = getattr(torch, TD[ab])
    ta = (torch.randn(m, k, device="cuda", generator=g) / k ** 0.5).to(dt)
    tb = (torch.randn(k, n, device="cuda", generator=g) / k ** 0.5).to(dt)
    c = run_gemm(ta, tb, ab, "f32", "kn", "none", m, n, k)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = ta.float() @ tb.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    rms = ref.pow(2).mean().sqrt()
    assert torch.isclose(c, ref, rtol=RTOL, atol=float(RTOL * rms)).all()
    assert float((c - ref).norm() / ref.norm()) < 1e-5
    rng = np.random.default_rng(0)
    rows = rng.integers(0, m, 64)
    a64 = ta[torch.from_numpy(rows).cuda()].double().cpu().numpy()
    b64 = tb.double().cpu().numpy()
    ref_rows = a64 @ b64
    got = c[torch.from_numpy(rows).cuda()].double().cpu().numpy()
    np.testing.assert_allclose(got, ref_rows, rtol=1e-4, atol=1e-4 * float(np.sqrt(np.mean(ref_rows ** 2))))
