"""Dot2 known-answer cases on the B200: this backend and the reference's own PTX, both exact.

The seven packages of tests/golden/make_precision.py restate the reference's
exact-cancellation cases (tests/test_precision.py:39-188).  Each runs through
this backend's drop-in path (compile.py plan -> C ABI, natively compiled and
interpreted register programs) and as the reference's own PTX (its unchanged
compiler, default policy: compensated because meta.json states a tolerance);
both must return the exact integers bit for bit.
"""
import numpy as np
import pytest

from conftest import GOLDEN
from lazy_compiler_b200.runner import run_package
from oracle.ref_launch import RefKernel, manifest

pytestmark = pytest.mark.gpu

PRECISION = sorted(p.name for p in GOLDEN.glob("precision_*"))


def expected(name):
    with np.load(GOLDEN / name / "expected.npz") as z:
        return z["out"]


@pytest.mark.parametrize("jit", ["1", "0"])
@pytest.mark.parametrize("name", PRECISION)
def test_ours_exact_on_the_gpu(name, jit, cuda_device, monkeypatch):
    monkeypatch.setenv("LC_JIT", jit)
    got = run_package(GOLDEN / name)["out"]
    want = expected(name)
    np.testing.assert_array_equal(np.asarray(got).reshape(want.shape), want)


@pytest.mark.parametrize("name", PRECISION)
def test_reference_ptx_exact_on_the_gpu(name, cuda_device):
    if name not in manifest():
        pytest.skip("oracle/_ref has no reference PTX for this package")
    got = RefKernel(name).run()["out"]
    want = expected(name)
    np.testing.assert_array_equal(np.asarray(got).reshape(want.shape), want)


# ---------------------------------------------------------------- the fixed FP32 classes
# The reference's own matmul and attention packages, fed inputs built from the
# exact-cancellation pair of its precision tests: a = (4097, -4096) against
# b = (4097, 4098) contributes 4097^2 - 4096 * 4098 = 1 to a dot product,
# while separately rounded f32 products cancel to 0.  Which pairs meet is
# seeded, so every output is a different small integer.

def pair_operands(m, k, n, seed):
    """A [m, k], B [k, n] whose product is the count of meeting pairs (exact in f32 only with Dot2)."""
    rng = np.random.default_rng(seed)
    ma = rng.random((m, k // 2)) < 0.5
    mb = rng.random((k // 2, n)) < 0.5
    a = np.zeros((m, k), np.float32)
    b = np.zeros((k, n), np.float32)
    a[:, 0::2] = np.where(ma, 4097, 0)
    a[:, 1::2] = np.where(ma, -4096, 0)
    b[0::2, :] = np.where(mb, 4097, 0)
    b[1::2, :] = np.where(mb, 4098, 0)
    exact = ma.astype(np.int64) @ mb.astype(np.int64)
    return a, b, exact.astype(np.float32)


@pytest.mark.parametrize("name", ["m01_matmul_512", "m02_matmul_rect"])
def test_fixed_matmul_class_keeps_the_cancellation_exact(name, cuda_device):
    import json
    meta = json.loads((GOLDEN / name / "meta.json").read_text())
    shapes = {a["name"]: a["shape"] for a in meta["kernels"][0]["args"]}
    (m, k), (_, n) = shapes["x0"], shapes["x1"]
    a, b, exact = pair_operands(m, k, n, seed=len(name))
    got = run_package(GOLDEN / name, inputs={"x0": a, "x1": b})["matmul"]
    np.testing.assert_array_equal(got, exact)
    if name in manifest():
        ref = RefKernel(name).run({"x0": a, "x1": b})["matmul"]
        np.testing.assert_array_equal(ref, exact)


@pytest.mark.parametrize("name", ["a01_attention", "a02_attention_128"])
def test_fixed_attention_class_keeps_the_cancellation_exact(name, cuda_device):
    import ctypes
    import json

    import torch

    from lazy_compiler_b200 import runtime
    from oracle import expressions as O
    meta = json.loads((GOLDEN / name / "meta.json").read_text())
    args = {a["name"]: a for a in meta["kernels"][0]["args"]}
    (s_q, d), (_, s_kv), (_, dv) = args["q"]["shape"], args["kt"]["shape"], args["v"]["shape"]
    q, kt, scores = pair_operands(s_q, d, s_kv, seed=len(name))
    v = O.normal((s_kv, dv), 2)
    c = float(args["div_c1"]["data"][0])
    x = scores.astype(np.float64) / c
    p = np.exp(x - x.max(-1, keepdims=True))
    want = (p / p.sum(-1, keepdims=True)) @ v.astype(np.float64)
    got = run_package(GOLDEN / name, inputs={"q": q, "kt": kt, "v": v})["matmul_1"]
    assert O.compare(got, want.astype(np.float32), meta["rtol"], meta["atol"])["pass"]
    if name in manifest():
        ref = RefKernel(name).run({"q": q, "kt": kt, "v": v})["matmul_1"]
        assert O.compare(ref, want.astype(np.float32), meta["rtol"], meta["atol"])["pass"]
    # the same launch without compensation loses the scores (all dots round to 0)
    tq, tk, tv = (torch.from_numpy(t).cuda() for t in (q, kt, v))
    tc = torch.tensor([c], device="cuda")
    plain = torch.empty(s_q, dv, device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    runtime.call("lc_attention_f32", runtime.SCALE_MODES["div"], 0, P(tc), P(tq), P(tk), P(tv), P(plain),
                 1, s_q, s_kv, d, dv, None)
    assert not O.compare(plain.cpu().numpy(), want.astype(np.float32), meta["rtol"], meta["atol"])["pass"]
