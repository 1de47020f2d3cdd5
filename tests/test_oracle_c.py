"""The C restatement of the oracle (CPU baseline) agrees with the numpy oracle."""
import ctypes
import subprocess

import numpy as np
import pytest

from conftest import ROOT
from oracle import expressions as O

LIB = ROOT / "oracle" / "_build" / "liboracle.so"


@pytest.fixture(scope="module")
def oc():
    subprocess.run(["make", "-s", "-C", str(ROOT / "oracle")], check=True)
    lib = ctypes.CDLL(str(LIB))
    lib.oc_sum.restype = ctypes.c_double
    return lib


def ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_pointwise(oc):
    n = 100_003
    x = O.normal(n, 0)
    y = O.normal(n, 1)
    out = np.empty_like(x)
    oc.oc_add(ptr(x), ptr(y), ptr(out), ctypes.c_int64(n))
    np.testing.assert_array_equal(out, O.add(x, y)[0])
    oc.oc_axpb(ctypes.c_float(1.5), ctypes.c_float(-0.25), ptr(x), ptr(out), ctypes.c_int64(n))
    np.testing.assert_array_equal(out, O.axpb(1.5, -0.25, x)[0])
    oc.oc_relumul(ptr(x), ptr(y), ptr(out), ctypes.c_int64(n))
    np.testing.assert_array_equal(out, O.relumul(x, y)[0])
    xs = x[:5000]
    for mode, approx in ((0, "none"), (1, "tanh")):
        o = np.empty_like(xs)
        oc.oc_gelu(mode, ptr(xs), ptr(o), ctypes.c_int64(xs.size))
        np.testing.assert_allclose(o, O.gelu(xs, approx), rtol=1e-6, atol=1e-7)


def test_sum_and_rows(oc):
    x = O.uniform(1 << 20, 0)
    assert np.float32(oc.oc_sum(ptr(x), ctypes.c_int64(x.size))) == O.sum_(x)[0]
    X = O.normal((37, 300), 2)
    w = O.normal((300,), 3, mean=1.0, std=0.1)
    out = np.empty_like(X)
    rs = np.empty(37, np.float32)
    oc.oc_rowsum(ptr(X), ptr(rs), ctypes.c_int64(37), ctypes.c_int64(300))
    np.testing.assert_allclose(rs, O.rowsum(X)[0], rtol=1e-6)
    oc.oc_rmsnorm(ptr(X), ptr(w), ptr(out), ctypes.c_int64(37), ctypes.c_int64(300),
                  ctypes.c_double(1e-6), ctypes.c_double(300))
    np.testing.assert_allclose(out, O.rmsnorm(X, w, 1e-6)[0], rtol=1e-6)
    oc.oc_softmax(ptr(X), ptr(out), ctypes.c_int64(37), ctypes.c_int64(300))
    np.testing.assert_allclose(out, O.softmax(X)[0], rtol=1e-6)
    oc.oc_l2norm(ptr(X), ptr(out), ctypes.c_int64(37), ctypes.c_int64(300))
    np.testing.assert_allclose(out, O.l2norm(X)[0], rtol=1e-6)
