"""The runner layer: meta.json kernel chaining through ``intermediate``
arguments (submit.py:112-122) and ``run_request``, the reference runner's
``POST /run`` request and response (docs/API.md:26-72) with a compiled plan
in place of PTX."""
import json

import numpy as np
import pytest

import pw_packages as W
from conftest import golden, golden_ir
from lazy_compiler_b200.compiler import compile_file
from lazy_compiler_b200.runner import run_package, run_request, seeded_input


def test_chain_package_compiles_each_kernel(tmp_path):
    folder = W.chain_package(tmp_path / "chain")
    plans = [compile_file(folder / f"{e}.ir.json", folder / "meta.json") for e in ("k_first", "k_second")]
    assert [p["entry"] for p in plans] == ["k_first", "k_second"]
    assert plans[1]["arg_order"] == ["t", "y", "out"]


def request_for(name, **extra):
    meta = json.loads((golden(name) / "meta.json").read_text())
    k = meta["kernels"][0]
    req = {"plan": compile_file(golden_ir(name)), "entry": k["entry"], "grid": k["grid"], "block": k["block"],
           "smem_bytes": k["smem_bytes"], "zero_outputs": k["zero_outputs"], "args": k["args"]}
    req.update(extra)
    return req


def test_request_validation_needs_no_gpu():
    assert run_request({"entry": "k"})["stage"] == "request"
    r = run_request(request_for("p01_vector_add", entry="k_other"))
    assert not r["ok"] and r["stage"] == "run" and "k_other" in r["stderr"]
    assert run_request(request_for("p01_vector_add", iters=0))["stage"] == "request"
    req = request_for("p01_vector_add")
    req["args"] = list(reversed(req["args"]))
    assert run_request(req)["stage"] == "request"
    req = request_for("p01_vector_add", grid=[7, 1, 1])
    assert run_request(req)["stage"] == "request"


@pytest.mark.gpu
def test_chained_kernels_run_in_meta_order(tmp_path, cuda_device):
    folder = W.chain_package(tmp_path / "chain")
    meta = json.loads((folder / "meta.json").read_text())
    x = seeded_input(meta["kernels"][0]["args"][0])
    y = seeded_input(meta["kernels"][1]["args"][1])
    out = run_package(folder)["out"]
    np.testing.assert_array_equal(out, x * np.float32(2) + y)


@pytest.mark.gpu
def test_run_request_matches_runner_semantics(cuda_device):
    r = run_request(request_for("p01_vector_add", warmup=2, iters=5, max_return=100))
    assert r["ok"] and r["iters"] == 5 and r["median_us"] > 0
    o = r["outputs"]["add"]
    meta = json.loads((golden("p01_vector_add") / "meta.json").read_text())
    x0, x1 = (seeded_input(a) for a in meta["kernels"][0]["args"][:2])
    assert o["shape"] == [1024] and o["truncated"] and len(o["values"]) == 100
    np.testing.assert_array_equal(np.asarray(o["values"], np.float32), (x0 + x1)[:100])
    assert abs(o["sum"] - float((x0 + x1).astype(np.float64).sum())) < 1e-3


@pytest.mark.gpu
def test_run_request_zero_outputs_between_launches(cuda_device):
    """m02 accumulates with atomics: zero_outputs keeps repeated launches equal to one."""
    once = run_request(request_for("m02_matmul_rect", iters=1, max_return=1 << 16))
    many = run_request(request_for("m02_matmul_rect", warmup=3, iters=4, max_return=1 << 16))
    assert once["ok"] and many["ok"]
    np.testing.assert_allclose(many["outputs"]["matmul"]["values"], once["outputs"]["matmul"]["values"],
                               rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
def test_submit_style_chaining_through_requests(tmp_path, cuda_device):
    """Kernel 2's intermediate arrives as ``data`` from kernel 1's output, as submit.py chains them."""
    folder = W.chain_package(tmp_path / "chain", n=512)
    meta = json.loads((folder / "meta.json").read_text())
    produced = {}
    for k in meta["kernels"]:
        args = []
        for a in k["args"]:
            a = dict(a)
            if a.pop("intermediate", False):
                a["data"] = produced[a["name"]]
            args.append(a)
        plan = compile_file(folder / f"{k['entry']}.ir.json", folder / "meta.json")
        r = run_request({"plan": plan, "entry": k["entry"], "grid": k["grid"], "block": k["block"],
                         "zero_outputs": k["zero_outputs"], "args": args, "max_return": 4096})
        assert r["ok"], r
        produced.update({n: v["values"] for n, v in r["outputs"].items()})
    x = seeded_input(meta["kernels"][0]["args"][0])
    y = seeded_input(meta["kernels"][1]["args"][1])
    np.testing.assert_array_equal(np.asarray(produced["out"], np.float32), x * np.float32(2) + y)
