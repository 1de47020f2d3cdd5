"""GPU parity of lane programs (one-warp fragment programs run per lane by
lc_pointwise): the tensor-core fixtures forced through the lane compiler
(exercising gathers, mma.sync, repack and every store variant on the
device) against the reference's golden vectors, and changed fragment
programs against the fragment oracle."""
import json

import numpy as np
import pytest

from conftest import golden, golden_ir, golden_meta
from lazy_compiler_b200.fragment_vm import compile_fragment_lanes
from lazy_compiler_b200.ir import load_package
from lazy_compiler_b200.runtime import launch
from oracle import expressions as O
from oracle import fragment_ir

pytestmark = pytest.mark.gpu

TORCH = {"f32": "float32", "f16": "float16", "bf16": "bfloat16", "i32": "int32"}


def run_plan(plan, meta, arrays):
    import torch
    k = meta["kernels"][0]
    bufs = {}
    for a in k["args"]:
        dt = getattr(torch, TORCH[a["dtype"]])
        shape = tuple(a.get("shape") or [1])
        if a.get("output"):
            t = torch.full(shape, float("nan"), device="cuda").to(dt)
        else:
            t = torch.as_tensor(np.ascontiguousarray(arrays[a["name"]])).to("cuda", dt)
        bufs[a["name"]] = t
    for n in k.get("zero_outputs", []):
        bufs[n].zero_()
    launch(plan, {n: t.data_ptr() for n, t in bufs.items()}, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return {n: bufs[n].float().cpu().numpy() for n in meta["graph_outputs"]}


LANE_FIXTURES = sorted(p.name for p in golden("").iterdir() if p.name.startswith("tensor_")
                       and p.name != "tensor_cp_async_shared" and not p.name.startswith("tensor_shared"))


@pytest.mark.parametrize("name", LANE_FIXTURES)
@pytest.mark.parametrize("offset", [0, 3])
def test_tensor_fixture_as_lane_program(name, offset, cuda_device):
    pkg = load_package(golden_ir(name))
    plan = compile_fragment_lanes(pkg, pkg.body[0]).to_json()
    meta = golden_meta(name)
    arrays = {a["name"]: O.input_array(a, offset) for a in meta["kernels"][0]["args"] if not a.get("output")}
    got = run_plan(plan, meta, arrays)
    ref = fragment_ir.evaluate(golden_ir(name), arrays)
    for key, value in ref.items():
        row = O.compare(got[key].reshape(value.shape), value, meta["rtol"], meta["atol"])
        assert row["pass"], (key, row)
    if offset == 0:
        with np.load(golden(name) / "expected.npz") as z:
            for key in z.files:
                assert O.compare(got[key].reshape(z[key].shape), z[key], meta["rtol"], meta["atol"])["pass"]
