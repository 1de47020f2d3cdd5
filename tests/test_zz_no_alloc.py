"""lc_sum_f32_noalloc: the whole-array sum for callers that cannot let a library allocate.

Some callers cannot have the library call cudaMalloc: their device memory is
owned entirely by their own allocator, or their launch path must not pay
cudaMalloc's implicit device-wide synchronisation.  For them the library
exports lc_sum_f32_noalloc, which keeps its partials in a fixed device array
instead of the workspace lc_sum_f32 allocates.  These tests call it through
the C ABI twice in a row (the second call reuses the array the first one left
behind) and check each result against the float64 oracle and against
lc_sum_f32, within the reductions' relative tolerance of 1e-5.  A separate
fresh process checks that not even the first call changes the device's free
memory.  The file is named so pytest collects it last.
"""
import ctypes
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest

from lazy_compiler_b200 import runtime
from oracle import expressions as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5
MAX_N = 1 << 32
ROOT = Path(__file__).resolve().parents[1]


def P(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("n", [1, 1000, 65536, 1000003, 1 << 24, (1 << 26) + 5])
def test_noalloc_sum_matches_oracle_and_lc_sum_f32_on_two_calls(n, cuda_device):
    import torch
    host = O.uniform(n, seed=n)
    exact = float(O.sum_(host)[0])
    x = torch.from_numpy(host).cuda()
    expected = torch.empty(1, device="cuda")
    runtime.call("lc_sum_f32", P(x), P(expected), n, None)
    want = float(expected.item())
    for _ in range(2):
        got = torch.full((1,), float("nan"), device="cuda")
        runtime.call("lc_sum_f32_noalloc", P(x), P(got), n, None)
        value = float(got.item())
        assert np.isclose(value, exact, rtol=RTOL, atol=1e-30), (value, exact)
        assert np.isclose(value, want, rtol=RTOL, atol=1e-30), (value, want)


def test_noalloc_sum_unaligned_input(cuda_device):
    import torch
    host = O.uniform(100001, seed=9)
    x = torch.from_numpy(host).cuda()
    out = torch.empty(2, device="cuda")
    runtime.call("lc_sum_f32", P(x[1:]), P(out[0:]), 100000, None)
    runtime.call("lc_sum_f32_noalloc", P(x[1:]), P(out[1:]), 100000, None)
    a, b = out.cpu().numpy()
    assert np.isclose(b, float(O.sum_(host[1:])[0]), rtol=RTOL, atol=1e-30)
    assert np.isclose(b, a, rtol=RTOL, atol=1e-30)


def test_noalloc_sum_rejects_sizes_beyond_its_maximum(cuda_device):
    import torch
    x = torch.zeros(16, device="cuda")
    out = torch.zeros(1, device="cuda")
    with pytest.raises(runtime.LcError) as err:
        runtime.call("lc_sum_f32_noalloc", P(x), P(out), MAX_N + 1, None)
    assert err.value.status == -5
    assert "exceeds the maximum" in err.value.message


_FRESH = textwrap.dedent("""
    import ctypes, sys
    sys.path.insert(0, sys.argv[1])
    import numpy as np
    import torch
    from lazy_compiler_b200 import runtime
    from oracle import expressions as O
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    n = (1 << 22) + 3
    host = O.uniform(n, seed=2)
    x = torch.from_numpy(host).cuda()
    out = torch.full((2,), float("nan"), device="cuda")
    total = torch.zeros(1, dtype=torch.float64, device="cuda")
    warm, stream = torch.cuda.Stream(), torch.cuda.Stream()
    # load the library's reduction module without the entry point under test:
    # lc_sum_finalize lives in the same module and allocates nothing
    runtime.call("lc_sum_finalize", P(total), ctypes.c_void_p(0), P(out), ctypes.c_void_p(warm.cuda_stream))
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for i in range(2):
        runtime.call("lc_sum_f32_noalloc", P(x), P(out[i:]), n, ctypes.c_void_p(stream.cuda_stream))
    torch.cuda.synchronize()
    free_after = torch.cuda.mem_get_info()[0]
    got = out.cpu().numpy()
    exact = float(O.sum_(host)[0])
    assert free_after == free_before, ("device memory changed", free_before, free_after)
    assert np.allclose(got, exact, rtol=1e-5, atol=1e-30), (got, exact)
    print("fresh-process no-alloc check: ok")
""")


def test_noalloc_sum_first_call_leaves_device_memory_unchanged(cuda_device):
    """A fresh process, a new non-default stream, free memory read before the first-ever call."""
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    result = subprocess.run([sys.executable, "-c", _FRESH, str(ROOT)], capture_output=True, text=True,
                            timeout=300, env=env)
    assert result.returncode == 0, result.stdout[-2000:] + result.stderr[-4000:]
    assert "ok" in result.stdout
