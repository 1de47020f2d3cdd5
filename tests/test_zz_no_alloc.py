"""lc_sum_f32_noalloc: the whole-array sum for callers that cannot let a library allocate.

Some callers cannot have the library call cudaMalloc — their device memory is
owned entirely by their own allocator, or their launch path must not pay
cudaMalloc's implicit device-wide synchronisation.  For them the library
exports lc_sum_f32_noalloc, which keeps its partials in a fixed device array
instead of the workspace lc_sum_f32 allocates.  This test calls it through the
C ABI twice in a row (the second call reuses the array the first one left
behind) and checks each result against lc_sum_f32 within the reductions'
relative tolerance of 1e-5.  The file is named so pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

from lazy_compiler_b200 import runtime
from oracle import expressions as O

pytestmark = pytest.mark.gpu

RTOL = 1e-5
MAX_N = 1 << 32


def P(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("n", [1, 1000, 65536, 1000003, 1 << 24])
def test_noalloc_sum_matches_lc_sum_f32_on_two_calls(n, cuda_device):
    import torch
    x = torch.from_numpy(O.uniform(n, seed=n)).cuda()
    expected = torch.empty(1, device="cuda")
    runtime.call("lc_sum_f32", P(x), P(expected), n, None)
    want = float(expected.item())
    for _ in range(2):
        got = torch.full((1,), float("nan"), device="cuda")
        runtime.call("lc_sum_f32_noalloc", P(x), P(got), n, None)
        value = float(got.item())
        assert np.isclose(value, want, rtol=RTOL, atol=1e-30), (value, want)


def test_noalloc_sum_unaligned_input(cuda_device):
    import torch
    x = torch.from_numpy(O.uniform(100001, seed=9)).cuda()
    out = torch.empty(2, device="cuda")
    runtime.call("lc_sum_f32", P(x[1:]), P(out[0:]), 100000, None)
    runtime.call("lc_sum_f32_noalloc", P(x[1:]), P(out[1:]), 100000, None)
    a, b = out.cpu().numpy()
    assert np.isclose(b, a, rtol=RTOL, atol=1e-30)


def test_noalloc_sum_rejects_sizes_beyond_its_maximum(cuda_device):
    import torch
    x = torch.zeros(16, device="cuda")
    out = torch.zeros(1, device="cuda")
    with pytest.raises(runtime.LcError) as err:
        runtime.call("lc_sum_f32_noalloc", P(x), P(out), MAX_N + 1, None)
    assert err.value.status == -5
    assert "exceeds the maximum" in err.value.message


def test_noalloc_sum_leaves_device_memory_unchanged(cuda_device):
    import torch
    n = 1 << 22
    x = torch.from_numpy(O.uniform(n, seed=2)).cuda()
    out = torch.empty(1, device="cuda")
    runtime.call("lc_sum_f32_noalloc", P(x), P(out), n, None)
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        runtime.call("lc_sum_f32_noalloc", P(x), P(out), n, None)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
