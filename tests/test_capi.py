"""The C-ABI library: loads, exports every entry point include/lazyb200.h declares,
and validates arguments on the host (no device work, so these run without a GPU)."""
import ctypes
import re

import pytest

from conftest import ROOT
from lazy_compiler_b200 import runtime


def declared():
    text = (ROOT / "include" / "lazyb200.h").read_text()
    return sorted(set(re.findall(r"^int (lc_\w+)\(", text, flags=re.M)))


def test_header_and_bindings_agree():
    assert declared() == sorted(runtime.SIGNATURES)


@pytest.mark.parametrize("name", declared())
def test_library_exports_symbol(name):
    lib = runtime.library()
    assert getattr(lib, name) is not None


def test_version_and_error_buffer():
    assert runtime.library().lc_version() >= 10000


NULL = ctypes.c_void_p(0)


@pytest.mark.parametrize("call", [
    lambda: runtime.call("lc_add_f32", NULL, NULL, NULL, 16, NULL),
    lambda: runtime.call("lc_axpb_f32", NULL, NULL, NULL, NULL, 16, NULL),
    lambda: runtime.call("lc_relumul_f32", NULL, NULL, NULL, 16, NULL),
    lambda: runtime.call("lc_gelu", 0, 0, NULL, NULL, 16, NULL),
    lambda: runtime.call("lc_gelu", 7, 0, ctypes.c_void_p(16), ctypes.c_void_p(16), 16, NULL),
    lambda: runtime.call("lc_gelu", 0, 3, ctypes.c_void_p(16), ctypes.c_void_p(16), 16, NULL),
    lambda: runtime.call("lc_sum_f32", NULL, NULL, 16, NULL),
    lambda: runtime.call("lc_mean_f32", ctypes.c_void_p(16), NULL, ctypes.c_void_p(16), 16, NULL),
    lambda: runtime.call("lc_rowsum_f32", NULL, NULL, 4, 4, NULL),
    lambda: runtime.call("lc_rmsnorm_f32", NULL, NULL, ctypes.c_void_p(16), NULL, ctypes.c_void_p(16), 4, 4, NULL),
    lambda: runtime.call("lc_softmax_f32", ctypes.c_void_p(16), ctypes.c_void_p(16), -1, 4, NULL),
    lambda: runtime.call("lc_l2norm_f32", NULL, NULL, 4, 4, NULL),
    lambda: runtime.call("lc_add_f32", ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), -5, NULL),
])
def test_invalid_arguments_are_rejected_on_host(call):
    with pytest.raises(runtime.LcError) as err:
        call()
    assert err.value.status == -1
    assert err.value.message
