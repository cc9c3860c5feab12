"""CPU-side checks of the C ABI library: it loads without a GPU and exports
every entry point include/streamlx_cuda.h declares."""

import ctypes
import os
import re

from streamlx_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    hdr = open(os.path.join(ROOT, "include", "streamlx_cuda.h")).read()
    return sorted(set(re.findall(r"\b(slx_[a-z0-9_]+)\s*\(", hdr)))


def test_header_matches_binding_table():
    assert sorted(L.EXPORTS) == declared_symbols()


def test_library_exports_all_symbols():
    lib = L.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.slx_version() == 1
    assert lib.slx_last_error_string() == b""


def test_scratch_size_helpers_need_no_gpu():
    n = L.switchglu_scratch_bytes(1, 10, 1024, 0)
    assert n >= 10 * 1024 * 2 and n % 256 == 0
    assert L.router_scratch_bytes(4, 256) >= 4 * 256 * 4 + 16


def test_host_side_errors_without_gpu():
    # argument checks run before any CUDA call
    lib = L.lib()
    bank = L.slx_expert_bank()
    rc = lib.slx_switchglu(ctypes.byref(bank), None, None, 1, 4, None, None,
                           None, 0, None, None, 0, None, None)
    assert rc == -2 or rc == -1
    assert lib.slx_last_error_string() != b""
