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


def test_prefill_host_helpers_need_no_gpu():
    """Block splitting of expert-grouped pairs and the prefill entry's
    host-side checks (streamlx/integrate.py:141-232 groups the sweep's pairs
    by expert; the library takes them as blocks of at most PREFILL_BLOCK)."""
    import numpy as np

    from streamlx_b200 import ops
    nb = ops.PREFILL_BLOCK
    blocks = ops.prefill_blocks([5, 2, 9], [3, 2 * nb + 1, 0])
    assert blocks.tolist() == [[5, 0, 3, 0], [2, 3, nb, 0],
                               [2, 3 + nb, nb, 0], [2, 3 + 2 * nb, 1, 0]]
    assert ops.prefill_blocks([], []).shape == (0, 4)
    assert ops.prefill_supported(2560, 1024, 2)
    assert not ops.prefill_supported(2560, 1024, 4)
    assert not ops.prefill_supported(2048, 768, 2)
    # scratch: both phases' operand images, 16 KB per chunk of a block
    n = L.prefill_scratch_bytes(10, 2560, 1024, 2)
    assert n == 10 * ((40 + 2) + (16 + 1)) * 128 * 128
    assert L.prefill_scratch_bytes(10, 2560, 1024, 4) == 0
    lib = L.lib()
    bank = L.slx_expert_bank(None, 0, 1, 2560, 1024, 4)
    rc = lib.slx_prefill_grouped(ctypes.byref(bank), None, 0, None, 0, None,
                                 1, None, None, 0, None, 0, None, None)
    assert rc == -2 and b"2-bit" in lib.slx_last_error_string()
    assert np.dtype(np.int32) == blocks.dtype
