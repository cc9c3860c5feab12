"""slx_router_topk_noalloc (router with the library's static scratch) against
slx_router_topk (caller scratch), called through the C ABI.  Collected last
so it also runs after every other kernel test in the same process."""

from __future__ import annotations

import ctypes as C

import numpy as np
import pytest
import torch

from oracle import affine as A
from streamlx_b200 import _lib as L
from streamlx_b200 import synth

from .kernel_cases import bf16_tensor

pytestmark = pytest.mark.gpu

SLX_ERR_SCRATCH = -7


def _inputs(seed: int, T: int, H: int, E: int, dev):
    rng = np.random.default_rng(seed)
    x = A.bf16_round(rng.standard_normal((T, H)).astype(np.float32))
    wg = A.bf16_round((rng.standard_normal((E, H)) / np.sqrt(H))
                      .astype(np.float32))
    bias = synth.zipf_bias(E, 1.0, seed)
    return (bf16_tensor(x, dev), bf16_tensor(wg, dev),
            torch.from_numpy(bias).to(dev))


def _noalloc(x, wg, bias, k, ids, scores, status, T=None, E=None):
    T = x.shape[0] if T is None else T
    E = wg.shape[0] if E is None else E
    return L.lib().slx_router_topk_noalloc(
        x.data_ptr(), None, wg.data_ptr(), bias.data_ptr(), T, x.shape[1], E,
        k, 1, None, None, ids.data_ptr(), scores.data_ptr(),
        status.data_ptr(), C.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("T,E,k", [(1, 256, 8), (32, 256, 10), (128, 256, 8)])
def test_noalloc_router_matches_scratch_router(T, E, k):
    dev = torch.device("cuda", 0)
    H = 2048
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    for call in range(2):          # twice in a row: tickets left at zero
        x, wg, bias = _inputs(10 * T + call, T, H, E, dev)
        want_ids = torch.empty(T, k, dtype=torch.int32, device=dev)
        want_sc = torch.empty(T, k, dtype=torch.float32, device=dev)
        scratch = torch.zeros(L.router_scratch_bytes(T, E), dtype=torch.uint8,
                              device=dev)
        L.router_topk(x, wg, bias, k, True, want_ids, want_sc, scratch, status)
        got_ids = torch.full((T, k), -1, dtype=torch.int32, device=dev)
        got_sc = torch.zeros(T, k, dtype=torch.float32, device=dev)
        rc = _noalloc(x, wg, bias, k, got_ids, got_sc, status)
        assert rc == 0, L.lib().slx_last_error_string()
        torch.cuda.synchronize()
        assert status.item() == 0
        assert torch.equal(got_ids, want_ids), call
        assert torch.equal(got_sc, want_sc), call


def test_noalloc_router_rejects_oversize():
    dev = torch.device("cuda", 0)
    x, wg, bias = _inputs(1, 1, 64, 16, dev)
    ids = torch.empty(1, 4, dtype=torch.int32, device=dev)
    sc = torch.empty(1, 4, dtype=torch.float32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    # argument checks only: no kernel is launched for either call
    assert _noalloc(x, wg, bias, 4, ids, sc, status, T=129, E=256) == \
        SLX_ERR_SCRATCH
    assert b"static scratch" in L.lib().slx_last_error_string()
    assert _noalloc(x, wg, bias, 4, ids, sc, status, T=1025, E=1) == \
        SLX_ERR_SCRATCH
