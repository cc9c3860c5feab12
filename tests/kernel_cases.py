"""Shared builders for kernel parity tests: seeded quantized expert banks on
both sides (torch tensors for the CUDA path, numpy for the oracle)."""

from __future__ import annotations

import numpy as np
import torch

from oracle import affine as A
from streamlx_b200 import synth

TOL_MAX_ABS = 2e-2   # parity tolerance on bf16 layer outputs
TOL_REL_L2 = 1e-3


def quant_stack(E: int, out: int, inp: int, bits: int, seed: int,
                std: float = 0.02):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(E, out, inp, generator=g) * std
    pk, s, b = synth.quantize_affine(w, bits, 64)
    return pk, s, b


def to_np(pk, s, b):
    return (pk.numpy().view(np.uint32), s.view(torch.int16).numpy()
            .view(np.uint16), b.view(torch.int16).numpy().view(np.uint16))


def make_bank(E, H, I, bits, seed, device="cuda"):
    """Returns (torch dict proj->(w,s,b) on device, numpy triples, qparams)."""
    tt, npt, qp = {}, {}, {}
    for j, (proj, o, i) in enumerate((("gate_proj", I, H), ("up_proj", I, H),
                                      ("down_proj", H, I))):
        pk, s, b = quant_stack(E, o, i, bits, seed * 10 + j)
        tt[proj] = (pk.to(device), s.to(device), b.to(device))
        w, sn, bn = to_np(pk, s, b)
        npt[proj] = {"weight": w, "scales": sn, "biases": bn}
        qp[proj] = (i, o, bits, 64)
    return tt, npt, qp


def bf16_tensor(a: np.ndarray, device="cuda") -> torch.Tensor:
    u = A.bf16_to_bits(a)
    return torch.from_numpy(u.view(np.int16).copy()).view(torch.bfloat16) \
        .to(device)


def bf16_np(t: torch.Tensor) -> np.ndarray:
    return A.bf16_from_bits(t.detach().cpu().view(torch.int16).numpy()
                            .view(np.uint16))


def check_close(got: np.ndarray, want: np.ndarray, max_abs=TOL_MAX_ABS,
                rel=TOL_REL_L2):
    d = float(np.max(np.abs(got.astype(np.float64) - want)))
    r = A.rel_l2(got, want)
    assert np.isfinite(got).all(), "non-finite output"
    assert d <= max_abs and r <= rel, f"max_abs {d:.3e} rel_l2 {r:.3e}"
    return d, r


def pack_pool(tt: dict, expert_of_slot, H: int, I: int, bits: int,
              device="cuda"):
    """Tile-format slot pool on `device`: slot s holds expert
    expert_of_slot[s] of the MLX-layout CPU bank `tt` (make_bank output)."""
    from streamlx_b200 import _lib as L
    stride = L.slot_stride(H, I, bits)
    n = len(expert_of_slot)
    pool = torch.zeros(n * stride, dtype=torch.uint8, device=device)
    ex = []
    keep = []
    for e in expert_of_slot:
        trip = []
        for proj in ("gate_proj", "up_proj", "down_proj"):
            w, s, b = tt[proj]
            t3 = (w[e].contiguous().to(device), s[e].contiguous().to(device),
                  b[e].contiguous().to(device))
            keep.append(t3)
            trip.append(t3)
        ex.append(tuple(trip))
    L.pack_experts(ex, H, I, bits, [pool.data_ptr() + i * stride
                                    for i in range(n)])
    torch.cuda.synchronize()
    return pool, stride
