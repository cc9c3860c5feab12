"""ORACLE — test infrastructure only; never imported by the product path.

numpy restatement of the tile format the CUDA pack kernels write
(streamlx_b200/csrc/slx_tiles.cuh), for a byte-exact check of the packers.
"""

from __future__ import annotations

import numpy as np


def _swz_rows(rows: np.ndarray, RB: int) -> np.ndarray:
    """rows [16, RB] uint8 -> swizzled row block (16-byte units XOR row&7)."""
    out = rows.copy()
    if RB % 128:
        return out
    units = RB // 16
    for r in range(rows.shape[0]):
        u = np.arange(units)
        dst = (u ^ (r & 7))
        out[r].reshape(units, 16)[dst] = rows[r].reshape(units, 16)[u]
    return out


def _sb(s16: np.ndarray, b16: np.ndarray) -> np.ndarray:
    return s16.astype(np.uint32) | (b16.astype(np.uint32) << 16)


def pair_tile(P: tuple, p0: int, Q: tuple, q0: int, nrows: int,
              in_f: int, bits: int) -> bytes:
    RB, nG = in_f * bits // 8, in_f // 64
    blocks = []
    sbs = []
    for (w, s, b), r0 in ((P, p0), (Q, q0)):
        wb = np.zeros((16, RB), np.uint8)
        sw = np.zeros((16, nG), np.uint32)
        n = max(0, min(16, nrows - r0))
        if n:
            wb[:n] = w[r0:r0 + n].view(np.uint8).reshape(n, RB)
            sw[:n] = _sb(s[r0:r0 + n], b[r0:r0 + n])
        blocks.append(_swz_rows(wb, RB))
        sbs.append(sw)
    sb = np.stack(sbs, 0).transpose(2, 0, 1).reshape(-1)   # [G][m][row]
    return b"".join(bl.tobytes() for bl in blocks) + sb.astype(np.uint32).tobytes()


def single_tile(D: tuple, r0: int, in_f: int, bits: int) -> bytes:
    w, s, b = D
    RB, nG = in_f * bits // 8, in_f // 64
    wb = w[r0:r0 + 16].view(np.uint8).reshape(16, RB)
    sb = _sb(s[r0:r0 + 16], b[r0:r0 + 16]).T.reshape(-1)   # [G][row]
    return _swz_rows(wb, RB).tobytes() + sb.astype(np.uint32).tobytes()


def expert_tiled(gate: tuple, up: tuple, down: tuple, H: int, I: int,
                 bits: int) -> bytes:
    parts = [pair_tile(gate, 16 * t, up, 16 * t, I, H, bits)
             for t in range(I // 16)]
    parts += [single_tile(down, 16 * t, I, bits) for t in range(H // 16)]
    return b"".join(parts)


def dense_tiled(W: tuple, out_f: int, in_f: int, bits: int) -> bytes:
    return b"".join(pair_tile(W, 32 * t, W, 32 * t + 16, out_f, in_f, bits)
                    for t in range((out_f + 31) // 32))
