"""ORACLE — test infrastructure only; never imported by the product path.

numpy restatement of the synthetic decoder trunk that surrounds the expert
path (the reference leaves the trunk to mlx-lm; this mirrors a Qwen3-MoE
style block): RMSNorm with fused residual add, per-head q/k RMSNorm,
rotate-half RoPE, GQA attention over a KV cache, greedy argmax.  Rounding
model: every op's output is rounded to bf16; reductions accumulate in fp32.
"""

from __future__ import annotations

import numpy as np

from .affine import bf16_round


def add_rmsnorm(h: np.ndarray, delta: np.ndarray | None, w: np.ndarray,
                eps: float):
    """Returns (h', y): h' = bf16(h + delta); y = bf16(h' * rsqrt(mean h'^2 +
    eps) * w).  h, delta, w are bf16 values in float32 arrays."""
    h = h.astype(np.float32)
    if delta is not None:
        h = bf16_round(h + delta.astype(np.float32))
    ms = np.mean(h.astype(np.float32) ** 2, axis=-1, keepdims=True,
                 dtype=np.float32)
    inv = (1.0 / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return h, bf16_round(h * inv * w.astype(np.float32))


def rope_inv_freq(hd: int, theta: float) -> np.ndarray:
    i = np.arange(hd // 2, dtype=np.float64)
    return (theta ** (-2.0 * i / hd)).astype(np.float32)


def qk_norm_rope(v: np.ndarray, nw: np.ndarray, eps: float, pos: int,
                 inv_freq: np.ndarray) -> np.ndarray:
    """One head vector [hd]: RMSNorm(hd) * nw then rotate-half RoPE at pos."""
    hd = v.shape[-1]
    half = hd // 2
    v = v.astype(np.float32)
    ms = np.mean(v * v, dtype=np.float32)
    inv = np.float32(1.0) / np.sqrt(ms + np.float32(eps))
    n = bf16_round(v * inv * nw.astype(np.float32))
    a, b = n[:half], n[half:]
    ang = (np.float32(pos) * inv_freq).astype(np.float32)
    cs = np.cos(ang.astype(np.float64)).astype(np.float32)
    sn = np.sin(ang.astype(np.float64)).astype(np.float32)
    return bf16_round(np.concatenate([a * cs - b * sn, a * sn + b * cs]))


def attn_decode(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, n: int,
                n_q: int, n_kv: int) -> np.ndarray:
    """q [n_q, hd]; kc/vc [L, n_kv, hd]; attends positions 0..n-1."""
    hd = q.shape[-1]
    rep = n_q // n_kv
    out = np.zeros((n_q, hd), dtype=np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    for h in range(n_q):
        kh = h // rep
        s = (kc[:n, kh].astype(np.float32) @ q[h].astype(np.float32)) * scale
        s = s - s.max()
        p = np.exp(s.astype(np.float64)).astype(np.float32)
        out[h] = (p @ vc[:n, kh].astype(np.float32)) / p.sum()
    return bf16_round(out)


def argmax_first(v: np.ndarray) -> int:
    """Greedy pick, ties -> lowest index."""
    v = np.asarray(v, dtype=np.float32)
    return int(np.flatnonzero(v == v.max())[0])
