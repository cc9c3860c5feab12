"""ORACLE — test infrastructure only; never imported by the product path.

CPU restatement (numpy) of the arithmetic on the reference's expert path.
The reference delegates it to MLX (absent here), so this file restates MLX's
documented semantics at the reference's call sites:

* ``mx.gather_qmm(x, W, S, B, rhs_indices, transpose=True, group_size, bits,
  mode="affine")`` -- streamlx/pool.py:40-45.  Affine format: uint32 words
  packed low bits first, ``32/bits`` values per word; per group of
  ``group_size`` input columns ``w = scale * q + bias`` with bf16 scale/bias.
* ``swiglu(gate, up) = silu(gate) * up`` -- streamlx/pool.py:24,49
  (mlx_lm.models.activations).
* ``switch_forward`` composition (up, gate, swiglu, down, squeeze) --
  streamlx/pool.py:30-50; per-expert outputs are returned *unweighted*.
* the MoE block around it (router linear -> softmax -> top-k -> optional
  renormalisation -> score-weighted sum), which the reference leaves to
  mlx-lm (streamlx/integrate.py:5-7, 81-85).

Rounding model (what the CUDA kernels must match to tolerance): every
``gather_qmm`` output is rounded to bf16 (MLX returns the input dtype), the
SwiGLU product is rounded to bf16 before the down projection, and the
score-weighted combine rounds once.  The oracle accumulates in fp64, i.e. it
is the correctly rounded version of that bf16 pipeline; MLX and the CUDA
kernels accumulate in fp32.

Dequantised weights are exactly defined in fp32: ``scale*q`` is exact (<= 16
significant bits) so ``scale*q + bias`` has one rounding whether or not it is
fused; ``dequant`` is therefore a bit-exact reference.

Routing is made bit-exact by construction: logits are the fp64 sum of exact
bf16*bf16 products rounded once to fp32 (order-independent whenever that sum
is exact, which holds for the workloads' value ranges), plus an fp32 bias;
top-k is taken on the logits (softmax is monotonic), descending, ties to the
lower expert id.  Scores are softmax probabilities of the selected logits and
are compared to tolerance.

Parity status: unpinned for this arithmetic (the reference's MLX path cannot
run here and ships no golden vectors); the pool / trace side is pinned against
the reference's own code (tests/golden).
"""

from __future__ import annotations

import ml_dtypes
import numpy as np

BF16 = ml_dtypes.bfloat16


def bf16_round(a) -> np.ndarray:
    """Round-to-nearest-even to bf16 (from fp32 or fp64 in ONE step),
    returned as float32 values."""
    a = np.asarray(a)
    if a.dtype == np.float64:
        return a.astype(BF16).astype(np.float32)
    return np.asarray(a, dtype=np.float32).astype(BF16).astype(np.float32)


def bf16_from_bits(u16) -> np.ndarray:
    u = np.asarray(u16).astype(np.uint32) << 16
    return u.view(np.float32)


def bf16_to_bits(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(BF16).view(np.uint16)


def unpack(packed, bits: int) -> np.ndarray:
    """uint32 words [..., W] -> integer codes [..., W*32/bits] (low bits first)."""
    w = np.asarray(packed).view(np.uint32)
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = (w[..., None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(*w.shape[:-1], w.shape[-1] * per).astype(np.uint32)


def dequant(packed, scales_u16, biases_u16, bits: int, gs: int) -> np.ndarray:
    """Affine dequantisation -> fp32 [..., in]; bit-exact (see module doc)."""
    q = unpack(packed, bits).astype(np.float32)
    s = bf16_from_bits(scales_u16)
    b = bf16_from_bits(biases_u16)
    *lead, n = q.shape
    qg = q.reshape(*lead, n // gs, gs)
    w = qg * s[..., None] + b[..., None]      # s*q exact; one rounding in +b
    return w.reshape(*lead, n).astype(np.float32)


def qmv(x: np.ndarray, w_deq: np.ndarray) -> np.ndarray:
    """x [T, in] (bf16 values) @ w_deq[out, in]^T, accumulated in fp64 and
    rounded once to bf16."""
    return bf16_round(x.astype(np.float64) @ w_deq.T.astype(np.float64))


def silu(g: np.ndarray) -> np.ndarray:
    g = g.astype(np.float64)
    return g / (1.0 + np.exp(-g))


def swiglu(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    """bf16(silu(gate) * up) with bf16 inputs."""
    return bf16_round(silu(gate) * up.astype(np.float64))


def expert_forward(x: np.ndarray, deq: dict) -> np.ndarray:
    """One expert on rows x [T, H]: down(swiglu(gate(x), up(x))) -> [T, H]."""
    up = qmv(x, deq["up_proj"])
    gate = qmv(x, deq["gate_proj"])
    return qmv(swiglu(gate, up), deq["down_proj"])


def dequant_expert(triples: dict, e: int, qparams: dict) -> dict:
    """Dequantised {proj: fp32 [out, in]} of stacked row ``e``."""
    out = {}
    for proj, t in triples.items():
        _, _, bits, gs = qparams[proj]
        out[proj] = dequant(t["weight"][e], t["scales"][e], t["biases"][e],
                            bits, gs)
    return out


def switch_forward(x: np.ndarray, inds: np.ndarray, triples: dict,
                   qparams: dict) -> np.ndarray:
    """streamlx/pool.py:30-50 on numpy: x [B,T,H] bf16 values, inds [B,T,k]
    -> per-expert unweighted outputs [B,T,k,H] (bf16 values)."""
    B, T, H = x.shape
    k = inds.shape[-1]
    out = np.zeros((B, T, k, triples["down_proj"]["weight"].shape[1]),
                   dtype=np.float32)
    cache: dict = {}
    for b in range(B):
        for t in range(T):
            for j in range(k):
                e = int(inds[b, t, j])
                if e not in cache:
                    cache[e] = dequant_expert(triples, e, qparams)
                out[b, t, j] = expert_forward(x[b, t][None], cache[e])[0]
    return out


def router_logits(x: np.ndarray, w_gate_u16: np.ndarray,
                  bias: np.ndarray | None) -> np.ndarray:
    """fp32(fp64 sum of exact products) + fp32 bias -> [T, E] fp32."""
    xw = bf16_from_bits(bf16_to_bits(x)).astype(np.float64)
    w = bf16_from_bits(w_gate_u16).astype(np.float64)
    lg = (xw @ w.T).astype(np.float32)
    if bias is not None:
        lg = (lg + np.asarray(bias, dtype=np.float32)).astype(np.float32)
    return lg


def topk_ids(logits: np.ndarray, k: int) -> np.ndarray:
    """Top-k per row, descending logit, ties -> lower expert id."""
    order = np.argsort(-logits, axis=-1, kind="stable")
    return order[..., :k].astype(np.int32)


def topk_margin(logits: np.ndarray, k: int) -> float:
    """Smallest gap between logits that decides an ordered top-k: adjacent
    pairs among the k + 1 largest (the order of the picks and the cut)."""
    s = np.sort(np.asarray(logits, dtype=np.float64))[::-1][:k + 1]
    return float(np.min(s[:-1] - s[1:])) if s.size > 1 else np.inf


def softmax_rows(logits: np.ndarray) -> np.ndarray:
    z = logits.astype(np.float64)
    z = z - z.max(axis=-1, keepdims=True)
    p = np.exp(z)
    return (p / p.sum(axis=-1, keepdims=True)).astype(np.float32)


def router(x: np.ndarray, w_gate_u16: np.ndarray, bias, k: int,
           norm_topk: bool, forced_ids: np.ndarray | None = None):
    """Router restatement: returns (ids [T,k] int32, scores [T,k] fp32,
    logits [T,E] fp32).  ``forced_ids`` replaces the top-k selection (the
    temporal-reuse routing override) while scores still come from this
    token's softmax."""
    lg = router_logits(x, w_gate_u16, bias)
    ids = topk_ids(lg, k) if forced_ids is None else np.asarray(
        forced_ids, dtype=np.int32).reshape(lg.shape[0], k)
    p = softmax_rows(lg)
    sc = np.take_along_axis(p, ids.astype(np.int64), axis=-1)
    if norm_topk:
        sc = (sc / sc.sum(axis=-1, keepdims=True)).astype(np.float32)
    return ids, sc.astype(np.float32), lg


def moe_combine(y: np.ndarray, scores: np.ndarray,
                shared: np.ndarray | None = None) -> np.ndarray:
    """bf16( sum_j score_j * y_j (+ shared) ), accumulated in fp64;
    y [T,k,H], scores [T,k]."""
    acc = np.einsum("tkh,tk->th", y.astype(np.float64),
                    scores.astype(np.float64))
    if shared is not None:
        acc = acc + shared.astype(np.float64)
    return bf16_round(acc)


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    d = np.linalg.norm(a - b)
    n = np.linalg.norm(b)
    return float(d / n) if n > 0 else float(d)
