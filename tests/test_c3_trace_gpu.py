"""117B-shaped decode on the GPU: pool trace and routing against the
reference.

The workload is the 117B-shaped decoder (hidden 2560, 24/4 heads, 256 2-bit
experts top-10, inter 1024, Zipf 1.1 routing with 60% temporal reuse) cut to
4 layers and a 4096-token vocabulary, 64 LRU slots per layer (25% of the
experts), next-layer prefetch top-m 7, a fixed 48-token sequence.

Three checks:

1. Bookkeeping.  Every pool call of the graph decoder (whose slot fills and
   table installs happen inside parked kernels and between steps) leaves the
   pool in exactly the state that this package's pool code reaches when the
   GPU run's own routed ids and next-layer predictions are replayed through
   it on the CPU -- and that pool code is pinned, call for call, to the
   reference's own pool.py / integrate.py by the CPU golden tests
   (test_pool_trace.py).  Including the IO counters.
2. Routing against the reference composition.  tests/golden/c3_trace.npz
   holds what the CPU oracle decoded on the same sequence (routed ids,
   predictions, logits, and the smallest logit gap behind each decision) and
   the reference pool's state after every call when fed those ids.  The
   GPU's ids and predictions must equal the oracle's, in order, up to the
   first decision whose oracle margin is below NEAR_TIE (the two runs'
   activations differ by bf16 rounding flips, so a near-tied decision may
   fall either way; after it the runs follow different experts).  Until then
   the pool states equal the reference's and the logits are within
   tolerance.  That point must come after MIN_STEPS steps.
3. Misses were served by parked kernels (in-step slot fills).
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import affine as A
from streamlx_b200 import synth
from streamlx_b200.integrate import StreamingSwitchGLU, _pf_ex, \
    load_streaming_model
from streamlx_b200.pool import StreamingSwitchMLP
from streamlx_b200.reader import ExpertReader
from streamlx_b200.stindex import SafetensorsIndex

from .kernel_cases import bf16_np
from .test_pool_trace import check_snap, snap

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NEAR_TIE = 5e-3     # logit units: far above the routers' input noise
MIN_STEPS = 8
LOGIT_MAX_ABS = 2e-2
LOGIT_REL = 5e-3    # bf16 SwiGLU rounding flips (measured ~3e-3)


def _stats(p):
    return {k: v for k, v in p.stats.items()
            if k not in ("fetch_s", "sweep_fetch_s")}


def test_c3_shape_decode_trace(tmp_path, monkeypatch):
    meta = json.load(open(os.path.join(GOLD, "c3_trace.json")))
    g = np.load(os.path.join(GOLD, "c3_trace.npz"))
    monkeypatch.setenv("STREAMLX_EVICT", "lru")
    monkeypatch.setenv("STREAMLX_PREFETCH", "1")
    monkeypatch.setattr(StreamingSwitchMLP, "_PF_TOPM", meta["topm"])
    cfg = synth.PRESETS[meta["preset"]]
    d = synth.write_model(str(tmp_path / "c3"), cfg, seed=meta["seed"])
    bpe = synth.expert_bytes(cfg.hidden, cfg.inter, cfg.expert_bits, 64)
    model, _, pools, reader = load_streaming_model(
        d, budget_bytes=meta["slots"] * bpe * cfg.layers, k=cfg.top_k)
    assert all(p.n_slots == meta["slots"] for p in pools.values())
    assert model.use_graphs
    L, k = cfg.layers, cfg.top_k
    T = len(g["tokens"])

    ids_gpu = np.full((T, L, k), -1, np.int64)
    pred_gpu = {}                       # (t, layer) -> (ids, scores)
    snaps: dict = {l: [] for l in pools}
    clock = {"t": 0}
    for l in pools:
        w = model.layers[l].mlp.switch_mlp
        orig_route, orig_pf = w.route, w.start_prefetch

        def route(idx, pred=None, start_prefetch=True, _o=orig_route, _l=l):
            ids_gpu[clock["t"], _l] = np.asarray(idx).reshape(-1)
            r = _o(idx, pred, start_prefetch=start_prefetch)
            snaps[_l].append(snap(pools[_l]))
            return r

        def start_prefetch(pred, _o=orig_pf, _l=l):
            pred_gpu[(clock["t"], _l)] = (np.asarray(pred[0]).copy(),
                                          np.asarray(pred[1]).copy())
            return _o(pred)
        w.route, w.start_prefetch = route, start_prefetch

    logits = []
    for t in range(T):
        clock["t"] = t
        model.step(torch.tensor([int(g["tokens"][t])], dtype=torch.int32,
                                device=model.device))
        logits.append(bf16_np(model.logits)[0])
    model.flush()
    _pf_ex().submit(lambda: None).result()     # the last prefetch reads
    assert model.host_times["parks"] > 0       # misses served in-step
    assert all(len(s) == T for s in snaps.values())
    gpu_stats = [_stats(pools[l]) for l in range(L)]
    reader.close()

    # 1. the GPU run's bookkeeping == the pinned pool code on its inputs
    index = SafetensorsIndex(d)
    rd = ExpertReader(index, pinned=False)
    cpu = [StreamingSwitchMLP(d, l, meta["slots"], index=index, reader=rd,
                              store="null") for l in range(L)]
    wr = [StreamingSwitchGLU(p) for p in cpu]
    for l in range(L - 1):
        wr[l]._pf_next = (cpu[l + 1],
                          lambda x, l=l: pred_gpu[(clock["t"], l)])
    for t in range(T):
        clock["t"] = t
        for l in range(L):
            pred = wr[l]._pf_pred(None, k) if (t, l) in pred_gpu else None
            assert wr[l].route(ids_gpu[t, l][None, None, :], pred) == "pool"
            assert snap(cpu[l]) == snaps[l][t], (t, l)
    _pf_ex().submit(lambda: None).result()
    assert [_stats(p) for p in cpu] == gpu_stats
    rd.close()

    # 2. agreement with the oracle and the reference pool up to the first
    #    near-tied decision
    first = None
    for t in range(T):
        for l in range(L):
            same = np.array_equal(ids_gpu[t, l], g["ids"][t, l])
            if (t, l) in pred_gpu and l + 1 < L:
                same &= np.array_equal(pred_gpu[(t, l)][0],
                                       g["pred_ids"][t, l + 1])
            if not same:
                first = (t, l)
                break
        if first:
            break
    if first is not None:
        t0, l0 = first
        margin = min(g["route_margin"][t0, l0],
                     g["pred_margin"][t0, l0 + 1] if l0 + 1 < L else np.inf)
        assert margin < NEAR_TIE, (first, margin)
        assert t0 >= MIN_STEPS, first
    n_steps = T if first is None else first[0]
    worst_rel = worst_abs = 0.0
    for t in range(n_steps):
        want = A.bf16_from_bits(g["logits_bf16"][t])
        worst_rel = max(worst_rel, A.rel_l2(logits[t], want))
        worst_abs = max(worst_abs, float(np.max(np.abs(logits[t] - want))))
        for l in range(L):
            check_snap(g, f"L{l}_", t, snaps[l][t], "lru")
    print(f"c3 trace: oracle agreement for {n_steps}/{T} steps "
          f"(first near-tie {first}); logits worst rel-L2 {worst_rel:.2e} "
          f"max-abs {worst_abs:.2e}; parks {model.host_times['parks']}")
    assert worst_abs <= LOGIT_MAX_ABS
    assert worst_rel <= LOGIT_REL, worst_rel
