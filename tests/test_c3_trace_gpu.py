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
   (test_pool_trace.py).  Including the IO counters.  Misses were served by
   parked kernels (in-step slot fills).
2. Routing and logits against the oracle.  The oracle decodes the same
   tokens with every layer's experts forced to the ones the GPU routed, so
   the two runs stay on one trajectory and every routing decision (ordered
   top-k and next-layer prediction) is compared on its own.  The runs'
   activations differ by bf16 rounding flips; the GPU's combine weights
   measure the resulting router-logit noise (bounded by F32_FACTOR times
   the fp32 restatement's), and a decision may differ only where the
   oracle's own margin is within twice that noise.  The logits
   must be within 1e-3 rel-L2 / 2e-2 max-abs of the oracle's, or within
   F32_FACTOR of the distance an fp32-accumulating restatement of the same
   pipeline, run on the same trajectory, has from it (see F32_FACTOR).
3. Reference pool states.  tests/golden/c3_trace.npz holds the reference
   pool's state after every call on the oracle's own (unforced) trajectory;
   the GPU's pools equal them for as long as the GPU follows that
   trajectory.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import affine as A
from oracle.model import OracleDecoder
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
T_FORCED = 32       # steps of the oracle run on the GPU's trajectory
LOGIT_MAX_ABS = 2e-2
LOGIT_REL = 1e-3
# On this model two CPU restatements of one bf16 pipeline that differ only
# in accumulation (fp64 exact vs fp32) already differ by 7e-3..1.2e-2
# rel-L2 and 2.5e-2..4.7e-2 max-abs in the logits: every bf16 rounding
# turns a tiny difference of its input into whole-ulp flips, and the 4
# layers compound them.  The GPU (fp32 tensor-core accumulation) must stay
# within F32_FACTOR of what the fp32 restatement reaches (worst step), and
# so must its router-logit noise.
F32_FACTOR = 2.5


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
    scores_gpu = np.zeros((T, L, k), np.float32)
    for t in range(T):
        clock["t"] = t
        model.step(torch.tensor([int(g["tokens"][t])], dtype=torch.int32,
                                device=model.device))
        logits.append(bf16_np(model.logits)[0])
        scores_gpu[t] = model.g_scores.reshape(L, k).cpu().numpy()
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

    # 2. every routing decision and every step's logits against the oracle
    #    run on the GPU's own trajectory (each layer's experts forced to the
    #    GPU's), next to an fp32-accumulating restatement of the same bf16
    #    pipeline on that trajectory (what an fp32 implementation such as
    #    MLX's reaches; the calibration of the logits bar)
    forced_by_coin = np.isinf(g["route_margin"])
    ox = OracleDecoder(d, max_len=T + 4)
    of = OracleDecoder(d, max_len=T + 4, exact=False)
    noise = noise32 = 0.0
    n_dec, odd, odd32 = 0, [], 0
    rows = []
    for t in range(T_FORCED):
        forced = {l: ids_gpu[t, l] for l in range(L)}
        lx, _, preds = ox.step(int(g["tokens"][t]), forced=forced,
                               predict=True)
        lf, _, preds32 = of.step(int(g["tokens"][t]), forced=forced,
                                 predict=True)
        noise32 = max(noise32, max(_log_ratio_spread(of.route_scores[l],
                                                     ox.route_scores[l])
                                   for l in range(L)))
        want, f32 = A.bf16_round(lx), A.bf16_round(lf)
        rows.append((A.rel_l2(logits[t], want),
                     float(np.max(np.abs(logits[t] - want))),
                     A.rel_l2(f32, want), float(np.max(np.abs(f32 - want)))))
        for l in range(L):
            noise = max(noise, _log_ratio_spread(scores_gpu[t, l],
                                                 ox.route_scores[l]))
            if not forced_by_coin[t, l]:
                n_dec += 1
                if not np.array_equal(ox.route_own[l], ids_gpu[t, l]):
                    odd.append((t, l, "route", float(ox.own_margin[l])))
                odd32 += not np.array_equal(ox.route_own[l], of.route_own[l])
            if (t, l) in pred_gpu and l + 1 < L:
                n_dec += 1
                pid, psc = pred_gpu[(t, l)]
                odd32 += not np.array_equal(preds[l][0], preds32[l][0])
                if np.array_equal(preds[l][0], pid):
                    noise = max(noise, _log_ratio_spread(psc, preds[l][1]))
                else:
                    odd.append((t, l, "pred", float(ox.pred_margin[l])))
    r = np.array(rows)
    print(f"c3 trace: {n_dec} routing decisions over {T_FORCED} steps, "
          f"{len(odd)} differ ({odd32} for the fp32 restatement; oracle "
          f"margins "
          f"{[round(m, 4) for *_, m in odd]}); router-logit noise "
          f"{noise:.2e} (fp32 restatement {noise32:.2e}); logits rel-L2 "
          f"GPU {r[:, 0].max():.2e} vs fp32 restatement "
          f"{r[:, 2].max():.2e}, max-abs GPU {r[:, 1].max():.2e}"
          f" vs {r[:, 3].max():.2e}; parks {model.host_times['parks']}")
    assert noise <= F32_FACTOR * noise32, (noise, noise32)
    for t, l, kind, m in odd:
        assert m <= 2 * noise, (t, l, kind, m, noise)
    assert len(odd) <= n_dec // 5, odd
    assert r[:, 0].max() <= max(LOGIT_REL, F32_FACTOR * r[:, 2].max())
    assert r[:, 1].max() <= max(LOGIT_MAX_ABS, F32_FACTOR * r[:, 3].max())

    # 3. while the GPU follows the oracle's own (unforced) trajectory, its
    #    pools equal the reference pool's states on it
    n_same = T
    for t in range(T):
        same = all(np.array_equal(ids_gpu[t, l], g["ids"][t, l])
                   for l in range(L))
        same &= all(np.array_equal(pred_gpu[(t, l)][0], g["pred_ids"][t, l + 1])
                    for l in range(L - 1) if (t, l) in pred_gpu)
        if not same:
            n_same = t
            break
        for l in range(L):
            check_snap(g, f"L{l}_", t, snaps[l][t], "lru")
    print(f"c3 trace: reference pool states matched for {n_same}/{T} steps")
    assert n_same >= 1


def _log_ratio_spread(a, b) -> float:
    """max |log a_i - log b_i - mean_j(log a_j - log b_j)|: the largest
    difference between two runs' router logits of the same picks, up to
    the common offset that the softmax removes."""
    dd = np.log(np.asarray(a, np.float64)) - np.log(np.asarray(b, np.float64))
    return float(np.max(np.abs(dd - dd.mean())))
