"""Generate the golden fixtures in tests/golden/ by running the REFERENCE's own
Python code (streamlx/stindex.py, reader.py, pool.py, integrate.py) under a
numpy stand-in for mlx (tests/golden/mlx_stub).

Run from the repo root, naming the reference checkout (the directory that
holds the ``streamlx`` package):

    python tests/golden/make_golden.py --reference <path-to-streamlx-checkout>

(or set ``STREAMLX_REFERENCE``).  The fixtures pin, bit-exactly, what the
reference decides: safetensors byte ranges, span-merge plans, the per-call
pool state (LRU order, slots, S3-FIFO queues, hit/miss/eviction/adopt/
prefetch counters) for decode, prefetch, expert-major prefill sweeps and
slice prefill, the residency water-fill, and the warm-start preload.  The
routing inputs are stored beside the traces, so replaying them needs neither
the reference nor this script.

The reference's S3-FIFO raises KeyError whenever one call inserts more new
experts than its small FIFO holds (streamlx/pool.py:139-150 evicts them, then
pool.py:195-196 looks them up).  That is recorded as-is (``s3_unpatched``),
and the S3-FIFO traces are taken from a runtime-patched copy in which ids
touched or inserted during the current wrapper call are protected: a
protected small-queue head is promoted to main instead of being ghosted, and
main eviction skips protected entries.  The reference checkout itself is
never modified.
"""

from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(HERE, "mlx_stub"))

import ml_dtypes  # noqa: E402

from streamlx_b200 import synth  # noqa: E402

BF16 = ml_dtypes.bfloat16
ref_int = ref_pool = ref_reader = ref_st = None


def load_reference(path: str) -> None:
    """Import the reference's streamlx modules from a checkout directory."""
    global ref_int, ref_pool, ref_reader, ref_st
    if not os.path.isdir(os.path.join(path, "streamlx")):
        raise SystemExit(f"{path}: no streamlx package there")
    sys.path.insert(0, path)
    import streamlx.integrate as ri
    import streamlx.pool as rp
    import streamlx.reader as rr
    import streamlx.stindex as rs
    ref_int, ref_pool, ref_reader, ref_st = ri, rp, rr, rs


# ---------------------------------------------------------------- inputs --

def zipf_routing(E, k, steps, layers, s, repeat_p, seed):
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    rank = np.empty(E, dtype=np.int64)
    rank[perm] = np.arange(E)
    p = 1.0 / np.power(rank + 1.0, s)
    p /= p.sum()
    ids = np.zeros((steps, layers, k), dtype=np.int32)
    for t in range(steps):
        for l in range(layers):
            if t > 0 and rng.random() < repeat_p:
                ids[t, l] = ids[t - 1, l]
            else:
                ids[t, l] = rng.choice(E, k, replace=False, p=p)
    return ids


def predictions(ids, E, agree, seed):
    rng = np.random.default_rng(seed)
    steps, layers, k = ids.shape
    pi = np.zeros_like(ids)
    ps = np.zeros(ids.shape, dtype=np.float32)
    for t in range(steps):
        for l in range(layers):
            cur = [int(e) for e in ids[t, l]]
            out = []
            for e in cur:
                if rng.random() > agree:
                    while True:
                        c = int(rng.integers(E))
                        if c not in cur and c not in out:
                            break
                    out.append(c)
                else:
                    out.append(e)
            pi[t, l] = out
            ps[t, l] = rng.random(k).astype(np.float32)
    return pi, ps


class GateStub:
    """Stands in for the next layer's router: returns (inds, scores)."""

    def __init__(self, pi, ps, layer, clock, score_dtype=BF16):
        self.pi, self.ps, self.layer, self.clock = pi, ps, layer, clock
        self.score_dtype = score_dtype

    def __call__(self, x):
        t = self.clock["t"]
        return (self.pi[t, self.layer][None, None, :].astype(np.uint32),
                self.ps[t, self.layer][None, None, :].astype(
                    self.score_dtype))


# ------------------------------------------------------------ patching --

def install_s3_protection():
    """Runtime patch of the reference S3-FIFO (see module docstring)."""
    P = ref_pool.StreamingSwitchMLP
    W = ref_int.StreamingSwitchGLU
    if getattr(P, "_golden_patched", False):
        return
    orig_call, orig_ensure, orig_touch, orig_adopt = (
        W.__call__, P.ensure, P.touch, P.adopt)

    def call(self, x, indices):
        self.pool._protect = set()
        return orig_call(self, x, indices)

    def ensure(self, ids):
        self.__dict__.setdefault("_protect", set()).update(int(e) for e in ids)
        return orig_ensure(self, ids)

    def touch(self, ids):
        self.__dict__.setdefault("_protect", set()).update(int(e) for e in ids)
        return orig_touch(self, ids)

    def adopt(self, e, arrays):
        self.__dict__.setdefault("_protect", set()).add(int(e))
        return orig_adopt(self, e, arrays)

    def s3_evict_main(self):
        prot = self.__dict__.get("_protect", set())
        skipped = 0
        while self.q_main:
            e, f = self.q_main.popitem(last=False)
            if e in prot:
                self.q_main[e] = f
                skipped += 1
                if skipped > len(self.q_main):
                    break
                continue
            skipped = 0
            if f > 0:
                self.q_main[e] = f - 1
                continue
            return e
        raise RuntimeError("s3fifo: no evictable main entry")

    def s3_insert(self, e):
        prot = self.__dict__.get("_protect", set())
        if e in self.q_ghost:
            del self.q_ghost[e]
            victim = (self._s3_evict_main()
                      if len(self.q_main) >= self.n_main else None)
            self.q_main[e] = 0
            return victim
        victim = None
        if len(self.q_small) >= self.n_small:
            e2, f = self.q_small.popitem(last=False)
            if f > 0 or e2 in prot:
                if len(self.q_main) >= self.n_main:
                    victim = self._s3_evict_main()
                self.q_main[e2] = 0
            else:
                if len(self.q_ghost) >= self.n_main:
                    self.q_ghost.popitem(last=False)
                self.q_ghost[e2] = True
                victim = e2
        self.q_small[e] = 0
        return victim

    W.__call__ = call
    P.ensure, P.touch, P.adopt = ensure, touch, adopt
    P._s3_evict_main, P._s3_insert = s3_evict_main, s3_insert
    P._golden_patched = True


# ------------------------------------------------------------ snapshots --

COUNTERS = ("hits", "misses", "evictions", "adopted", "pf_calls",
            "pf_launched", "pf_used", "pf_agree_hit", "pf_agree_tot",
            "sweep_experts")


def snap(pool):
    c = [getattr(pool, n) for n in COUNTERS]
    lru = list(pool.id2slot.items())
    s3 = (list(pool.q_small.items()), list(pool.q_main.items()),
          list(pool.q_ghost.keys()))
    return c, lru, s3, list(pool.free)


def pack_snaps(snaps, n_slots, n_small, n_main):
    n = len(snaps)
    cnt = np.array([s[0] for s in snaps], dtype=np.int64)
    lru = np.full((n, n_slots, 2), -1, dtype=np.int32)
    small = np.full((n, n_small + 1, 2), -1, dtype=np.int32)
    main = np.full((n, n_main + 1, 2), -1, dtype=np.int32)
    ghost = np.full((n, n_main + 1), -1, dtype=np.int32)
    free = np.full((n, n_slots), -1, dtype=np.int32)
    for i, (_, l, (sm, mn, gh), fr) in enumerate(snaps):
        if l:
            lru[i, :len(l)] = l
        if sm:
            small[i, :len(sm)] = sm
        if mn:
            main[i, :len(mn)] = mn
        if gh:
            ghost[i, :len(gh)] = gh
        if fr:
            free[i, :len(fr)] = fr
    return dict(counters=cnt, lru=lru, s3_small=small, s3_main=main,
                s3_ghost=ghost, free=free)


# -------------------------------------------------------------- drivers --

def norm_weights(L, H, seed):
    rng = np.random.default_rng(seed)
    return [(1.0 + 0.05 * rng.standard_normal(H)).astype(BF16)
            for _ in range(L)]


def run_decode(model_dir, n_slots, ids, pi, ps, policy, prefetch, topm, H,
               x_seed=5, score_dtype=BF16):
    os.environ["STREAMLX_EVICT"] = policy
    os.environ["STREAMLX_PREFILL"] = "sweep"
    ref_pool.StreamingSwitchMLP._PF_TOPM = topm
    index = ref_st.SafetensorsIndex(model_dir)
    reader = ref_reader.ExpertReader(index)
    steps, L, k = ids.shape
    pools = [ref_pool.StreamingSwitchMLP(model_dir, l, n_slots, index=index,
                                         reader=reader) for l in range(L)]
    wr = [ref_int.StreamingSwitchGLU(p) for p in pools]
    clock = {"t": 0}
    nw = norm_weights(L, H, 11)
    if prefetch:
        for l in range(L - 1):
            wr[l]._pf_next = (pools[l + 1],
                              GateStub(pi, ps, l + 1, clock, score_dtype),
                              nw[l], nw[l + 1])
    rng = np.random.default_rng(x_seed)
    snaps = [[] for _ in range(L)]
    err = None
    try:
        for t in range(steps):
            clock["t"] = t
            for l in range(L):
                x = rng.standard_normal((1, 1, H)).astype(BF16)
                wr[l](x, ids[t, l][None, None, :].astype(np.uint32))
                snaps[l].append(snap(pools[l]))
    except Exception as e:  # noqa: BLE001 - recorded, not hidden
        err = (type(e).__name__, str(e), t, l)
    ref_int._pf_ex().shutdown(wait=True)
    ref_int._PF_EX = None
    pf_rank = [{str(k): v for k, v in p.pf_rank.items()} for p in pools]
    reader.close()
    return snaps, pools, err, pf_rank


def save_decode(name, snaps, pools, ids, pi, ps, meta, pf_rank):
    arrays = {"ids": ids, "pred_ids": pi, "pred_scores": ps}
    p0 = pools[0]
    for l, s in enumerate(snaps):
        for k2, v in pack_snaps(s, p0.n_slots, p0.n_small, p0.n_main).items():
            arrays[f"L{l}_{k2}"] = v
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    meta = dict(meta, counters=list(COUNTERS), pf_rank=pf_rank,
                final_stats=[{k: v for k, v in p.stats.items()
                              if k not in ("fetch_s", "sweep_fetch_s")}
                             for p in pools])
    with open(os.path.join(HERE, f"{name}.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)


def main():
    import argparse
    ap = argparse.ArgumentParser(description="write tests/golden fixtures")
    ap.add_argument("--reference",
                    default=os.environ.get("STREAMLX_REFERENCE"),
                    help="reference checkout (holds the streamlx package)")
    ap.add_argument("--only", default=None,
                    help="comma list of fixture groups to (re)write: "
                         "core,residency")
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("name the reference checkout with --reference or "
                         "STREAMLX_REFERENCE")
    load_reference(args.reference)
    only = set(args.only.split(",")) if args.only else {"core", "residency",
                                                        "c3trace"}
    tmp = tempfile.mkdtemp(prefix="slx_golden_")
    try:
        if "core" in only:
            _main(tmp)
        if "residency" in only:
            _residency(tmp)
        if "c3trace" in only:
            _c3trace(tmp)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


C3_TRACE = dict(preset="laguna_c3_4l", seed=11, tokens=48, slots=64,
                topm=7, token_seed=5, repeat_seed=12345)


def _c3trace(tmp):
    """Decode trace of the 117B-shaped decoder cut to 4 layers: the CPU
    oracle decodes a fixed token sequence (routing, next-layer predictions,
    the temporal-reuse coin drawn as the decoder draws it, logits), and the
    reference's own pool code replays those ids and predictions with 64 LRU
    slots per layer and prefetch top-m 7 (streamlx/integrate.py:234-298,
    streamlx/pool.py:117-280)."""
    from oracle.model import OracleDecoder
    c = C3_TRACE
    cfg = synth.PRESETS[c["preset"]]
    d = synth.write_model(os.path.join(tmp, "c3"), cfg, seed=c["seed"])
    T, L, k = c["tokens"], cfg.layers, cfg.top_k
    toks = np.random.default_rng(c["token_seed"]).integers(0, cfg.vocab, T)
    coin = np.random.default_rng(c["repeat_seed"])
    o = OracleDecoder(d, max_len=T + 4)
    ids = np.zeros((T, L, k), np.int32)
    pi = np.full((T, L, k), -1, np.int32)
    ps = np.zeros((T, L, k), np.float32)
    logits = np.zeros((T, cfg.vocab), np.uint16)
    rmargin = np.zeros((T, L), np.float64)
    pmargin = np.full((T, L), np.inf)
    prev = None
    for t in range(T):
        forced = {}
        for i in range(L):
            if cfg.repeat_p and t > 0 and coin.random() < cfg.repeat_p:
                forced[i] = prev[i]
        lg, routed, preds = o.step(int(toks[t]), forced=forced, predict=True)
        logits[t] = BF16_BITS(lg)
        rmargin[t] = o.route_margin
        for i in range(L - 1):
            pmargin[t, i + 1] = o.pred_margin[i]
        for i in range(L):
            ids[t, i] = routed[i]
            if preds[i] is not None:
                # prediction made at layer i is for layer i + 1
                pi[t, i + 1], ps[t, i + 1] = preds[i]
        prev = [r.copy() for r in routed]
        print(f"[c3trace] token {t + 1}/{T}", flush=True)
    # the trace needs the reference's bookkeeping, not its expert outputs:
    # the stand-in's gather_qmm returns zeros of the right shape here
    import mlx.core as mxc
    full_qmm = mxc.gather_qmm

    def shape_only_qmm(x, w, scales, biases, rhs_indices=None, **kw):
        x = np.asarray(x)
        idx = np.asarray(rhs_indices)
        batch = np.broadcast_shapes(x.shape[:-2], idx.shape)
        return np.zeros(batch + (x.shape[-2], w.shape[-2]), dtype=BF16)

    mxc.gather_qmm = shape_only_qmm
    try:
        # the decoder orders a prediction by its fp32 scores
        snaps, pools, err, pfr = run_decode(d, c["slots"], ids, pi, ps, "lru",
                                            True, c["topm"], cfg.hidden,
                                            score_dtype=np.float32)
    finally:
        mxc.gather_qmm = full_qmm
    assert err is None, err
    arrays = {"tokens": toks.astype(np.int32), "ids": ids, "pred_ids": pi,
              "pred_scores": ps, "logits_bf16": logits,
              "route_margin": rmargin, "pred_margin": pmargin}
    p0 = pools[0]
    for l, sn in enumerate(snaps):
        for k2, v in pack_snaps(sn, p0.n_slots, p0.n_small,
                                p0.n_main).items():
            arrays[f"L{l}_{k2}"] = v
    np.savez_compressed(os.path.join(HERE, "c3_trace.npz"), **arrays)
    meta = dict(c, counters=list(COUNTERS), pf_rank=pfr,
                final_stats=[{k3: v for k3, v in p.stats.items()
                              if k3 not in ("fetch_s", "sweep_fetch_s")}
                             for p in pools])
    with open(os.path.join(HERE, "c3_trace.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)


def BF16_BITS(a):
    return np.asarray(a, dtype=np.float32).astype(BF16).view(np.uint16)


def _residency(tmp):
    """plan_residency water-fill decisions and preload_popular warm starts
    (streamlx/integrate.py:322-346, 476-506)."""
    cases = []
    # uniform widths: flips near the total expert bytes
    for budget in (0, 5, 40, 47, 48, 60, 100):
        cases.append(dict(layers=[0, 1, 2, 3], bpe={i: 10 for i in range(4)},
                          n_exp={i: 12 for i in range(4)},
                          budget=budget * 10, k=4))
    # mixed widths (dense-first style models): partial residency
    bpe = {0: 3, 1: 9, 2: 9, 3: 27, 4: 5}
    n_exp = {0: 8, 1: 16, 2: 16, 3: 64, 4: 32}
    for budget in (50, 200, 400, 700, 1500, 2300, 2600):
        for k in (2, 8):
            cases.append(dict(layers=[0, 1, 2, 3, 4], bpe=bpe, n_exp=n_exp,
                              budget=budget, k=k))
    out = []
    for c in cases:
        res, left = ref_int.plan_residency(c["layers"], c["bpe"], c["n_exp"],
                                           c["budget"], c["k"])
        out.append(dict(c, bpe={str(a): b for a, b in c["bpe"].items()},
                        n_exp={str(a): b for a, b in c["n_exp"].items()},
                        resident=sorted(res), left=left))

    # preload_popular on a 3-layer 256-expert stack, trace axes -> layers
    # [2, 0] (layer 1 absent from the trace), 24 slots per pool
    cfg = synth.SynthConfig(name="golden_e256", hidden=64, layers=3,
                            n_experts=256, top_k=10, inter=64, expert_bits=2,
                            zipf_s=1.1)
    d = synth.write_model(os.path.join(tmp, "e256r"), cfg, seed=3)
    rng = np.random.default_rng(41)
    ids = zipf_routing(256, 10, 120, 2, 1.1, 0.3, seed=42)
    # a popularity tie among rarely used experts: the argsort order decides
    ids[:, :, 9] = rng.integers(100, 140, size=ids.shape[:2])
    tr = os.path.join(tmp, "warm.npz")
    np.savez_compressed(tr, experts=ids.astype(np.uint16),
                        seq_id=np.zeros(ids.shape[0], np.uint32),
                        pos=np.arange(ids.shape[0], dtype=np.uint32),
                        prompt_class=np.zeros(ids.shape[0], np.uint8))
    with open(os.path.join(tmp, "warm.meta.json"), "w") as f:
        json.dump({"schema_version": 1, "layer_ids": [2, 0]}, f)
    os.environ["STREAMLX_EVICT"] = "lru"
    index = ref_st.SafetensorsIndex(d)
    reader = ref_reader.ExpertReader(index)
    pools = {i: ref_pool.StreamingSwitchMLP(d, i, 24, index=index,
                                            reader=reader) for i in range(3)}
    n = ref_int.preload_popular(pools, tr)
    pre = {"loaded": n,
           "pools": {str(i): {"id2slot": [[int(a), int(b)] for a, b in
                                          p.id2slot.items()],
                              "free": [int(x) for x in p.free],
                              "misses": p.misses, "hits": p.hits}
                     for i, p in pools.items()}}
    reader.close()
    np.savez_compressed(os.path.join(HERE, "warm_trace.npz"),
                        experts=ids.astype(np.uint16))
    with open(os.path.join(HERE, "residency.json"), "w") as f:
        json.dump({"plan_residency": out, "preload_popular": pre,
                   "preload_layer_ids": [2, 0], "preload_slots": 24},
                  f, indent=1, sort_keys=True)


def _main(tmp):
    # ---- a small 3-layer, 256-expert MoE stack (trace shapes of config 3)
    cfg = synth.SynthConfig(name="golden_e256", hidden=64, layers=3,
                            n_experts=256, top_k=10, inter=64, expert_bits=2,
                            zipf_s=1.1)
    d256 = synth.write_model(os.path.join(tmp, "e256"), cfg, seed=3)
    cfg1 = synth.SynthConfig(name="golden_c1", hidden=64, layers=1,
                             n_experts=32, top_k=4, inter=64, expert_bits=4)
    d32 = synth.write_model(os.path.join(tmp, "e32"), cfg1, seed=4)

    # ---- stindex: byte ranges / quant params
    st = {}
    for tag, d in (("e256", d256), ("e32", d32)):
        idx = ref_st.SafetensorsIndex(d)
        lay = {}
        n_layers = 3 if tag == "e256" else 1
        for L in range(n_layers):
            tr = idx.switch_triples(L)
            lay[str(L)] = {
                "bytes": idx.layer_expert_bytes(L),
                "qparams": {p: list(idx.quant_params(tr[p])) for p in tr},
                "locs": {p: {q: [os.path.basename(loc.path), loc.abs_start,
                                 loc.nbytes, loc.dtype, list(loc.shape),
                                 loc.name]
                             for q, loc in tr[p].items()} for p in tr},
                "ranges": {p: {q: [list(tr[p][q].expert_range(e))[1:]
                                   for e in (0, 1, tr[p][q].shape[0] - 1)]
                               for q in tr[p]} for p in tr},
            }
        st[tag] = lay
    with open(os.path.join(HERE, "stindex.json"), "w") as f:
        json.dump(st, f, indent=1, sort_keys=True)

    # ---- reader: span plans and IO counters
    idx = ref_st.SafetensorsIndex(d256)
    rd = ref_reader.ExpertReader(idx)
    plans = {}
    for tag, ids, gap, span in (("adj", [3, 4, 5, 17], 64 * 1024, 16 << 20),
                                ("scatter", [200, 3, 77, 9, 10], 64 * 1024,
                                 16 << 20),
                                ("nogap", [3, 4, 5, 17], 0, 16 << 20),
                                ("smallspan", list(range(40)), 64 * 1024,
                                 4096)):
        rd.merge_gap, rd.max_span = gap, span
        tr = idx.switch_triples(1)
        reqs = []
        for e in ids:
            for p in ref_st.PROJS:
                for q in ref_st.PARTS:
                    path, off, n = tr[p][q].expert_range(e)
                    reqs.append(((e, p, q), path, off, n))
        spans = rd._plan(reqs)
        rd.reset_stats()
        raw = rd.read_experts_raw(tr, ids)
        plans[tag] = {
            "ids": ids, "merge_gap": gap, "max_span": span,
            "spans": [[os.path.basename(s[0]), s[1], s[2],
                       [[list(m[0]), m[1], m[2]] for m in s[3]]]
                      for s in spans],
            "bytes_read": rd.bytes_read, "useful_bytes": rd.useful_bytes,
            "reads": rd.reads,
            "digest": {f"{e}.{p}.{q}": int(np.frombuffer(
                raw[(e, p, q)], dtype=np.uint8).astype(np.uint64).sum())
                for (e, p, q) in raw},
        }
    rd.close()
    with open(os.path.join(HERE, "reader_plans.json"), "w") as f:
        json.dump(plans, f, indent=1, sort_keys=True)

    # ---- decode traces
    E, k, H = 256, 10, 64
    ids3 = zipf_routing(E, k, 200, 3, 1.1, 0.6, seed=21)
    pi, ps = predictions(ids3, E, agree=0.7, seed=22)
    pi_bad, ps_bad = predictions(ids3, E, agree=0.25, seed=23)
    ids1 = zipf_routing(32, 4, 256, 1, 1.0, 0.0, seed=24)
    z1 = np.zeros_like(ids1)

    jobs = [
        ("trace_c1_lru", d32, 8, ids1, z1, z1.astype(np.float32), "lru",
         False, 7, False),
        ("trace_e256_lru_pf", d256, 64, ids3, pi, ps, "lru", True, 7, False),
        ("trace_e256_lru_nopf", d256, 64, ids3, pi, ps, "lru", False, 7,
         False),
        ("trace_e256_lru_pfbad", d256, 64, ids3, pi_bad, ps_bad, "lru", True,
         7, False),
        ("trace_e256_lru_pf_topm3", d256, 64, ids3, pi, ps, "lru", True, 3,
         False),
    ]
    unpatched = {}
    for tag, d, ns, ids, kk in (("c1", d32, 8, ids1, 4),
                                ("e256", d256, 64, ids3, 10)):
        _, _, err, _ = run_decode(d, ns, ids, z1 if tag == "c1" else pi,
                                  (z1.astype(np.float32) if tag == "c1"
                                   else ps), "s3fifo", False, 7, H)
        unpatched[tag] = {"n_slots": ns, "k": kk, "error": err}
    with open(os.path.join(HERE, "s3_unpatched.json"), "w") as f:
        json.dump(unpatched, f, indent=1, sort_keys=True)

    for name, d, ns, ids, a, b, pol, pf, topm, _ in jobs:
        snaps, pools, err, pfr = run_decode(d, ns, ids, a, b, pol, pf, topm,
                                            H)
        assert err is None, (name, err)
        save_decode(name, snaps, pools, ids, a, b,
                    {"n_slots": ns, "policy": pol, "prefetch": pf,
                     "topm": topm}, pfr)

    install_s3_protection()
    for name, pf in (("trace_e256_s3p_pf", True), ("trace_e256_s3p_nopf",
                                                   False)):
        snaps, pools, err, pfr = run_decode(d256, 64, ids3, pi, ps, "s3fifo",
                                            pf, 7, H)
        assert err is None, (name, err)
        save_decode(name, snaps, pools, ids3, pi, ps,
                    {"n_slots": 64, "policy": "s3fifo-protected",
                     "prefetch": pf, "topm": 7}, pfr)
    snaps, pools, err, pfr = run_decode(d32, 8, ids1, z1,
                                        z1.astype(np.float32), "s3fifo",
                                        False, 7, H)
    assert err is None, err
    save_decode("trace_c1_s3p", snaps, pools, ids1, z1,
                z1.astype(np.float32),
                {"n_slots": 8, "policy": "s3fifo-protected",
                 "prefetch": False, "topm": 7}, pfr)

    # ---- prefill: expert-major sweep, fast path, slice mode; decode after
    rng = np.random.default_rng(31)
    pre_ids = zipf_routing(E, k, 48, 1, 1.1, 0.0, seed=32)[:, 0, :]
    small_ids = zipf_routing(E, k, 3, 1, 1.1, 0.0, seed=33)[:, 0, :]
    dec_ids = zipf_routing(E, k, 40, 1, 1.1, 0.6, seed=34)[:, 0, :]
    xs = rng.standard_normal((48, H)).astype(BF16)
    xd = rng.standard_normal((40, H)).astype(BF16)
    out = {}
    for mode, pol, warm in (("sweep", "lru", "1"), ("sweep", "lru", "0"),
                            ("slice", "lru", "1"),
                            ("sweep", "s3fifo", "1")):
        os.environ["STREAMLX_EVICT"] = pol
        os.environ["STREAMLX_PREFILL"] = mode
        os.environ["STREAMLX_SWEEP_BATCH"] = "16"
        os.environ["STREAMLX_SWEEP_WARM"] = warm
        index = ref_st.SafetensorsIndex(d256)
        reader = ref_reader.ExpertReader(index)
        pool = ref_pool.StreamingSwitchMLP(d256, 1, 24, index=index,
                                           reader=reader)
        w = ref_int.StreamingSwitchGLU(pool)
        recs = []
        y_small = w(xs[:3][None], small_ids[None].astype(np.uint32))
        recs.append(snap(pool))
        y_big = w(xs[None], pre_ids[None].astype(np.uint32))
        recs.append(snap(pool))
        for t in range(40):
            w(xd[t][None, None], dec_ids[t][None, None].astype(np.uint32))
            recs.append(snap(pool))
        tag = f"{mode}_{pol}_warm{warm}"
        out[tag] = pack_snaps(recs, pool.n_slots, pool.n_small, pool.n_main)
        out[tag]["y_small"] = np.asarray(y_small, dtype=np.float32)
        out[tag]["y_big"] = np.asarray(y_big, dtype=np.float32)
        reader.close()
    arrays = {"pre_ids": pre_ids, "small_ids": small_ids, "dec_ids": dec_ids,
              "xs": xs.view(np.uint16), "xd": xd.view(np.uint16)}
    for tag, d in out.items():
        for k2, v in d.items():
            arrays[f"{tag}__{k2}"] = v
    np.savez_compressed(os.path.join(HERE, "trace_prefill.npz"), **arrays)
    with open(os.path.join(HERE, "trace_prefill.json"), "w") as f:
        json.dump({"n_slots": 24, "layer": 1, "sweep_batch": 16,
                   "tags": sorted(out), "model": "golden_e256 seed 3",
                   "counters": list(COUNTERS)}, f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
