"""Pool / IO bookkeeping parity against the reference's own code (CPU).

The fixtures in tests/golden were produced by running the reference's
streamlx/stindex.py, reader.py, pool.py and integrate.py under a numpy
stand-in for mlx (tests/golden/make_golden.py).  Here the same inputs are
replayed through this package's pools with a bookkeeping-only slot store and
every per-call state is compared bit-exactly: LRU order and slots, free list,
S3-FIFO queues, hit/miss/eviction/adopt/prefetch counters, IO counters.
"""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

from streamlx_b200 import synth
from streamlx_b200.integrate import StreamingSwitchGLU
from streamlx_b200.pool import StreamingSwitchMLP
from streamlx_b200.reader import ExpertReader
from streamlx_b200.stindex import PARTS, PROJS, SafetensorsIndex

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
COUNTERS = ("hits", "misses", "evictions", "adopted", "pf_calls",
            "pf_launched", "pf_used", "pf_agree_hit", "pf_agree_tot",
            "sweep_experts")


@pytest.fixture(scope="module")
def models(tmp_path_factory):
    root = tmp_path_factory.mktemp("golden_models")
    cfg = synth.SynthConfig(name="golden_e256", hidden=64, layers=3,
                            n_experts=256, top_k=10, inter=64, expert_bits=2,
                            zipf_s=1.1)
    d256 = synth.write_model(str(root / "e256"), cfg, seed=3)
    cfg1 = synth.SynthConfig(name="golden_c1", hidden=64, layers=1,
                             n_experts=32, top_k=4, inter=64, expert_bits=4)
    d32 = synth.write_model(str(root / "e32"), cfg1, seed=4)
    return {"e256": d256, "e32": d32}


def snap(pool):
    c = [getattr(pool, n) for n in COUNTERS]
    return (c, list(pool.id2slot.items()),
            (list(pool.q_small.items()), list(pool.q_main.items()),
             list(pool.q_ghost.keys())), list(pool.free))


def check_snap(g: dict, prefix: str, i: int, s, policy: str):
    c, lru, (sm, mn, gh), fr = s
    assert list(g[prefix + "counters"][i]) == c, (prefix, i, "counters")
    gl = g[prefix + "lru"][i]
    assert [tuple(x) for x in gl[gl[:, 0] >= 0].tolist()] == lru, (prefix, i)
    gf = g[prefix + "free"][i]
    assert gf[gf >= 0].tolist() == fr, (prefix, i, "free")
    if policy.startswith("s3"):
        for key, got in (("s3_small", sm), ("s3_main", mn)):
            a = g[prefix + key][i]
            assert [tuple(x) for x in a[a[:, 0] >= 0].tolist()] == got, key
        a = g[prefix + "s3_ghost"][i]
        assert a[a >= 0].tolist() == gh


def _pools(d, n_layers, n_slots):
    index = SafetensorsIndex(d)
    reader = ExpertReader(index, pinned=False)
    pools = [StreamingSwitchMLP(d, l, n_slots, index=index, reader=reader,
                                store="null") for l in range(n_layers)]
    return index, reader, pools


DECODE = ["trace_c1_lru", "trace_e256_lru_pf", "trace_e256_lru_nopf",
          "trace_e256_lru_pfbad", "trace_e256_lru_pf_topm3",
          "trace_e256_s3p_pf", "trace_e256_s3p_nopf", "trace_c1_s3p"]


@pytest.mark.parametrize("name", DECODE)
def test_decode_trace_matches_reference(models, name, monkeypatch):
    meta = json.load(open(os.path.join(GOLD, name + ".json")))
    g = np.load(os.path.join(GOLD, name + ".npz"))
    policy = "s3fifo" if meta["policy"].startswith("s3fifo") else "lru"
    monkeypatch.setenv("STREAMLX_EVICT", policy)
    monkeypatch.setattr(StreamingSwitchMLP, "_PF_TOPM", meta["topm"])
    d = models["e32" if name.startswith("trace_c1") else "e256"]
    ids, pi, ps = g["ids"], g["pred_ids"], g["pred_scores"]
    # the reference's gate stand-in returned bf16 scores (ties by index)
    import ml_dtypes
    ps = ps.astype(ml_dtypes.bfloat16).astype(np.float32)
    steps, L, k = ids.shape
    _, reader, pools = _pools(d, L, meta["n_slots"])
    wr = [StreamingSwitchGLU(p) for p in pools]
    clock = {"t": 0}
    if meta["prefetch"]:
        for l in range(L - 1):
            wr[l]._pf_next = (pools[l + 1],
                              lambda x, l=l: (pi[clock["t"], l + 1],
                                              ps[clock["t"], l + 1]))
    for t in range(steps):
        clock["t"] = t
        for l in range(L):
            pred = wr[l]._pf_pred(None, k)
            assert wr[l].route(ids[t, l][None, None, :], pred) == "pool"
            check_snap(g, f"L{l}_", t, snap(pools[l]), meta["policy"])
    from streamlx_b200.integrate import _pf_ex
    _pf_ex().submit(lambda: None).result()
    for l, p in enumerate(pools):
        want = meta["final_stats"][l]
        got = {k2: v for k2, v in p.stats.items()
               if k2 not in ("fetch_s", "sweep_fetch_s")}
        assert got == want, (l, got, want)
        assert {str(k2): v for k2, v in p.pf_rank.items()} == meta["pf_rank"][l]
    reader.close()


@pytest.mark.parametrize("tag", ["sweep_lru_warm1", "sweep_lru_warm0",
                                 "slice_lru_warm1", "sweep_s3fifo_warm1"])
def test_prefill_trace_matches_reference(models, tag, monkeypatch):
    g = np.load(os.path.join(GOLD, "trace_prefill.npz"))
    mode, pol, warm = tag.split("_")
    monkeypatch.setenv("STREAMLX_EVICT", pol)
    monkeypatch.setenv("STREAMLX_PREFILL", mode)
    monkeypatch.setenv("STREAMLX_SWEEP_BATCH", "16")
    monkeypatch.setenv("STREAMLX_SWEEP_WARM", warm[-1])
    d = models["e256"]
    index = SafetensorsIndex(d)
    reader = ExpertReader(index, pinned=False)
    pool = StreamingSwitchMLP(d, 1, 24, index=index, reader=reader,
                              store="null")
    w = StreamingSwitchGLU(pool)
    pre = f"{tag}__"
    calls = [g["small_ids"][None]] + [g["pre_ids"][None]] + \
        [g["dec_ids"][t][None, None] for t in range(40)]
    for i, idx in enumerate(calls):
        mode_run = w.route(idx)
        if mode_run == "sweep":
            w._expert_sweep(None, idx)
        elif mode_run == "slice":
            w._slice_prefill(None, idx)
        check_snap(g, pre, i, snap(pool), pol)
    reader.close()


def test_unpatched_reference_s3fifo_raises_keyerror():
    """The reference's S3-FIFO crashes at step 0 on both workload shapes;
    the protected variant here replays the same inputs without error
    (test_decode_trace_matches_reference[...s3p...])."""
    rec = json.load(open(os.path.join(GOLD, "s3_unpatched.json")))
    for tag in ("c1", "e256"):
        assert rec[tag]["error"][0] == "KeyError"
        assert rec[tag]["error"][2] == 0


def test_stindex_matches_reference(models):
    gold = json.load(open(os.path.join(GOLD, "stindex.json")))
    for tag, layers in gold.items():
        idx = SafetensorsIndex(models[tag])
        for L, want in layers.items():
            tr = idx.switch_triples(int(L))
            assert idx.layer_expert_bytes(int(L)) == want["bytes"]
            for p in PROJS:
                assert list(idx.quant_params(tr[p])) == want["qparams"][p]
                for q in PARTS:
                    loc = tr[p][q]
                    assert [os.path.basename(loc.path), loc.abs_start,
                            loc.nbytes, loc.dtype, list(loc.shape),
                            loc.name] == want["locs"][p][q]
                    assert [list(loc.expert_range(e))[1:]
                            for e in (0, 1, loc.shape[0] - 1)] == \
                        want["ranges"][p][q]
        with pytest.raises(IndexError):
            tr["gate_proj"]["weight"].expert_range(10 ** 6)
        with pytest.raises(KeyError):
            idx.switch_triples(99)


def test_reader_plans_and_counters_match_reference(models):
    gold = json.load(open(os.path.join(GOLD, "reader_plans.json")))
    idx = SafetensorsIndex(models["e256"])
    rd = ExpertReader(idx, pinned=False)
    tr = idx.switch_triples(1)
    for tag, want in gold.items():
        rd.merge_gap, rd.max_span = want["merge_gap"], want["max_span"]
        reqs = []
        for e in want["ids"]:
            for p in PROJS:
                for q in PARTS:
                    path, off, n = tr[p][q].expert_range(e)
                    reqs.append(((e, p, q), path, off, n))
        spans = rd._plan(reqs)
        got = [[os.path.basename(s[0]), s[1], s[2],
                [[list(m[0]), m[1], m[2]] for m in s[3]]] for s in spans]
        assert got == want["spans"], tag
        rd.reset_stats()
        raw = rd.read_experts_raw(tr, want["ids"])
        assert (rd.bytes_read, rd.useful_bytes, rd.reads) == \
            (want["bytes_read"], want["useful_bytes"], want["reads"])
        for key, dsum in want["digest"].items():
            e, p, q = key.split(".")
            v = raw[(int(e), p, q)]
            assert int(np.frombuffer(v, dtype=np.uint8).astype(np.uint64)
                       .sum()) == dsum
        rd.release_raw(raw)
    rd.close()


def test_short_read_raises_ioerror(models, tmp_path):
    import shutil
    d = tmp_path / "trunc"
    shutil.copytree(models["e32"], d)
    shard = sorted(p for p in os.listdir(d) if p.endswith(".safetensors"))[0]
    full = os.path.getsize(d / shard)
    idx = SafetensorsIndex(str(d))
    with open(d / shard, "r+b") as f:
        f.truncate(full - 4096)
    rd = ExpertReader(idx, pinned=False)
    tr = idx.switch_triples(0)
    with pytest.raises(IOError):
        rd.read_experts_raw(tr, [31])
    rd.close()


def test_pool_argument_errors(models):
    with pytest.raises(ValueError):
        StreamingSwitchMLP(models["e32"], 0, 0, store="null")
    p = StreamingSwitchMLP(models["e32"], 0, 2, store="null")
    with pytest.raises(ValueError):
        p(None, [1, 2, 3])          # k > n_slots (streamlx/pool.py:300-301)


def test_vlm_export_names_resolve(tmp_path):
    """An mlx-vlm export of a text-only checkpoint (keys and quantization
    overrides prefixed with ``language_model.``, router matrix under
    ``.mlp.gate.proj.``) resolves every mlx-lm name to the same bytes, and
    its expert tensors to the same ranges and quantization parameters, as
    the native export (streamlx/integrate.py:349-394)."""
    from .vlm_copy import write_vlm_copy
    cfg = synth.PRESETS["tiny_dec"]
    d = synth.write_model(str(tmp_path / "native"), cfg, seed=5)
    v = write_vlm_copy(d, str(tmp_path / "vlm"))
    a, b = SafetensorsIndex(d), SafetensorsIndex(v)
    assert a.aliases == {} and len(b.aliases) == len(a.tensors)
    assert any(".mlp.gate.proj." in k for k in b.tensors)
    for name, loc in a.tensors.items():
        got = b.get(name)
        assert (got.nbytes, got.dtype, got.shape) == \
            (loc.nbytes, loc.dtype, loc.shape), name
        assert b.read_tensor(name) == a.read_tensor(name), name
    for L in range(cfg.layers):
        ta, tb = a.switch_triples(L), b.switch_triples(L)
        assert a.layer_expert_bytes(L) == b.layer_expert_bytes(L)
        for p in PROJS:
            assert b.quant_params(tb[p]) == a.quant_params(ta[p])
            for q in PARTS:
                for e in (0, cfg.n_experts - 1):
                    (pa, oa, na), (pb, ob, nb) = (ta[p][q].expert_range(e),
                                                  tb[p][q].expert_range(e))
                    with open(pa, "rb") as fa, open(pb, "rb") as fb:
                        assert os.pread(fa.fileno(), na, oa) == \
                            os.pread(fb.fileno(), nb, ob)
    with pytest.raises(KeyError):
        b.get("model.layers.0.mlp.nothing.weight")
    # one unprefixed key in the weight map: a native export, no remap
    p = os.path.join(v, "model.safetensors.index.json")
    wm = json.load(open(p))
    wm["weight_map"]["lm_head.weight"] = "x"
    json.dump(wm, open(p, "w"))
    assert SafetensorsIndex(v).aliases == {}
