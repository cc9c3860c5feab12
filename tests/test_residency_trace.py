"""Residency water-fill, warm-start preload and the routing-trace format:
decisions pinned against the reference's own functions (tests/golden,
written by make_golden.py from streamlx/integrate.py:322-346,476-506), and
the trace writer's format round trip (examples/capture_trace.py:98-139)."""

from __future__ import annotations

import json
import os

import numpy as np
import pytest

from streamlx_b200 import synth
from streamlx_b200.integrate import plan_residency, preload_popular
from streamlx_b200.pool import StreamingSwitchMLP
from streamlx_b200.reader import ExpertReader
from streamlx_b200.stindex import SafetensorsIndex
from streamlx_b200.trace import PAD, TraceRecorder, read_trace, write_trace

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _gold():
    with open(os.path.join(GOLD, "residency.json")) as f:
        return json.load(f)


def test_plan_residency_matches_reference():
    for c in _gold()["plan_residency"]:
        bpe = {int(a): b for a, b in c["bpe"].items()}
        n_exp = {int(a): b for a, b in c["n_exp"].items()}
        res, left = plan_residency(c["layers"], bpe, n_exp, c["budget"],
                                   c["k"])
        assert sorted(res) == c["resident"], c
        assert left == c["left"], c


@pytest.fixture(scope="module")
def e256(tmp_path_factory):
    cfg = synth.SynthConfig(name="golden_e256", hidden=64, layers=3,
                            n_experts=256, top_k=10, inter=64, expert_bits=2,
                            zipf_s=1.1)
    return synth.write_model(str(tmp_path_factory.mktemp("e256r")), cfg,
                             seed=3)


def test_preload_popular_matches_reference(e256, tmp_path, monkeypatch):
    monkeypatch.setenv("STREAMLX_EVICT", "lru")
    g = _gold()
    ids = np.load(os.path.join(GOLD, "warm_trace.npz"))["experts"]
    lids = g["preload_layer_ids"]
    out, side = write_trace(str(tmp_path / "warm.npz"), ids,
                            np.zeros(ids.shape[0], np.uint32),
                            np.arange(ids.shape[0], dtype=np.uint32), lids,
                            n_experts=256,
                            bytes_per_expert={i: 1 for i in lids})
    index = SafetensorsIndex(e256)
    reader = ExpertReader(index, pinned=False)
    pools = {i: StreamingSwitchMLP(e256, i, g["preload_slots"], index=index,
                                   reader=reader, store="null")
             for i in range(3)}
    n = preload_popular(pools, str(out))
    want = g["preload_popular"]
    assert n == want["loaded"]
    for i, p in pools.items():
        w = want["pools"][str(i)]
        assert [[a, b] for a, b in p.id2slot.items()] == w["id2slot"], i
        assert p.free == w["free"]
        assert (p.misses, p.hits) == (w["misses"], w["hits"])
    reader.close()


class _Wrapper:
    def __init__(self):
        self.record_sink = None


class _Layer:
    def __init__(self):
        self.mlp = type("M", (), {})()
        self.mlp.switch_mlp = _Wrapper()


class _Pool:
    def __init__(self, index, lid):
        self.index = index
        self.n_experts = 256
        self.layer = lid


class _Model:
    def __init__(self, n):
        self.layers = [_Layer() for _ in range(n)]


def test_trace_recorder_format_roundtrip(e256, tmp_path):
    """Per-call records -> [tokens, layers, k] uint16 + sidecar; a decode
    call records [1, 1, k], a prefill call [1, T, k]; a layer that routed
    fewer ids is padded with 0xFFFF."""
    index = SafetensorsIndex(e256)
    model = _Model(3)
    pools = {0: _Pool(index, 0), 2: _Pool(index, 2)}
    rec = TraceRecorder(model, pools)
    rng = np.random.default_rng(0)
    seqs = []
    for s, T in enumerate((5, 3)):
        rows0 = rng.integers(0, 256, (T, 10))
        rows2 = rng.integers(0, 256, (T, 10))
        if s == 0:     # prefill-shaped call for the whole sequence
            model.layers[0].mlp.switch_mlp.record_sink.append(
                (0, rows0[None]))
            model.layers[2].mlp.switch_mlp.record_sink.append(
                (2, rows2[None]))
        else:          # decode calls, one token at a time
            for t in range(T):
                rec._sink.append((0, rows0[t][None, None]))
                rec._sink.append((2, rows2[t][None, None]))
        assert rec.end_sequence() == T
        seqs.append((rows0, rows2))
    out, side = rec.write(str(tmp_path / "trace"), model_name="golden_e256")
    arrays, meta = read_trace(str(out))
    e = arrays["experts"]
    assert e.dtype == np.uint16 and e.shape == (8, 2, 10)
    np.testing.assert_array_equal(e[:5, 0], seqs[0][0])
    np.testing.assert_array_equal(e[5:, 1], seqs[1][1])
    np.testing.assert_array_equal(arrays["seq_id"], [0] * 5 + [1] * 3)
    np.testing.assert_array_equal(arrays["pos"], [0, 1, 2, 3, 4, 0, 1, 2])
    assert arrays["prompt_class"].dtype == np.uint8
    assert meta["schema_version"] == 1 and meta["layer_ids"] == [0, 2]
    assert meta["k"] == 10 and meta["tokens"] == 8 and meta["sequences"] == 2
    assert meta["bytes_per_expert"]["2"] == index.layer_expert_bytes(2)
    rec.detach()
    assert model.layers[0].mlp.switch_mlp.record_sink is None

    # padding: a layer that routed k=4 ids in a k=10 trace
    ids = np.full((2, 1, 10), PAD, dtype=np.uint16)
    ids[:, 0, :4] = [[1, 2, 3, 4], [1, 2, 5, 6]]
    p2, _ = write_trace(str(tmp_path / "pad.npz"), ids, [0, 0], [0, 1], [1],
                        n_experts=256, bytes_per_expert={1: 7})
    ip = SafetensorsIndex(e256)
    pool = StreamingSwitchMLP(e256, 1, 3, index=ip,
                              reader=ExpertReader(ip, pinned=False),
                              store="null")
    assert preload_popular({1: pool}, str(p2)) == 3
    counts = np.bincount(ids[ids != PAD], minlength=256)
    assert sorted(pool.id2slot) == sorted(
        int(x) for x in np.argsort(counts)[::-1][:3])
    assert {1, 2} <= set(pool.id2slot)      # the two ids routed twice
    pool.reader.close()
