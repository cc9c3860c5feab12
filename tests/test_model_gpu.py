"""End-to-end GPU parity: pool-backed decoder vs the CPU oracle decoder, the
pool's drop-in SwitchGLU call, and the expert-major prefill sweep vs the
reference-composed outputs in tests/golden."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import affine as A
from oracle.model import OracleDecoder
from streamlx_b200 import synth
from streamlx_b200.integrate import (StreamingSwitchGLU, aggregate_stats,
                                     load_streaming_model)
from streamlx_b200.pool import StreamingSwitchMLP
from streamlx_b200.reader import ExpertReader
from streamlx_b200.stindex import SafetensorsIndex

from .kernel_cases import bf16_np, bf16_tensor, check_close

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    root = tmp_path_factory.mktemp("models")
    return {name: synth.write_model(str(root / name), synth.PRESETS[name],
                                    seed=5)
            for name in ("tiny_dec", "tiny_dec2")}


# Logit tolerances of the free-running decoder against the fp64 oracle:
# max-abs 2e-2, and rel-L2 1e-3 or, where the bf16 pipeline itself cannot
# get that close, F32_FACTOR times the distance an fp32-accumulating
# restatement of the same pipeline (oracle exact=False, forced onto the same
# routing) has from the fp64 one.  Both round at the same points; a value
# whose exact result sits near a bf16 rounding boundary rounds either way
# under fp32 accumulation, one flipped SwiGLU activation moves ~10% of the
# down projection's bf16 outputs by an ulp, and later roundings compound
# it.  On these decoders the fp32 restatement reaches 2.8-2.9e-3 over 24
# steps (max-abs one logit ulp, 7.8e-3), the GPU 2.5-3.4e-3.
LOGIT_MAX_ABS = 2e-2
LOGIT_REL = 1e-3
F32_FACTOR = 1.5


@pytest.mark.parametrize("path", ["graph", "eager"])
@pytest.mark.parametrize("name,slots", [("tiny_dec", 6), ("tiny_dec2", 5)])
def test_decoder_matches_oracle(tiny, name, slots, path, monkeypatch):
    monkeypatch.setenv("STREAMLX_EVICT", "lru")
    d = tiny[name]
    cfg = synth.load_config(d)
    bpe = synth.expert_bytes(cfg.hidden, cfg.inter, cfg.expert_bits, 64)
    model, tok, pools, reader = load_streaming_model(
        d, budget_bytes=slots * bpe * cfg.layers, k=cfg.top_k)
    model.use_graphs = path == "graph"
    model.pipeline = False          # routed ids recorded within each step
    assert all(p.n_slots == slots for p in pools.values())
    sinks = []
    for i in range(cfg.layers):
        s = []
        model.layers[i].mlp.switch_mlp.record_sink = s
        sinks.append(s)
    oracle = OracleDecoder(d)
    fp32 = OracleDecoder(d, exact=False)
    rng = np.random.default_rng(0)
    seq = rng.integers(0, cfg.vocab, 24)
    worst_rel = worst_rel32 = 0.0
    prev = {}
    for t, tk in enumerate(seq):
        model.step(torch.tensor([int(tk)], dtype=torch.int32,
                                device=model.device))
        got_logits = bf16_np(model.logits)[0]
        ids_gpu = [sinks[i][-1][1].reshape(-1) for i in range(cfg.layers)]
        # the same temporal-reuse decisions as the GPU run
        forced = {i: prev[i] for i in range(cfg.layers)
                  if t > 0 and cfg.repeat_p and np.array_equal(ids_gpu[i],
                                                                prev.get(i))}
        want_logits, ids_cpu = oracle.step(int(tk), forced=forced)
        for i in range(cfg.layers):
            # the same experts in the same order, every layer and step
            assert np.array_equal(ids_gpu[i], ids_cpu[i]), (t, i, ids_gpu[i],
                                                            ids_cpu[i])
        prev = {i: ids_gpu[i] for i in range(cfg.layers)}
        lf, _ = fp32.step(int(tk), forced=dict(enumerate(ids_cpu)))
        want = A.bf16_round(want_logits)
        worst_rel = max(worst_rel, A.rel_l2(got_logits, want))
        worst_rel32 = max(worst_rel32, A.rel_l2(A.bf16_round(lf), want))
        assert np.max(np.abs(got_logits - want)) <= LOGIT_MAX_ABS, t
    assert worst_rel <= max(LOGIT_REL, F32_FACTOR * worst_rel32), \
        (worst_rel, worst_rel32)
    st = aggregate_stats(pools)
    assert st["misses"] > 0 and st["evictions"] > 0      # the pool streamed
    assert st["hits"] + st["misses"] == 24 * cfg.layers * cfg.top_k
    reader.close()


def _pool_state(p):
    return (p.stats, list(p.id2slot.items()), list(p.free),
            {str(k): v for k, v in p.pf_rank.items()})


@pytest.mark.parametrize("policy", ["lru", "s3fifo"])
@pytest.mark.parametrize("name,slots", [("tiny_dec", 6), ("tiny_dec2", 5)])
def test_graph_step_trace_equals_eager(tiny, name, slots, policy, monkeypatch):
    """The graph step (pipelined, with reruns after misses) gives the eager
    step's tokens, logits and pool bookkeeping, call for call."""
    monkeypatch.setenv("STREAMLX_EVICT", policy)
    d = tiny[name]
    cfg = synth.load_config(d)
    bpe = synth.expert_bytes(cfg.hidden, cfg.inter, cfg.expert_bits, 64)
    runs = []
    for path in ("eager", "graph"):
        model, _, pools, reader = load_streaming_model(
            d, budget_bytes=slots * bpe * cfg.layers, k=cfg.top_k)
        model.use_graphs = path == "graph"
        sinks = []
        for i in range(cfg.layers):
            sinks.append([])
            model.layers[i].mlp.switch_mlp.record_sink = sinks[-1]
        rng = np.random.default_rng(7)
        toks, logits = [], []
        tok = None
        for t in range(40):
            if t < 8 or tok is None:    # prompt, then greedy decode
                tok = torch.tensor([int(rng.integers(cfg.vocab))],
                                   dtype=torch.int32, device=model.device)
            tok = model.step(tok)
            toks.append(int(tok.item()))
            logits.append(model.logits.clone())
        model.flush()
        if path == "graph":
            # the pools are smaller than the routed sets: layers parked on a
            # miss and were filled by their own kernel
            assert model.host_times["parks"] > 0
            assert model.svc.stats["experts"] > 0
        state = [_pool_state(pools[i]) for i in sorted(pools)]
        seq = [[x[1].tolist() for x in s] for s in sinks]
        runs.append((toks, torch.cat(logits), state, seq))
        reader.close()
    (t0, l0, s0, q0), (t1, l1, s1, q1) = runs
    assert t0 == t1
    assert torch.equal(l0, l1)
    assert q0 == q1
    for a, b in zip(s0, s1):
        sa = {k: v for k, v in a[0].items() if not k.endswith("_s")}
        sb = {k: v for k, v in b[0].items() if not k.endswith("_s")}
        assert sa == sb and a[1:] == b[1:]
    assert sum(x[0]["misses"] for x in s1) > 0


def test_vlm_export_decodes_like_native(tiny, tmp_path, monkeypatch):
    """A checkpoint rewritten as an mlx-vlm export (prefixed keys, router
    matrix under ``.mlp.gate.proj.``) loads through load_streaming_model and
    decodes to the same logits bit for bit as the native export."""
    from .vlm_copy import write_vlm_copy
    monkeypatch.setenv("STREAMLX_EVICT", "lru")
    d = tiny["tiny_dec"]
    v = write_vlm_copy(d, str(tmp_path / "vlm"))
    cfg = synth.load_config(d)
    bpe = synth.expert_bytes(cfg.hidden, cfg.inter, cfg.expert_bits, 64)
    seq = np.random.default_rng(4).integers(0, cfg.vocab, 10)
    out = []
    for path in (d, v):
        model, _, pools, reader = load_streaming_model(
            path, budget_bytes=6 * bpe * cfg.layers, k=cfg.top_k)
        lg = []
        for tk in seq:
            model.step(torch.tensor([int(tk)], dtype=torch.int32,
                                    device=model.device))
            lg.append(model.logits.clone())
        torch.cuda.synchronize()
        out.append((torch.cat(lg).cpu(), aggregate_stats(pools)["misses"]))
        reader.close()
    assert torch.equal(out[0][0].view(torch.int16), out[1][0].view(torch.int16))
    assert out[0][1] == out[1][1] > 0


def test_resident_layers_skip_the_pool(tiny, monkeypatch):
    """Fully resident layers (plan_residency) run without slot service or
    host bookkeeping and stay out of the returned pools, as the reference's
    stock-path layers do (streamlx/integrate.py:425-437); the logits equal
    the streamed run's bit for bit, also with one layer put back on the
    serviced path between two static ones."""
    monkeypatch.setenv("STREAMLX_EVICT", "lru")
    d = tiny["tiny_dec"]
    cfg = synth.load_config(d)
    bpe = synth.expert_bytes(cfg.hidden, cfg.inter, cfg.expert_bits, 64)
    seq = np.random.default_rng(6).integers(0, cfg.vocab, 8)

    def run(budget, resident=None, serviced_layer=None):
        model, _, pools, reader = load_streaming_model(
            d, budget_bytes=budget, k=cfg.top_k, resident=resident)
        if serviced_layer is not None:
            model.static_glu[serviced_layer] = False
        lg = []
        for tk in seq:
            model.step(torch.tensor([int(tk)], dtype=torch.int32,
                                    device=model.device))
            lg.append(model.logits.clone())
        torch.cuda.synchronize()
        st = (list(model.static_glu), sorted(pools),
              aggregate_stats(pools)["misses"])
        reader.close()
        return torch.cat(lg).cpu().view(torch.int16), st

    a, sa = run(6 * bpe * cfg.layers)
    b, sb = run(10 ** 13, resident="on")
    c, sc = run(10 ** 13, resident="on", serviced_layer=1)
    assert sa == ([False] * cfg.layers, list(range(cfg.layers)), sa[2])
    assert sa[2] > 0
    assert sb == ([True] * cfg.layers, [], 0)
    assert sc[0] == [True, False] + [True] * (cfg.layers - 2)
    assert torch.equal(a, b) and torch.equal(a, c)


@pytest.mark.parametrize("resident", [True, False])
def test_host_token_equals_device_token(tiny, resident, monkeypatch):
    """step() with the token in pinned host memory (copied with the step's
    control words) decodes exactly as with a device token."""
    monkeypatch.setenv("STREAMLX_EVICT", "lru")
    d = tiny["tiny_dec"]
    cfg = synth.load_config(d)
    bpe = synth.expert_bytes(cfg.hidden, cfg.inter, cfg.expert_bits, 64)
    seq = np.random.default_rng(8).integers(0, cfg.vocab, 8)
    out = []
    for host in (False, True):
        if resident:
            model, _, _, reader = load_streaming_model(
                d, 10 ** 13, k=cfg.top_k, resident="on")
        else:
            model, _, _, reader = load_streaming_model(
                d, 6 * bpe * cfg.layers, k=cfg.top_k)
        lg = []
        for t in seq:
            tk = torch.tensor([int(t)], dtype=torch.int32)
            model.step(tk.pin_memory() if host else tk.to(model.device))
            lg.append(model.logits.clone())
        model.sync()
        out.append(torch.cat(lg).cpu().view(torch.int16))
        reader.close()
    assert torch.equal(out[0], out[1])


@pytest.mark.parametrize("resident", [True, False])
def test_step_device_error_is_raised(tiny, resident, monkeypatch):
    """A token id outside the vocabulary (the embedding kernel's bounds check
    sets SLX_ERR_OUT_OF_RANGE; nothing faults) is raised as SlxError: with
    every layer static the steps overlap, so the error surfaces at the next
    step or at sync(); with pools at the step itself.  The decoder keeps
    working afterwards."""
    from streamlx_b200 import _lib as L
    monkeypatch.setenv("STREAMLX_EVICT", "lru")
    d = tiny["tiny_dec"]
    cfg = synth.load_config(d)
    bpe = synth.expert_bytes(cfg.hidden, cfg.inter, cfg.expert_bits, 64)
    if resident:
        model, _, pools, reader = load_streaming_model(
            d, 10 ** 13, k=cfg.top_k, resident="on")
        assert model._overlapped()
    else:
        model, _, pools, reader = load_streaming_model(
            d, 6 * bpe * cfg.layers, k=cfg.top_k)
        assert not model._overlapped()

    def tok(t):
        return torch.tensor([t], dtype=torch.int32, device=model.device)

    for t in (3, 9):
        model.step(tok(t))
    with pytest.raises(L.SlxError):
        model.step(tok(cfg.vocab + 5))
        model.sync()
    for t in (4, 8):
        model.step(tok(t))
    model.sync()
    if resident:        # raised by the next step, and only once
        model.step(tok(cfg.vocab + 7))
        with pytest.raises(L.SlxError):
            model.step(tok(5))
        for t in (6, 2):
            model.step(tok(t))
        model.sync()
    assert int(model.g_status.item()) == 0
    reader.close()


def test_pool_dropin_call_matches_oracle(tiny):
    d = tiny["tiny_dec"]
    cfg = synth.load_config(d)
    pool = StreamingSwitchMLP(d, 1, 6)
    oracle = OracleDecoder(d)
    rng = np.random.default_rng(3)
    for step in range(6):
        ids = [int(e) for e in rng.choice(cfg.n_experts, cfg.top_k,
                                          replace=False)]
        x = A.bf16_round(rng.standard_normal((1, cfg.hidden))
                         .astype(np.float32))
        y = pool(bf16_tensor(x)[None], ids)             # [1,1,k,H]
        torch.cuda.synchronize()
        want = np.stack([A.expert_forward(x, oracle.expert(1, e))[0]
                         for e in ids])
        check_close(bf16_np(y)[0, 0], want)
    assert pool.misses > 0
    pool.reader.close()


@pytest.mark.parametrize("tag", ["sweep_lru_warm1", "sweep_lru_warm0",
                                 "slice_lru_warm1"])
def test_prefill_outputs_match_reference_composition(tmp_path, tag,
                                                     monkeypatch):
    """The reference's own _expert_sweep / slice path, run under the numpy
    mlx stand-in, produced y_small / y_big (tests/golden); the GPU sweep
    must give the same per-expert outputs."""
    g = np.load(os.path.join(GOLD, "trace_prefill.npz"))
    mode, pol, warm = tag.split("_")
    monkeypatch.setenv("STREAMLX_EVICT", pol)
    monkeypatch.setenv("STREAMLX_PREFILL", mode)
    monkeypatch.setenv("STREAMLX_SWEEP_BATCH", "16")
    monkeypatch.setenv("STREAMLX_SWEEP_WARM", warm[-1])
    cfg = synth.SynthConfig(name="golden_e256", hidden=64, layers=3,
                            n_experts=256, top_k=10, inter=64, expert_bits=2,
                            zipf_s=1.1)
    d = synth.write_model(str(tmp_path / "e256"), cfg, seed=3)
    index = SafetensorsIndex(d)
    pool = StreamingSwitchMLP(d, 1, 24, index=index,
                              reader=ExpertReader(index))
    w = StreamingSwitchGLU(pool)
    xs = A.bf16_from_bits(g["xs"])
    small = w(bf16_tensor(xs[:3])[None],
              torch.as_tensor(g["small_ids"][None].astype(np.int32)).cuda())
    big = w(bf16_tensor(xs)[None],
            torch.as_tensor(g["pre_ids"][None].astype(np.int32)).cuda())
    torch.cuda.synchronize()
    check_close(bf16_np(small), g[f"{tag}__y_small"])
    check_close(bf16_np(big), g[f"{tag}__y_big"])
    assert pool.sweep_experts > 0 if mode == "sweep" else True
    pool.reader.close()
