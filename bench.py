"""Benchmark: batch-1 greedy decode tok/s of the pool-backed MoE decoder on
B200, with the fused quantized SwitchGLU's HBM roofline.

Workload (N=1): the Qwen3-MoE-shaped synthetic decoder -- 40 layers, hidden
2048, GQA 16q/2kv x 128, vocab 151936, 256 routed experts top-8 + 1 shared
expert (intermediate 512), all 4-bit affine group 64, Zipf(1.0) router
bias -- written from a seed; expert pools get a 16 GiB budget (242 of 256
experts per layer in HBM, the rest streamed from the safetensors shards by
pread -> pinned -> HBM).  A 128-token random-id prompt is fed token by
token, then W warm-up and K timed decode steps (one step = one token).

Output: one JSON line (rank 0).  ``value`` is device-timed tokens/s (token
kept on the GPU between steps); ``e2e`` is the same loop through the public
step API with the token copied host->device and the sampled token read back
every step.  ``roofline`` times the SwitchGLU launch pairs of one layer in
eight inside the timed region with CUDA events recorded as graph nodes
(algorithmic bytes = routed experts + shared expert + activations per
launch) against the measured HBM copy peak.
``cpu_baseline`` times the CPU oracle decoder on a bounded sample.
``prefill`` (also ``--mode prefill`` on its own line) times the expert-major
prefill of one 117B-shaped MoE layer (2048 tokens x top-10 of 256 2-bit
experts) on the tensor cores, as TFLOP/s against the measured bf16 peak.
``host_ms_per_step`` splits the decode step's host time into the graph
launch, the previous step's deferred pool bookkeeping and the wait for the
device log.

``--impl reference`` times the reference's path restated on the CPU (the
oracle decoder; the reference's MLX backend is not installable here) on the
same checkpoint and metric.

Multi-GPU (torchrun): every rank decodes an independent replica (weak
scaling).  ``--mode ep`` (under torchrun) measures the expert-parallel MoE
layer instead: experts sharded 256/N per GPU, token rows exchanged by NCCL
all-to-all (batch-1 decode with the token replicated and one all-reduce;
batch-64 decode and a 2048-token prefill with tokens split over ranks);
``--check`` compares every rank's outputs with all experts run locally.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "laguna_c5"
SEED = 0
PROMPT_TOKENS = 128
SYNTH_ROOT = os.environ.get("STREAMLX_SYNTH_DIR",
                            os.path.join(tempfile.gettempdir(), "streamlx_synth"))
METRIC = "decode_tok_s"


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def synth_dir(preset: str, seed: int, local_rank: int, barrier) -> str:
    """Checkpoint shared by every run on this machine (written once)."""
    from streamlx_b200 import synth
    d = os.path.join(SYNTH_ROOT, f"{preset}_s{seed}")
    done = os.path.join(d, ".complete")
    if local_rank == 0 and not os.path.exists(done):
        import torch
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        t0 = time.time()
        synth.write_model(d, synth.PRESETS[preset], seed=seed, device=dev)
        open(done, "w").write(f"{time.time() - t0:.1f}s")
    barrier()
    return d


class Clocks:
    """nvidia-smi sampling while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.path = tempfile.mktemp(suffix=".csv")
        self.p = None

    def start(self):
        """Start sampling and return once the first sample is written (at
        most 5 s): nvidia-smi takes a while to start, longer than a short
        timed region."""
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:   # noqa: BLE001 - clocks are best effort
            self.p = None
            return
        t_end = time.time() + 5.0
        while (time.time() < t_end and self.p.poll() is None and
               os.path.getsize(self.path) == 0):
            time.sleep(0.01)

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.p.terminate()
        self.p.wait()
        self.f.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        for line in open(self.path):
            c = [x.strip() for x in line.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1]))
                mx.append(float(c[2]))
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak() -> tuple[float, str]:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:   # noqa: BLE001
        return 6650.0, "fallback"


def traffic_from_profile(model: str) -> float | None:
    """DRAM bytes per decode SwitchGLU launch from the committed ncu summary
    of that model's layer shape."""
    p = os.path.join(ROOT, "profiles", f"switchglu_decode_{model}.md")
    try:
        for line in open(p):
            if line.startswith(("traffic_bytes_per_launch:",
                                "traffic_bytes_per_launch_pair:")):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


SAMPLE_LAYERS = 4     # CPU timing sample: this many layers of each token


def _oracle_token_seconds(o, tok: int, n_layers: int) -> float:
    """Seconds of one decode token of the CPU oracle, measured on its first
    ``n_layers`` layers (+ final norm and head) and scaled to every layer;
    the head is timed once per call and not scaled."""
    t0 = time.perf_counter()
    o.step(tok, n_layers=n_layers)
    t_sample = time.perf_counter() - t0
    L = o.L
    if n_layers >= L:
        return t_sample
    t0 = time.perf_counter()
    o.step(tok, n_layers=0)                  # head only
    t_head = time.perf_counter() - t0
    return t_head + (t_sample - t_head) * L / n_layers


def cpu_oracle_rate(d: str, budget_s: float, max_steps: int | None = None
                    ) -> tuple[float, int, int]:
    """tok/s of the CPU oracle decoder (fp32 numpy BLAS) on a bounded
    sample: tokens run through their first SAMPLE_LAYERS layers, scaled to
    the whole model."""
    from oracle.model import OracleDecoder
    o = OracleDecoder(d, max_len=512, exact=False)
    rng = np.random.default_rng(SEED)
    n_lay = min(SAMPLE_LAYERS, o.L)
    o.step(int(rng.integers(o.cfg["vocab"])), n_layers=n_lay)   # warm-up
    secs, n, t0 = 0.0, 0, time.perf_counter()
    while True:
        secs += _oracle_token_seconds(o, int(rng.integers(o.cfg["vocab"])),
                                      n_lay)
        n += 1
        if time.perf_counter() - t0 > budget_s or \
                (max_steps and n >= max_steps):
            break
    cores = len(os.sched_getaffinity(0))
    return n / secs, n, cores


def run_reference(args) -> None:
    """The reference path restated on the CPU (the oracle decoder) on the
    workload's checkpoint: each step is one decode token measured on its
    first SAMPLE_LAYERS layers and scaled to the whole model."""
    rank, world, local = dist_env()
    if rank != 0:
        return
    preset = args.preset or WORKLOADS[args.workload][0]
    d = synth_dir(preset, SEED, 0, lambda: None)
    from oracle.model import OracleDecoder
    o = OracleDecoder(d, max_len=args.warmup + 2 * args.steps + 8,
                      exact=False)
    n_lay = min(SAMPLE_LAYERS, o.L)
    rng = np.random.default_rng(SEED)
    for _ in range(max(1, args.warmup)):
        o.step(int(rng.integers(o.cfg["vocab"])), n_layers=n_lay)
    budget_s = 240.0
    secs, n, t0 = 0.0, 0, time.perf_counter()
    while n < args.steps:
        secs += _oracle_token_seconds(o, int(rng.integers(o.cfg["vocab"])),
                                      n_lay)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    v = n / secs
    cores = len(os.sched_getaffinity(0))
    sample = (f"{n} of {args.steps} decode tokens of the {preset} decoder, "
              f"each timed on its first {n_lay} of {o.L} layers (+ head) and "
              f"scaled to all layers; fp32 numpy BLAS, experts dequantised "
              f"per use")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 5),
        "unit": "tok/s", "n_gpus": world, "steps": n, "warmup": args.warmup,
        "ms_per_step": round(1000 * secs / max(n, 1), 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "u2/u4-affine codes, fp32 accumulate",
        "data": "synthetic (seeded)",
        "config": {"workload": args.workload, "model": preset, "batch": 1},
        "cpu_baseline": {"value": round(v, 5), "unit": "tok/s",
                         "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 5), "unit": "tok/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


PREFILL_SHAPE = dict(hidden=2560, inter=1024, experts=256, top_k=10,
                     tokens=2048, zipf_s=1.1, layers=48)


def prefill_measure(dev, reps: int = 10, warmup: int = 3) -> dict:
    """Expert-major prefill of one 117B-shaped MoE layer on the tensor cores:
    2048 tokens x top-10 of 256 2-bit experts (Zipf 1.1 popularity via
    Gumbel-top-k on log p), every expert resident in an HBM slot pool
    (629 MB, larger than L2).  One step = one slx_prefill_grouped call
    (activation pack + gate/up/SwiGLU + down, three launches)."""
    import torch

    from streamlx_b200 import _lib as L
    from streamlx_b200 import ops, synth
    c = PREFILL_SHAPE
    H, I, E, k, T = c["hidden"], c["inter"], c["experts"], c["top_k"], c["tokens"]
    g = torch.Generator(device=dev).manual_seed(SEED)
    stride = L.slot_stride(H, I, 2)
    pool = torch.empty(E * stride, dtype=torch.uint8, device=dev)
    for e0 in range(0, E, 16):
        mats = []
        for (o, i) in ((I, H), (I, H), (H, I)):
            w = torch.randn(16, o, i, generator=g, device=dev) * 0.02
            mats.append(synth.quantize_affine(w, 2, 64))
            del w
        ex = [tuple((m[0][j], m[1][j], m[2][j]) for m in mats)
              for j in range(16)]
        L.pack_experts(ex, H, I, 2, [pool.data_ptr() + (e0 + j) * stride
                                     for j in range(16)])
    torch.cuda.synchronize()
    bank = L.bank_struct(pool, E, H, I, 2, stride)
    rng = np.random.default_rng(SEED)
    logp = synth.zipf_bias(E, c["zipf_s"], SEED)
    gum = rng.gumbel(size=(T, E)).astype(np.float32)
    ids = np.argsort(-(logp[None, :] + gum), axis=1)[:, :k]
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind="stable")
    slots, counts = np.unique(flat[order], return_counts=True)
    blocks = ops.prefill_blocks(slots, counts)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    pr = torch.as_tensor((order // k).astype(np.int32), device=dev)
    orow = torch.as_tensor(order.astype(np.int32), device=dev)
    bl = torch.as_tensor(blocks, device=dev)
    out = torch.empty(T * k, H, dtype=torch.bfloat16, device=dev)
    sc = torch.empty(L.prefill_scratch_bytes(blocks.shape[0], H, I, 2),
                     dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)

    def step():
        L.prefill_grouped(bank, x, pr, bl, out, sc, st, out_row=orow)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if int(st.item()) != 0:
        raise RuntimeError(f"prefill status {int(st.item())}")
    evs = [(torch.cuda.Event(enable_timing=True),
            torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in evs:
        a.record()
        step()
        b.record()
    torch.cuda.synchronize()
    ms = float(np.mean([a.elapsed_time(b) for a, b in evs]))
    flops = T * k * 6.0 * H * I
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, kind = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:   # noqa: BLE001
        peak, kind = 1590.0, "fallback"
    tf = flops / (ms / 1000.0) / 1e12
    return {"workload": "laguna_c4_layer", "tokens": T, "pairs": T * k,
            "blocks": int(blocks.shape[0]), "experts_routed": int(len(slots)),
            "ms_per_layer": round(ms, 4), "tflops": round(tf, 1),
            "peak_tflops": peak, "peak_kind": kind,
            "frac": round(tf / peak, 4), "bound": "tensor",
            "flops_per_layer": flops,
            "tokens_per_s_48_layers": round(T / (c["layers"] * ms / 1000.0), 1),
            "weights": "all 256 experts resident (629 MB); the sweep's disk "
                       "streaming is not in this number",
            "launches_per_layer": 3}


def run_prefill(args) -> None:
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    res = prefill_measure(torch.device("cuda", local), reps=args.steps,
                          warmup=args.warmup)
    if rank == 0:
        print(json.dumps({"metric": "prefill_tflops", "value": res["tflops"],
                          "unit": "TFLOP/s", "n_gpus": 1, **res}), flush=True)


def run_glu(args) -> None:
    """The decode SwitchGLU alone at the 117B shape: 256 2-bit experts
    (H 2560, I 1024) in a 630 MB slot pool, 48 launches of top-10 with
    different seeded routing per launch, back to back in a CUDA graph (PDL
    between them), timed with CUDA events around the graph; checked against
    the two-launch form on the same inputs first."""
    import torch

    from streamlx_b200 import _lib as L
    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    c = PREFILL_SHAPE
    H, I, E, k, n = c["hidden"], c["inter"], c["experts"], c["top_k"], 48
    pool, stride = _random_experts(E, H, I, dev, SEED)
    bank = L.bank_struct(pool, E, H, I, 2, stride)
    table = torch.arange(E, dtype=torch.int32, device=dev)
    rng = np.random.default_rng(SEED)
    ids = torch.as_tensor(np.stack([rng.choice(E, k, replace=False)
                                    for _ in range(n)]).astype(np.int32),
                          device=dev).reshape(n, 1, k)
    sc = rng.random((n, 1, k)).astype(np.float32)
    sc /= sc.sum(-1, keepdims=True)
    sc = torch.as_tensor(sc, device=dev)
    g = torch.Generator(device=dev).manual_seed(SEED)
    xs = (torch.randn(n, 1, H, generator=g, device=dev) * 0.5).to(torch.bfloat16)
    out = torch.empty(n, 1, H, dtype=torch.bfloat16, device=dev)
    ref = torch.empty_like(out)
    scr = torch.zeros(L.switchglu_scratch_bytes(1, k, I), dtype=torch.uint8,
                      device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)

    def launch_all(dst):
        for i in range(n):
            L.switchglu(bank, xs[i], ids[i], dst[i], scr, st, scores=sc[i],
                        slot_table=table)
    prev = L.set_switchglu_fused(False)
    launch_all(ref)
    L.set_switchglu_fused(True)
    launch_all(out)
    torch.cuda.synchronize()
    if int(st.item()) != 0:
        raise RuntimeError(f"switchglu status {int(st.item())}")
    a = out.float().cpu().numpy()
    b = ref.float().cpu().numpy()
    rel = float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
    L.set_pdl(True)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            launch_all(out)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=s):
            launch_all(out)
    torch.cuda.synchronize()
    ts = []
    e0, e1 = (torch.cuda.Event(enable_timing=True),
              torch.cuda.Event(enable_timing=True))
    for _ in range(args.warmup + args.steps):
        e0.record()
        gr.replay()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1000.0 / n)
    L.set_switchglu_fused(prev)
    us = float(np.median(ts[args.warmup:]))
    per_launch = k * synth_expert_bytes(H, I) + 2 * 2 * H
    peak, peak_kind = measured_peak()
    gbs = per_launch / (us * 1e-6) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "switchglu_decode_GBps", "value": round(gbs, 1),
            "unit": "GB/s", "n_gpus": 1, "launch_us": round(us, 2),
            "frac": round(gbs / peak, 4), "peak": peak,
            "peak_kind": peak_kind, "bytes_per_launch": int(per_launch),
            "launches_per_graph": n, "replays_timed": args.steps,
            "vs_two_launch_rel_l2": rel,
            "config": {"workload": "117B-shaped decode SwitchGLU: H 2560, "
                       "I 1024, 2-bit g64, top-10 of 256 slots (630 MB pool)",
                       "l2": "inputs larger than L2"}}), flush=True)


def run_sweep(args) -> None:
    """Expert-major prefill with streaming (the C4 workload): one
    2048-token chunk of seeded N(0,1) bf16 hidden states through every MoE
    layer of the 117B-shaped checkpoint (the same chunk into each layer),
    experts in 7.5 GiB pools, every needed expert read once per layer from
    the shards in expert-id order through the sweep (STREAMLX_PREFILL=sweep)
    and the hottest adopted.  Timed twice: with the shards' pages dropped
    from the page cache first (cold), then again (warm)."""
    import torch

    from streamlx_b200 import synth
    from streamlx_b200.integrate import aggregate_stats, load_streaming_model
    rank, world, local = dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    preset = args.preset or "laguna_c3"
    d = synth_dir(preset, SEED, local, lambda: None)
    cfg = synth.load_config(d)
    budget = args.budget_gib if args.budget_gib is not None else 7.5
    model, _, pools, reader = load_streaming_model(
        d, int(budget * (1 << 30)), k=cfg.top_k, device=dev)
    g = torch.Generator(device=dev).manual_seed(SEED)
    T = PREFILL_SHAPE["tokens"]
    x = torch.randn(T, cfg.hidden, generator=g, device=dev).to(torch.bfloat16)
    shards = [os.path.join(d, f) for f in sorted(os.listdir(d))
              if f.endswith(".safetensors")]
    runs = {}
    for label in ("cold", "warm"):
        if label == "cold":
            for f in shards:
                fd = os.open(f, os.O_RDONLY)
                try:
                    os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
                finally:
                    os.close(fd)
        for p in pools.values():
            p.reset_stats()
        r0 = (reader.bytes_read, reader.reads)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for layer in range(cfg.layers):
            model.moe_forward(layer, x)
        torch.cuda.synchronize()
        secs = time.perf_counter() - t0
        st = aggregate_stats(pools)
        runs[label] = {"seconds": round(secs, 3),
                       "tok_s": round(T / secs, 1),
                       "bytes_read": reader.bytes_read - r0[0],
                       "reads": reader.reads - r0[1],
                       "sweep_experts": st["sweep_experts"],
                       "sweep_fetch_s": round(st["sweep_fetch_s"], 3),
                       "adopted": st["adopted"]}
    reader.close()
    if rank == 0:
        print(json.dumps({
            "metric": "prefill_tok_s_streaming", "value": runs["cold"]["tok_s"],
            "unit": "tok/s", "n_gpus": 1, "higher_is_better": True,
            "cold": runs["cold"], "warm": runs["warm"],
            "config": {"workload": "2048-token chunk through every MoE layer "
                       "of the 117B-shaped checkpoint (the same seeded "
                       "hidden states into each layer)", "model": preset,
                       "layers": cfg.layers, "expert_budget_gib": budget,
                       "prefill": os.environ.get("STREAMLX_PREFILL", "sweep")},
            "data": "synthetic (seeded)"}), flush=True)


def synth_expert_bytes(H: int, I: int) -> int:
    from streamlx_b200 import synth
    return synth.expert_bytes(H, I, 2, 64)


def _random_experts(E, H, I, dev, seed, pool=None, ids=None):
    """Tile-format pool of E 2-bit experts with random codes and sane
    scales/biases (throughput runs: values only need to be finite).  With
    ``ids``, slot j holds expert ids[j] of the seeded set (same bytes on every
    rank)."""
    import torch

    from streamlx_b200 import _lib as L
    stride = L.slot_stride(H, I, 2)
    ids = list(range(E)) if ids is None else list(ids)
    if pool is None:
        pool = torch.empty(len(ids) * stride, dtype=torch.uint8, device=dev)
    for j0 in range(0, len(ids), 16):
        chunk = ids[j0:j0 + 16]
        ex = []
        keep = []
        for e in chunk:
            g = torch.Generator(device=dev).manual_seed(seed * 100003 + e)
            trip = []
            for (o, i) in ((I, H), (I, H), (H, I)):
                w = torch.randint(-2**31, 2**31 - 1, (o, i // 16), generator=g,
                                  device=dev, dtype=torch.int32)
                sc = (torch.rand(o, i // 64, generator=g, device=dev) * 0.01
                      + 0.005).to(torch.bfloat16)
                bi = (torch.rand(o, i // 64, generator=g, device=dev) * -0.02
                      - 0.01).to(torch.bfloat16)
                trip.append((w, sc, bi))
                keep.append((w, sc, bi))
            ex.append(tuple(trip))
        L.pack_experts(ex, H, I, 2, [pool.data_ptr() + (j0 + j) * stride
                                     for j in range(len(chunk))])
        torch.cuda.synchronize()
    return pool, stride


class _ResidentPool:
    """Slot pool view for expert_parallel.pool_expert_fn: expert ids
    [e0, e1) in slots 0.. (every expert resident)."""

    def __init__(self, bank, e0, e1, hidden, inter):
        self.id2slot = {e: e - e0 for e in range(e0, e1)}
        self.hidden, self.inter, self.bits = hidden, inter, 2

        class _S:
            pass
        self.store = _S()
        self.store.bank = bank


def run_ep(args) -> None:
    """Expert-parallel MoE layer (117B-shaped: hidden 2560, 256 2-bit
    experts top-10, inter 1024) over the torchrun ranks: experts 256/N per
    GPU, NCCL all-to-all of token rows.  Workloads: batch-1 decode (the
    token on every rank, one all-reduce), batch-64 decode and a 2048-token
    prefill (tokens split over the ranks, dispatch + combine all-to-all)."""
    import datetime

    import torch
    import torch.distributed as tdist

    from streamlx_b200 import _lib as L
    from streamlx_b200 import expert_parallel as EPM
    from streamlx_b200 import synth
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                             device_id=dev)
    H, I, E, k = 2560, 1024, 256, 10
    n_layers = 2           # distinct weights, alternated: > L2 per rank
    e0, e1 = EPM.local_range(E, world, rank)
    banks = []
    pools = []
    for li in range(n_layers):
        pool, stride = _random_experts(E, H, I, dev, seed=li,
                                       ids=range(e0, e1))
        pools.append(pool)
        banks.append(L.bank_struct(pool, e1 - e0, H, I, 2, stride))
    moes = [EPM.ExpertParallelMoE(
        E, EPM.pool_expert_fn(_ResidentPool(b, e0, e1, H, I)))
        for b in banks]
    logp = synth.zipf_bias(E, 1.1, SEED)

    def route(T, seed):
        r = np.random.default_rng(seed)
        g = r.gumbel(size=(T, E)).astype(np.float32)
        ids = np.argsort(-(logp[None, :] + g), axis=1)[:, :k]
        sc = r.random((T, k)).astype(np.float32)
        return ids, sc / sc.sum(1, keepdims=True)

    results = {}
    for name, T_glob, mode in (("decode_b1", 1, "replicated"),
                               ("decode_b64", 64, "sharded"),
                               ("prefill_2048", 2048, "sharded")):
        T = T_glob if mode == "replicated" else T_glob // world
        gx = torch.Generator(device=dev).manual_seed(SEED + (0 if mode == "replicated" else rank))
        x = torch.randn(T, H, generator=gx, device=dev).to(torch.bfloat16)
        seeds = [1000 * (0 if mode == "replicated" else rank) + s
                 for s in range(args.steps + args.warmup)]
        plans = [route(T, s) for s in seeds]
        for s in range(args.warmup):
            ids, sc = plans[s]
            moes[s % n_layers].forward(x, ids, sc, tokens=mode)
        torch.cuda.synchronize()
        tdist.barrier()
        e_a, e_b = (torch.cuda.Event(enable_timing=True),
                    torch.cuda.Event(enable_timing=True))
        b0 = sum(m.bytes_sent for m in moes)
        e_a.record()
        for s in range(args.warmup, args.warmup + args.steps):
            ids, sc = plans[s]
            moes[s % n_layers].forward(x, ids, sc, tokens=mode)
        e_b.record()
        torch.cuda.synchronize()
        t = torch.tensor([e_a.elapsed_time(e_b) / args.steps], device=dev)
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
        ms = float(t.item())
        moved = (sum(m.bytes_sent for m in moes) - b0) / args.steps
        uniq = len(np.unique(np.concatenate([p[0].reshape(-1) for p in plans[args.warmup:]])))
        results[name] = {"tokens": T_glob, "ms_per_layer": round(ms, 4),
                         "tok_s_48_layers": round(T_glob / (48 * ms / 1000.0), 2),
                         "comm_bytes_per_layer_rank0": int(moved),
                         "tokens_mode": mode}
        if args.check:
            # every rank recomputes its own tokens with all 256 experts
            from streamlx_b200 import ops
            full, fstride = _random_experts(E, H, I, dev, seed=(args.warmup) % n_layers)
            fbank = L.bank_struct(full, E, H, I, 2, fstride)
            ids, sc = plans[args.warmup]
            y_ep = moes[args.warmup % n_layers].forward(x, ids, sc, tokens=mode)
            flat = ids.reshape(-1)
            order = np.argsort(flat, kind="stable")
            sl, cn = np.unique(flat[order], return_counts=True)
            yp = ops.prefill_grouped(fbank, x, order // k, sl, cn,
                                     out_row=order, n_out=flat.size) \
                if flat.size >= 64 else ops.switchglu(
                    fbank, x[torch.as_tensor(np.arange(flat.size) // k, device=dev)].contiguous(),
                    torch.as_tensor(flat.astype(np.int32), device=dev).reshape(-1, 1), 1,
                    inter=I).reshape(flat.size, H)
            want = (yp.float().view(T, k, H) *
                    torch.as_tensor(sc, device=dev).reshape(T, k, 1)).sum(1)
            want = want.to(torch.bfloat16).float()   # rounded like the output
            d = (y_ep.float() - want).abs().max().item()
            rel = ((y_ep.float() - want).norm() / want.norm()).item()
            dd = torch.tensor([d, rel], device=dev)
            tdist.all_reduce(dd, op=tdist.ReduceOp.MAX)
            results[name]["check_max_abs"] = float(dd[0])
            results[name]["check_rel_l2"] = float(dd[1])
            del full
    tdist.barrier()
    tdist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"metric": "ep_moe_layer", "n_gpus": world,
                          "experts_per_gpu": e1 - e0, "steps": args.steps,
                          "warmup": args.warmup,
                          "config": {"workload": "laguna_c5_layer",
                                     "hidden": H, "inter": I, "experts": E,
                                     "top_k": k, "bits": 2,
                                     "parallelism": f"ep{world}"},
                          **results}), flush=True)
        if args.check:
            bad = [n for n, r in results.items()
                   if r["check_max_abs"] > 2e-2 or r["check_rel_l2"] > 1e-3]
            if bad:
                raise SystemExit(f"EP check failed: {bad}")


def switchglu_graph_us(model, pools, dev, reps: int = 6) -> float:
    """Average duration of one decode SwitchGLU launch (us): a CUDA graph of
    one launch per layer over the layers' own pools, with the routed ids and
    weights of the last decode step and seeded activations."""
    import torch
    from streamlx_b200 import _lib as L
    cfg = model.cfg
    n, k, H = cfg.layers, cfg.top_k, cfg.hidden
    g = torch.Generator(device="cpu").manual_seed(SEED)
    xs = (torch.randn(n, 1, H, generator=g) * 0.5).to(torch.bfloat16).to(dev)
    ids = model.g_ids.clone()
    scores = model.g_scores.clone()
    out = torch.empty(n, 1, H, dtype=torch.bfloat16, device=dev)
    scr = torch.zeros(L.switchglu_scratch_bytes(1, k, cfg.inter),
                      dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    prev_pdl = L.set_pdl(True)
    try:
        def launch_all():
            for i in range(n):
                p = pools[i]
                L.switchglu(p.store.bank, xs[i], ids[i], out[i], scr, st,
                            scores=scores[i], slot_table=p.store.table_dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            launch_all()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                launch_all()
        torch.cuda.synchronize()
        if int(st.item()) != 0:
            return None
        e0, e1 = (torch.cuda.Event(enable_timing=True),
                  torch.cuda.Event(enable_timing=True))
        ts = []
        for _ in range(reps):
            e0.record()
            gr.replay()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1000.0 / n)
        del gr
        return float(np.median(ts[1:]))
    finally:
        L.set_pdl(prev_pdl)


WORKLOADS = {
    # name: (preset, expert budget GiB or None = every expert resident and
    #        sharded over the ranks)
    "laguna_c5": ("laguna_c3", None),
    "laguna_c3": ("laguna_c3", 7.5),
    "qwen3moe_c2": ("qwen3moe_c2", 16.0),
}


def init_dist(world: int, local: int):
    """Process group of the run (one rank without torchrun), NCCL on GPUs."""
    import datetime

    import torch
    import torch.distributed as tdist
    if tdist.is_initialized():
        return tdist
    if world == 1 and "MASTER_ADDR" not in os.environ:
        import socket
        sk = socket.socket()
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
        sk.close()
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                          RANK="0", WORLD_SIZE="1", LOCAL_RANK="0")
    tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                             device_id=torch.device("cuda", local))
    return tdist


def run_ours(args) -> None:
    import torch

    from streamlx_b200 import _lib as L
    from streamlx_b200 import ops, synth
    from streamlx_b200.integrate import aggregate_stats, load_streaming_model

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tdist = init_dist(world, local)
    preset, budget_gib = WORKLOADS[args.workload]
    if args.budget_gib is not None:
        budget_gib = args.budget_gib
    if args.policy:
        os.environ["STREAMLX_EVICT"] = args.policy
    if args.prefetch is not None:
        os.environ["STREAMLX_PREFETCH"] = "1" if args.prefetch == "on" else "0"
    sharded = budget_gib is None
    if world > 1 and not sharded and not args.replicas:
        raise SystemExit(f"{args.workload} streams experts through per-GPU "
                         "pools; run it on one GPU or pass --replicas")

    def barrier():
        if world > 1:
            tdist.barrier()

    d = synth_dir(preset, SEED, local, barrier)
    cfg = synth.PRESETS[preset]
    t_load = time.time()
    if sharded:
        model, tok_, pools, reader = load_streaming_model(
            d, 0, k=cfg.top_k, device=dev, expert_parallel=True)
    else:
        model, tok_, pools, reader = load_streaming_model(
            d, int(budget_gib * (1 << 30)), k=cfg.top_k, device=dev)
    t_load = time.time() - t_load
    # no timing events inside the timed steps' graphs (the decoder's
    # default): an event node serialises its launch against the neighbours;
    # the bracketed in-step SwitchGLU times come from a separate loop after
    # the timed ones
    model.glu_events = False
    rng = np.random.default_rng(SEED)      # the same prompt on every rank
    prompt = rng.integers(0, cfg.vocab, args.prompt)
    total_steps = args.prompt + args.warmup + 2 * args.steps + 18
    if total_steps > model.max_len:
        raise SystemExit(f"steps too large for the KV cache ({model.max_len})")
    tok = None
    t_prompt = time.time()
    for pid in prompt:
        tok = model.step(torch.tensor([int(pid)], dtype=torch.int32,
                                      device=dev))
    for _ in range(args.warmup):
        tok = model.step(tok)
    torch.cuda.synchronize()
    t_prompt = time.time() - t_prompt

    def pool_counts():
        st = aggregate_stats(pools)
        return st["hits"], st["misses"], st["pf_used"]

    # ----------------------------------------------------- timed region --
    clocks = Clocks(local)
    for k_ in model.host_times:
        model.host_times[k_] = 0
    l0 = L.LAUNCHES[0]
    c0 = pool_counts()
    clocks.start()              # sampling before any rank starts timing
    barrier()
    torch.cuda.synchronize()
    e0, e1 = (torch.cuda.Event(enable_timing=True),
              torch.cuda.Event(enable_timing=True))
    e0.record()
    for _ in range(args.steps):
        tok = model.step(tok)
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = L.LAUNCHES[0] - l0
    c1 = pool_counts()
    ht = dict(model.host_times)
    host_ms = {k_: round(1000 * v / max(ht["steps"], 1), 3)
               for k_, v in ht.items()
               if k_ not in ("steps", "parks", "park_steps")}
    host_ms["parks"] = ht["parks"]
    host_ms["steps_with_a_park"] = ht["park_steps"]
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    ms_max = float(t.item())
    # batch-1 decode: every rank steps the same token (sharded experts) or
    # its own replica (--replicas)
    n_seq = world if (args.replicas and not sharded) else 1
    value = n_seq * args.steps / (ms_max / 1000.0)

    # ------------------------------------ end to end (host token in/out) --
    # the same number of steps right after, on the pools the timed loop
    # left (each loop's pool traffic is reported)
    tok_host = int(tok.item())
    barrier()
    torch.cuda.synchronize()
    f0, f1 = (torch.cuda.Event(enable_timing=True),
              torch.cuda.Event(enable_timing=True))
    t_in = torch.zeros(1, dtype=torch.int32).pin_memory()
    f0.record()
    for _ in range(args.steps):
        t_in[0] = tok_host      # the last step's copy from it has finished
        out = model.step(t_in)  # host token: copied with the step's controls
        tok_host = int(out.item())
    f1.record()
    torch.cuda.synchronize()
    c2 = pool_counts()
    t2 = torch.tensor([f0.elapsed_time(f1)], device=dev)
    if world > 1:
        tdist.all_reduce(t2, op=tdist.ReduceOp.MAX)
    e2e_value = n_seq * args.steps / (float(t2.item()) / 1000.0)

    # SwitchGLU launches bracketed by event pairs inside the step graph
    # (layers 3, 11, 19, ...), a few steps after the timed loops
    model.glu_events = True
    model._graphs = None
    model.glu_times = []
    for _ in range(min(args.steps, 16)):
        tok = model.step(tok)
    torch.cuda.synchronize()
    glu_ms, model.glu_times = model.glu_times, None

    # --------------------------------------------------------- roofline --
    # one SwitchGLU launch per layer, back to back in a graph of its own (the
    # layers' own pools and the last step's routing; no event between the
    # launches), timed with CUDA events around the graph: the kernel's
    # average launch duration in the decode's own launch pattern
    glu_graph_us = None
    if world == 1:      # (at N = 1 every expert is in this GPU's pools)
        glu_graph_us = switchglu_graph_us(model, pools, dev)
    H = cfg.hidden
    bpe = synth.expert_bytes(H, cfg.inter, cfg.expert_bits, 64)
    sh_b = synth.expert_bytes(H, cfg.shared_inter, cfg.trunk_bits, 64) \
        if cfg.shared_inter else 0
    # routed experts this rank computes per launch (all of them at N = 1)
    units = cfg.top_k / (world if sharded else 1)
    per_launch = units * bpe + sh_b + 2 * 2 * H
    mean_ms = float(np.mean(glu_ms)) if glu_ms else float("nan")
    launch_ms = glu_graph_us / 1000.0 if glu_graph_us else mean_ms
    achieved = per_launch / (launch_ms / 1000.0) / 1e9
    peak, peak_kind = measured_peak()
    traffic = traffic_from_profile(cfg.name)

    pre = None
    if not args.no_prefill and rank == 0 and world == 1:
        pre = prefill_measure(dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, cores = cpu_oracle_rate(d, budget_s=args.cpu_seconds)
        cpu = {"value": round(rate, 4), "unit": "tok/s", "cores": cores,
               "kind": "port",
               "sample": f"{n} decode tokens of the same {preset} checkpoint "
                         f"on the CPU oracle decoder (fp32 numpy BLAS)"}

    if sharded and model.ep is not None:
        model.ep.close()
    barrier()
    if world > 1 or tdist.is_initialized():
        model._graphs = None
        tdist.destroy_process_group()
    if rank != 0:
        return
    hits0 = (c1[0] - c0[0], c1[1] - c0[1])
    hits1 = (c2[0] - c1[0], c2[1] - c1[1])
    res = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong" if sharded else "weak", "vs_baseline": None,
        "dtype": f"u{cfg.expert_bits}-affine codes x bf16, fp32 accumulate",
        "data": "synthetic (seeded random-init weights and prompt)",
        "config": {"workload": args.workload, "model": preset,
                   "layers": cfg.layers, "hidden": cfg.hidden,
                   "experts": cfg.n_experts, "top_k": cfg.top_k,
                   "expert_bits": cfg.expert_bits,
                   "shared_expert": bool(cfg.shared_inter),
                   "experts_in_hbm": (
                       "all, sharded over the GPUs" if sharded and world > 1
                       else "all" if sharded else f"{budget_gib} GiB pools"),
                   "slots_per_layer": pools[0].n_slots,
                   "evict": os.environ.get("STREAMLX_EVICT", "lru"),
                   "prefetch": os.environ.get("STREAMLX_PREFETCH", "1") != "0",
                   "prompt_tokens": args.prompt, "batch": 1,
                   "l2": "inputs larger than L2: ~1 GB of weights per step",
                   "parallelism": (
                       f"expert parallel x{world}" if sharded and world > 1
                       else "one GPU, every expert local" if sharded
                       else f"replicas x{world}")},
        "e2e": {"value": round(e2e_value, 3), "unit": "tok/s",
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
        "roofline": {"kernel": "decode SwitchGLU (k_switchglu_fused, one "
                               "cooperative launch per layer)",
                     "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": traffic,
                     "algorithmic_bytes_per_launch": int(per_launch),
                     "launch_us": round(1000 * launch_ms, 2),
                     "timing": ("graph of one launch per layer, back to back"
                                if glu_graph_us else
                                "event pairs around layers 3, 11, 19, ... "
                                "inside the decode graph"),
                     "in_step_bracketed_us": round(1000 * mean_ms, 2),
                     "in_step_launches_timed": len(glu_ms)},
        "gpu_launches": launches,
        "host_ms_per_step": host_ms,
        "clocks": clk,
        "pool": {"timed_loop": {"hits": hits0[0], "misses": hits0[1]},
                 "e2e_loop": {"hits": hits1[0], "misses": hits1[1]},
                 "prefetch_used_timed": c1[2] - c0[2]},
        "setup_s": {"load": round(t_load, 1), "prompt_and_warmup":
                    round(t_prompt, 1)},
    }
    if pre:
        res["prefill"] = pre
    if cpu:
        res["cpu_baseline"] = cpu
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default=WORKLOAD, choices=sorted(WORKLOADS),
                    help="laguna_c5: the 117B-shaped decoder, every expert "
                         "resident and sharded over the GPUs (default); "
                         "laguna_c3: the same model streaming from 7.5 GiB "
                         "pools; qwen3moe_c2: the Qwen3-MoE-shaped decoder "
                         "with 16 GiB pools")
    ap.add_argument("--preset", default=None,
                    help="checkpoint preset of the reference arm (default: "
                         "the workload's)")
    ap.add_argument("--prompt", type=int, default=PROMPT_TOKENS)
    ap.add_argument("--budget-gib", type=float, default=None,
                    help="override the workload's expert budget")
    ap.add_argument("--policy", choices=["lru", "s3fifo"], default=None)
    ap.add_argument("--prefetch", choices=["on", "off"], default=None)
    ap.add_argument("--replicas", action="store_true",
                    help="pool workloads on N GPUs: N independent replicas")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the expert-major prefill measurement")
    ap.add_argument("--check", action="store_true",
                    help="ep mode: compare with an all-experts computation")
    ap.add_argument("--mode", default="decode",
                    choices=["decode", "prefill", "ep", "glu", "sweep"],
                    help="prefill: only the prefill measurement (its own "
                         "line); glu: only the decode SwitchGLU kernel; "
                         "sweep: 2048-token prefill through every MoE layer "
                         "with expert streaming (cold and warm page cache)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "prefill":
        run_prefill(args)
    elif args.mode == "ep":
        run_ep(args)
    elif args.mode == "glu":
        run_glu(args)
    elif args.mode == "sweep":
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
