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

``--impl reference`` times the reference's path restated on the CPU (the
oracle decoder; the reference's MLX backend is not installable here) on the
same checkpoint and metric.

Multi-GPU (torchrun): every rank decodes an independent replica (weak
scaling; expert-parallel serving is a separate mode).
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

PRESET = "qwen3moe_c2"
SEED = 0
PROMPT_TOKENS = 128
BUDGET = 16 << 30
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
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:   # noqa: BLE001 - clocks are best effort
            self.p = None

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


def traffic_from_profile() -> float | None:
    """DRAM bytes per SwitchGLU launch pair from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "switchglu_decode_qwen3moe_c2.md")
    try:
        for line in open(p):
            if line.startswith("traffic_bytes_per_launch_pair:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def cpu_oracle_rate(d: str, budget_s: float, max_steps: int | None = None
                    ) -> tuple[float, int, int]:
    """tok/s of the CPU oracle decoder (fp32 BLAS) on a bounded sample."""
    from oracle.model import OracleDecoder
    o = OracleDecoder(d, max_len=64, exact=False)
    rng = np.random.default_rng(SEED)
    tok = int(rng.integers(o.cfg["vocab"]))
    logits, _ = o.step(tok)            # untimed warm-up (weight dequant)
    tok = int(np.argmax(logits))
    n, t0 = 0, time.perf_counter()
    while True:
        logits, _ = o.step(tok)
        tok = int(np.argmax(logits))
        n += 1
        el = time.perf_counter() - t0
        if el > budget_s or (max_steps and n >= max_steps):
            break
    cores = len(os.sched_getaffinity(0))
    return n / el, n, cores


def run_reference(args) -> None:
    rank, world, local = dist_env()
    if rank != 0:
        return
    d = synth_dir(args.preset, SEED, 0, lambda: None)
    from oracle.model import OracleDecoder
    o = OracleDecoder(d, max_len=args.warmup + args.steps + 8, exact=False)
    rng = np.random.default_rng(SEED)
    tok = int(rng.integers(o.cfg["vocab"]))
    for _ in range(max(1, args.warmup)):
        logits, _ = o.step(tok)
        tok = int(np.argmax(logits))
    budget_s = 180.0
    n, t0 = 0, time.perf_counter()
    while n < args.steps:
        logits, _ = o.step(tok)
        tok = int(np.argmax(logits))
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    el = time.perf_counter() - t0
    v = n / el
    cores = len(os.sched_getaffinity(0))
    sample = (f"{n} of {args.steps} decode tokens of the {args.preset} decoder "
              f"(fp32 numpy, all experts dequantised per use), short context")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(v, 4),
        "unit": "tok/s", "n_gpus": world, "steps": n, "warmup": args.warmup,
        "ms_per_step": round(1000 * el / max(n, 1), 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u2/u4-affine codes, fp32 accumulate",
        "data": "synthetic (seeded)",
        "config": {"workload": args.preset, "batch": 1},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s",
                         "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": round(v, 4), "unit": "tok/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def run_ours(args) -> None:
    import torch
    import torch.distributed as tdist

    from streamlx_b200 import _lib as L
    from streamlx_b200 import ops, synth
    from streamlx_b200.integrate import aggregate_stats, load_streaming_model

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))

    def barrier():
        if world > 1:
            tdist.barrier()

    d = synth_dir(args.preset, SEED, local, barrier)
    cfg = synth.PRESETS[args.preset]
    budget = int(args.budget_gib * (1 << 30))
    t_load = time.time()
    model, tok_, pools, reader = load_streaming_model(d, budget,
                                                      k=cfg.top_k, device=dev)
    t_load = time.time() - t_load
    rng = np.random.default_rng(SEED + rank)
    prompt = rng.integers(0, cfg.vocab, args.prompt)
    total_steps = args.prompt + args.warmup + 2 * args.steps + 2
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
    for p in pools.values():
        p.reset_stats()
    reader.reset_stats()

    # ----------------------------------------------------- timed region --
    clocks = Clocks(local)
    ops.TIMING = []                 # eager-path launches (none expected)
    model.glu_times = []            # graph-path launches: per-layer events
    l0 = L.LAUNCHES[0]
    model.flush()
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    e0, e1 = (torch.cuda.Event(enable_timing=True),
              torch.cuda.Event(enable_timing=True))
    e0.record()
    for _ in range(args.steps):
        tok = model.step(tok)
    model.flush()                   # the last step's deferred bookkeeping
    e1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = L.LAUNCHES[0] - l0
    timing, ops.TIMING = ops.TIMING, None
    glu_ms, model.glu_times = model.glu_times, None
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        tdist.all_reduce(t, op=tdist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * args.steps / (ms_max / 1000.0)
    st = aggregate_stats(pools)

    # ------------------------------------ end to end (host token in/out) --
    tok_host = int(tok.item())
    barrier()
    torch.cuda.synchronize()
    f0, f1 = (torch.cuda.Event(enable_timing=True),
              torch.cuda.Event(enable_timing=True))
    f0.record()
    for _ in range(args.steps):
        t_in = torch.tensor([tok_host], dtype=torch.int32).pin_memory()
        out = model.step(t_in.to(dev, non_blocking=True))
        tok_host = int(out.item())
    model.flush()
    f1.record()
    torch.cuda.synchronize()
    t2 = torch.tensor([f0.elapsed_time(f1)], device=dev)
    if world > 1:
        tdist.all_reduce(t2, op=tdist.ReduceOp.MAX)
    e2e_value = world * args.steps / (float(t2.item()) / 1000.0)

    # --------------------------------------------------------- roofline --
    durs = [a.elapsed_time(b) for a, b, *_ in timing] + list(glu_ms)
    H = cfg.hidden
    bpe = synth.expert_bytes(H, cfg.inter, cfg.expert_bits, 64)
    sh_b = synth.expert_bytes(H, cfg.shared_inter, cfg.trunk_bits, 64) \
        if cfg.shared_inter else 0
    per_launch = cfg.top_k * bpe + sh_b + 2 * 2 * H
    mean_ms = float(np.mean(durs)) if durs else float("nan")
    achieved = per_launch / (mean_ms / 1000.0) / 1e9
    peak, peak_kind = measured_peak()
    traffic = traffic_from_profile()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, cores = cpu_oracle_rate(d, budget_s=args.cpu_seconds)
        cpu = {"value": round(rate, 4), "unit": "tok/s", "cores": cores,
               "kind": "port",
               "sample": f"{n} decode tokens of the same {args.preset} checkpoint "
                         f"on the CPU oracle decoder (fp32 numpy BLAS)"}

    if world > 1:
        tdist.barrier()
        tdist.destroy_process_group()
    if rank != 0:
        return
    res = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_max / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "u4-affine codes x bf16, fp32 accumulate",
        "data": "synthetic (seeded random-init weights and prompt)",
        "config": {"workload": args.preset, "layers": cfg.layers,
                   "hidden": cfg.hidden, "experts": cfg.n_experts,
                   "top_k": cfg.top_k, "shared_expert": True,
                   "expert_budget_gib": args.budget_gib,
                   "slots_per_layer": pools[0].n_slots,
                   "prompt_tokens": args.prompt, "batch": 1,
                   "l2": "inputs larger than L2: ~0.9 GB of weights per step",
                   "parallelism": f"replicas x{world}"},
        "e2e": {"value": round(e2e_value, 3), "unit": "tok/s",
                "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
        "roofline": {"kernel": "slx_switchglu (k_qgemv + k_down, PDL pair)",
                     "bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                     "frac": round(achieved / peak, 4),
                     "traffic": traffic,
                     "algorithmic_bytes_per_launch": per_launch,
                     "launches_timed": len(durs),
                     "sampling": "layers 3, 11, 19, 27, 35 of every step",
                     "mean_launch_us": round(1000 * mean_ms, 2)},
        "gpu_launches": launches,
        "clocks": clk,
        "pool": {"miss_rate": round(st["miss_rate"], 5),
                 "hits": st["hits"], "misses": st["misses"],
                 "prefetch_used": st["pf_used"]},
        "setup_s": {"load": round(t_load, 1), "prompt_and_warmup":
                    round(t_prompt, 1)},
    }
    if cpu:
        res["cpu_baseline"] = cpu
    print(json.dumps(res), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--preset", default=PRESET,
                    help="synthetic model shape (parity/debug runs)")
    ap.add_argument("--prompt", type=int, default=PROMPT_TOKENS)
    ap.add_argument("--budget-gib", type=float, default=BUDGET / (1 << 30))
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
