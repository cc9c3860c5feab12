"""Worker of tests/test_ep_decode_gpu.py (run under torchrun, one process per
GPU): the synthetic decoder with its experts sharded over the ranks decodes
a fixed token sequence; rank 0 then decodes the same sequence with every
expert on its own GPU and checks that the logits and tokens are
bit-identical.  Prints one JSON line on rank 0."""

import datetime
import json
import os
import sys
import tempfile

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from streamlx_b200 import synth  # noqa: E402
from streamlx_b200.integrate import load_streaming_model  # noqa: E402


def decode(model, toks, ids=None):
    out = []
    for t in toks:
        model.step(torch.tensor([int(t)], dtype=torch.int32,
                                device=model.device))
        out.append(model.logits.clone())
        if ids is not None:
            ids.append(model.g_ids.reshape(model.cfg.layers, -1).cpu().numpy())
    torch.cuda.synchronize()
    return torch.cat(out).cpu()


def oracle_check(d, toks, ids, got):
    """The sharded run against the CPU oracle: the same ordered experts at
    every layer and step (the temporal-reuse decisions taken from the GPU
    run, as in tests/test_model_gpu.py), logits within 2e-2 max-abs and
    5e-3 rel-L2 (the bf16 pipeline's own spread on these decoders)."""
    from oracle import affine as A
    from oracle.model import OracleDecoder
    o = OracleDecoder(d)
    prev = None
    worst_rel = worst_abs = 0.0
    ids_ok = True
    for t, tk in enumerate(toks):
        forced = {} if prev is None else {
            i: prev[i] for i in range(len(prev))
            if np.array_equal(ids[t][i], prev[i])}
        want, routed = o.step(int(tk), forced=forced)
        ids_ok &= all(np.array_equal(ids[t][i], routed[i])
                      for i in range(len(routed)))
        g = A.bf16_from_bits(got[t].view(torch.int16).numpy().view(np.uint16))
        w = A.bf16_round(want)
        worst_rel = max(worst_rel, A.rel_l2(g, w))
        worst_abs = max(worst_abs, float(np.max(np.abs(g - w))))
        prev = ids[t]
    return {"oracle_ids_equal": bool(ids_ok), "oracle_rel_l2": worst_rel,
            "oracle_max_abs": worst_abs,
            "oracle_ok": bool(ids_ok and worst_rel <= 5e-3 and
                              worst_abs <= 2e-2)}


def main():
    preset, steps = sys.argv[1], int(sys.argv[2])
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    root = os.environ.get("EP_TEST_DIR") or tempfile.gettempdir()
    d = os.path.join(root, f"ep_{preset}")
    if rank == 0 and not os.path.exists(os.path.join(d, ".done")):
        synth.write_model(d, synth.PRESETS[preset], seed=9)
        open(os.path.join(d, ".done"), "w").close()
    dist.barrier()
    cfg = synth.PRESETS[preset]
    toks = np.random.default_rng(3).integers(0, cfg.vocab, steps)
    model, _, pools, reader = load_streaming_model(d, 0, k=cfg.top_k,
                                                   device=dev,
                                                   expert_parallel=True)
    if model.ep is None and os.environ.get("EP_FORCE") == "1":
        model.enable_expert_parallel()      # one rank, exchange form anyway
    exchange = model.ep is not None
    ids = []
    got = decode(model, toks, ids)
    local_experts = sum(p.n_slots for p in pools.values())
    if model.ep is not None:        # one rank: every expert local, no exchange
        model.ep.close()
    dist.barrier()
    res = {"rank": rank, "world": dist.get_world_size(),
           "local_experts": local_experts, "exchange": exchange}
    if rank == 0:
        ref, _, _, rd = load_streaming_model(d, 10**13, k=cfg.top_k,
                                             device=dev, resident="on")
        want = decode(ref, toks)
        res["bit_identical"] = bool(torch.equal(got, want))
        res["max_abs"] = float((got.float() - want.float()).abs().max())
        res["tokens_equal"] = bool(torch.equal(got.argmax(-1),
                                               want.argmax(-1)))
        res.update(oracle_check(d, toks, ids, got))
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
