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


def decode(model, toks):
    out = []
    for t in toks:
        model.step(torch.tensor([int(t)], dtype=torch.int32,
                                device=model.device))
        out.append(model.logits.clone())
    torch.cuda.synchronize()
    return torch.cat(out).cpu()


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
    got = decode(model, toks)
    local_experts = sum(p.n_slots for p in pools.values())
    model.ep.close()
    dist.barrier()
    res = {"rank": rank, "world": dist.get_world_size(),
           "local_experts": local_experts}
    if rank == 0:
        ref, _, _, rd = load_streaming_model(d, 10**13, k=cfg.top_k,
                                             device=dev, resident="on")
        want = decode(ref, toks)
        res["bit_identical"] = bool(torch.equal(got, want))
        res["max_abs"] = float((got.float() - want.float()).abs().max())
        res["tokens_equal"] = bool(torch.equal(got.argmax(-1),
                                               want.argmax(-1)))
        print(json.dumps(res), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
