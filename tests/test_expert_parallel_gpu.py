"""Expert parallelism on real GPUs: two NCCL ranks (torchrun), experts of a
117B-shaped layer sharded 128 per GPU, token rows exchanged by all-to-all.
Each rank checks its combined outputs against the same tokens run through
all 256 experts on its own GPU (``bench.py --mode ep --check``): batch-1
decode (replicated token, all-reduce), batch-64 decode and a 2048-token
prefill (sharded tokens, dispatch/combine).  Needs two GPUs; skipped on a
machine with one GPU."""

import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(not torch.cuda.is_available() or
                    torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_ranks_nccl_matches_all_experts():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m",
           "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "bench.py"), "--mode", "ep", "--check",
           "--steps", "3", "--warmup", "3"]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert '"metric": "ep_moe_layer"' in r.stdout
