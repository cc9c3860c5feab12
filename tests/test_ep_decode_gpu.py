"""Expert-parallel decode on real GPUs: the decoder's experts sharded over
torchrun ranks (one per GPU), the owned experts' output rows exchanged over
NVLink peer memory inside the SwitchGLU launch and combined by each rank
(slx_switchglu_ep / slx_ep_combine_rmsnorm).  The combine sums in the same
order as the single-GPU kernel, so the logits must be bit-identical to the
same model decoded on one GPU with every expert resident; the sharded run is
also checked against the CPU oracle (ordered experts at every layer and step,
logits within the decoder tolerance).  One rank holds every expert and
decodes without the exchange (the loader's process-group path on one GPU);
it runs on any machine with a GPU.  Two ranks need two GPUs."""

import json
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


def _run(n: int, preset: str, steps: int, tmp, force_ep: bool = False) -> dict:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", EP_TEST_DIR=str(tmp),
               EP_FORCE="1" if force_ep else "0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m",
           "torch.distributed.run", "--nnodes=1", "--nproc-per-node", str(n),
           "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           os.path.join(ROOT, "tests", "ep_decode_worker.py"), preset,
           str(steps)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("{")][-1]
    return json.loads(line)


@pytest.mark.parametrize("force_ep", [False, True])
@pytest.mark.parametrize("preset", ["tiny_dec", "tiny_dec2"])
def test_ep_decode_one_rank_bit_identical(preset, force_ep, tmp_path):
    """force_ep: the exchange form anyway (rows written to this rank's own
    receive block, then slx_ep_combine_rmsnorm), which one GPU can run."""
    res = _run(1, preset, 12, tmp_path, force_ep)
    assert res["world"] == 1
    assert res["exchange"] == force_ep
    assert res["bit_identical"], res
    assert res["oracle_ok"], res


@pytest.mark.skipif(not torch.cuda.is_available() or
                    torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("preset", ["tiny_dec", "tiny_dec2"])
def test_ep_decode_two_ranks_bit_identical(preset, tmp_path):
    res = _run(2, preset, 12, tmp_path)
    assert res["world"] == 2
    assert res["bit_identical"], res
    assert res["oracle_ok"], res
