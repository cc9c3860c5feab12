"""Expert-parallel dispatch / combine (streamlx_b200/expert_parallel.py) on
CPU ranks: world size 2 over gloo, an injected expert function (so the test
checks the exchange, not the arithmetic), compared with the same layer
computed in one process."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from streamlx_b200 import expert_parallel as EP

E, H, K, T = 10, 32, 3, 7          # 10 experts over 2 ranks: 5 + 5


def _weights():
    rng = np.random.default_rng(123)
    return rng.standard_normal((E, H, H)) * 0.2


def _expert_rows(x: np.ndarray, eids, W) -> np.ndarray:
    y = np.stack([x[i].astype(np.float64) @ W[int(e)] for i, e in enumerate(eids)])
    return torch.from_numpy(y.astype(np.float32)).to(torch.bfloat16)


def _tokens(seed: int):
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)
                         ).to(torch.bfloat16)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)])
    sc = rng.random((T, K)).astype(np.float32)
    return x, ids, sc


def _reference(x, ids, sc, W, shared: bool):
    xp = x.float().numpy()[np.arange(T * K) // K]     # row of each pair
    y = _expert_rows(xp, ids.reshape(-1), W).view(T, K, H).float()
    acc = (y * torch.from_numpy(sc).reshape(T, K, 1)).sum(1)
    if shared:
        acc = acc + _shared(x).float()
    return acc.to(torch.bfloat16)


def _shared(x):
    return (x.float() * 0.5).to(torch.bfloat16)


def _worker(rank, world, port, mode):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}",
                            rank=rank, world_size=world)
    try:
        W = _weights()
        e0, e1 = EP.local_range(E, world, rank)

        def expert_fn(rows, eids):
            assert ((eids >= e0) & (eids < e1)).all(), "pair sent to wrong rank"
            return _expert_rows(rows.float().numpy(), eids, W)

        moe = EP.ExpertParallelMoE(E, expert_fn, shared_fn=_shared)
        if mode == "sharded":
            x, ids, sc = _tokens(seed=rank)          # each rank: own tokens
            got = moe.forward(x, ids, sc)
            want = _reference(x, ids, sc, W, shared=True)
            assert torch.equal(got.view(torch.int16), want.view(torch.int16))
            # an empty rank-local batch still takes part in the exchange
            got0 = moe.forward(x[:0], ids[:0], sc[:0])
            assert got0.shape == (0, H)
        else:
            x, ids, sc = _tokens(seed=99)            # same tokens everywhere
            got = moe.forward(x, ids, sc, tokens="replicated")
            want = _reference(x, ids, sc, W, shared=True)
            d = (got.float() - want.float()).abs().max().item()
            assert d <= 2e-2 * max(1.0, want.float().abs().max().item()), d
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("mode", ["sharded", "replicated"])
def test_ep_exchange_two_cpu_ranks(mode):
    mp.spawn(_worker, args=(2, _free_port(), mode), nprocs=2, join=True)


def test_plan_dispatch_groups_pairs_stably():
    ids = np.array([[9, 0, 4], [5, 1, 2]])
    plan = EP.plan_dispatch(ids, 10, 2)
    assert plan.send_counts.tolist() == [4, 2]
    assert plan.order.tolist() == [1, 2, 4, 5, 0, 3]
    assert EP.local_range(10, 4, 3) == (9, 10)
    assert EP.owner_of(7, 10, 4) == 2
    with pytest.raises(IndexError):
        EP.plan_dispatch(np.array([[10]]), 10, 2)
