"""Expert parallelism: one MoE layer's routed experts sharded over the ranks
of a process group (one process per GPU), token rows exchanged by
all-to-all over NVLink (NCCL) -- or over gloo on the CPU for the tests.

The reference serves one device (streamlx/pool.py keeps every slot of a
layer on it; README.md:52); this is the scale-out of its slot pool: rank r
holds the experts ``[r*per, (r+1)*per)`` (``per = ceil(E / world)``,
contiguous id blocks) fully resident, and a layer call is

  sharded tokens (each rank owns different token rows: batch decode,
  prefill chunks)
    1. pairs (token, pick) grouped by the rank that owns their expert
       (stable, so each rank's pairs keep token order);
    2. all-to-all of the per-rank pair counts, then of the pairs' token
       rows (bf16 pairs moved as raw 32-bit words; hidden is even) and
       expert ids;
    3. every rank runs its received pairs through its local experts
       (``expert_fn``: the grouped tensor-core prefill or the fused GEMV);
    4. all-to-all of the per-pair outputs back along the reverse splits;
    5. score-weighted combine (+ shared expert) on the source rank;

  replicated tokens (batch-1 decode: every rank runs the same token)
    each rank computes only the pairs whose expert it owns, combines them
    (score-weighted, fp32), and one all-reduce sums the partial outputs.

No collective needs TMA or cluster-broadcast loads: rows land in this GPU's memory
through NCCL before any kernel reads them.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist


def experts_per_rank(n_experts: int, world: int) -> int:
    return -(-n_experts // world)


def owner_of(e, n_experts: int, world: int):
    """Rank that holds expert ``e`` (contiguous id blocks)."""
    return np.asarray(e) // experts_per_rank(n_experts, world)


def local_range(n_experts: int, world: int, rank: int) -> tuple[int, int]:
    per = experts_per_rank(n_experts, world)
    return min(rank * per, n_experts), min((rank + 1) * per, n_experts)


@dataclass
class DispatchPlan:
    order: np.ndarray        # pair indices t*k + j in send order
    send_counts: np.ndarray  # pairs sent to each rank


def plan_dispatch(ids: np.ndarray, n_experts: int, world: int) -> DispatchPlan:
    """Group the pairs of ``ids [T, k]`` by destination rank, stable."""
    flat = np.asarray(ids).reshape(-1)
    if flat.size and (flat.min() < 0 or flat.max() >= n_experts):
        raise IndexError(f"expert id outside 0..{n_experts - 1}")
    dest = owner_of(flat, n_experts, world)
    order = np.argsort(dest, kind="stable")
    counts = np.bincount(dest, minlength=world).astype(np.int64)
    return DispatchPlan(order=order, send_counts=counts)


class ExpertParallelMoE:
    """Dispatch / combine of one MoE layer over a process group.

    expert_fn(rows [n, H] bf16 tensor, expert_ids np.ndarray [n]) -> [n, H]
    bf16 per-pair UNWEIGHTED outputs of this rank's experts (ids global).
    shared_fn(x [T, H]) -> [T, H] bf16 or None: the always-on shared expert,
    computed where the token lives."""

    def __init__(self, n_experts: int, expert_fn, shared_fn=None, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_experts = n_experts
        self.expert_fn = expert_fn
        self.shared_fn = shared_fn
        self.e0, self.e1 = local_range(n_experts, self.world, self.rank)
        self.bytes_sent = 0      # token rows + outputs moved by this rank

    def _a2a(self, t: torch.Tensor, out_splits, in_splits) -> torch.Tensor:
        out = t.new_empty((int(sum(out_splits)),) + tuple(t.shape[1:]))
        dist.all_to_all_single(out, t.contiguous(), [int(v) for v in out_splits],
                               [int(v) for v in in_splits], group=self.group)
        return out

    def forward(self, x2d: torch.Tensor, ids, scores,
                tokens: str = "sharded") -> torch.Tensor:
        """x2d [T, H] bf16 (this rank's tokens), ids [T, k] (host), scores
        [T, k] -> combined [T, H] bf16."""
        ids = np.asarray(ids)
        ids = ids.reshape(x2d.shape[0], ids.shape[-1])
        if tokens == "replicated":
            return self._replicated(x2d, ids, scores)
        T, k = ids.shape
        H = x2d.shape[1]
        plan = plan_dispatch(ids, self.n_experts, self.world)
        dev = x2d.device
        # 1-2: counts, then rows and expert ids
        send_counts = torch.as_tensor(plan.send_counts, device=dev)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc = plan.send_counts.tolist()
        rc = recv_counts.cpu().tolist()
        rows_idx = torch.as_tensor(plan.order // k, device=dev)
        send_rows = x2d.index_select(0, rows_idx).view(torch.int32)
        recv_rows = self._a2a(send_rows, rc, sc).view(torch.bfloat16)
        send_eid = torch.as_tensor(ids.reshape(-1)[plan.order].astype(np.int32),
                                   device=dev)
        recv_eid = self._a2a(send_eid, rc, sc).cpu().numpy()
        # 3: local experts
        if recv_rows.shape[0]:
            y_loc = self.expert_fn(recv_rows, recv_eid)
        else:
            y_loc = recv_rows.new_empty((0, H))
        # 4: outputs back along the reverse splits
        y_back = self._a2a(y_loc.contiguous().view(torch.int32), sc,
                           rc).view(torch.bfloat16)
        self.bytes_sent += 2 * H * (int(sum(sc)) + int(sum(rc)))
        # 5: combine on the source rank
        y_pair = torch.empty(T * k, H, dtype=torch.bfloat16, device=dev)
        y_pair[torch.as_tensor(plan.order, device=dev)] = y_back
        return self._combine(x2d, y_pair.view(T, k, H), scores)

    def _replicated(self, x2d, ids, scores) -> torch.Tensor:
        T, k = ids.shape
        H = x2d.shape[1]
        dev = x2d.device
        flat = ids.reshape(-1)
        mine = np.nonzero((flat >= self.e0) & (flat < self.e1))[0]
        part = torch.zeros(T, H, dtype=torch.float32, device=dev)
        if mine.size:
            rows = x2d.index_select(0, torch.as_tensor(mine // k, device=dev))
            y = self.expert_fn(rows, flat[mine]).float()
            sc = torch.as_tensor(np.asarray(scores, dtype=np.float32)
                                 .reshape(-1)[mine], device=dev)
            part.index_add_(0, torch.as_tensor(mine // k, device=dev),
                            y * sc[:, None])
        dist.all_reduce(part, group=self.group)
        self.bytes_sent += 4 * H * T
        if self.shared_fn is not None:
            part = part + self.shared_fn(x2d).float()
        return part.to(torch.bfloat16)

    def _combine(self, x2d, y, scores) -> torch.Tensor:
        s = torch.as_tensor(np.asarray(scores, dtype=np.float32),
                            device=y.device).reshape(y.shape[0], y.shape[1], 1)
        acc = (y.float() * s).sum(1)
        if self.shared_fn is not None:
            acc = acc + self.shared_fn(x2d).float()
        return acc.to(torch.bfloat16)


def pool_expert_fn(pool):
    """expert_fn over a pool that holds this rank's experts resident: pairs
    grouped by slot through the grouped tensor-core prefill (2-bit shapes it
    supports, enough pairs) or the fused GEMV kernels (ids given as slots)."""
    from . import ops

    def fn(rows: torch.Tensor, eids: np.ndarray) -> torch.Tensor:
        slot = np.array([pool.id2slot[int(e)] for e in eids], dtype=np.int64)
        n = slot.size
        if (n >= ops.PREFILL_MIN_PAIRS and
                ops.prefill_supported(pool.hidden, pool.inter, pool.bits)):
            order = np.argsort(slot, kind="stable")
            slots, counts = np.unique(slot[order], return_counts=True)
            return ops.prefill_grouped(pool.store.bank, rows, order, slots,
                                       counts, out_row=order, n_out=n)
        sid = torch.as_tensor(slot.astype(np.int32), device=rows.device)
        return ops.switchglu(pool.store.bank, rows.contiguous(),
                             sid.reshape(-1, 1), 1,
                             inter=pool.inter).reshape(n, -1)
    return fn


def load_local_experts(model_dir: str, layer: int, n_experts: int,
                       world: int, rank: int, device=None):
    """Pool of this rank's expert block of ``layer``, every expert resident
    (one coalesced read of the block, slot writes)."""
    from .pool import StreamingSwitchMLP
    e0, e1 = local_range(n_experts, world, rank)
    pool = StreamingSwitchMLP(model_dir, layer, max(1, e1 - e0), device=device)
    pool.begin_call()
    pool.ensure(list(range(e0, e1)))
    return pool


# ----------------------------------------------------------------------
# Expert-parallel decode over NVLink peer memory (slx_ep_exchange)


class EpExchange:
    """Receive blocks and counters of the expert-parallel decoder on one
    rank, with every peer's mapped through CUDA IPC.

    Layout (include/streamlx_cuda.h, slx_ep_exchange): recv bf16
    [2][n_layers][k + 1][hidden], counters uint32 [2][n_layers].  The
    SwitchGLU launch of each rank writes its owned units' rows into every
    rank's block and counts its CTAs on every rank's counter; each rank's
    combine kernel waits on its own counter.  The handles are exchanged with
    one all_gather_object over the process group (any backend)."""

    def __init__(self, n_layers: int, k: int, hidden: int, device,
                 group=None, wait_s: float = 10.0):
        from . import _lib as L
        self.L = L
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > L.EP_MAX_RANKS:
            raise ValueError(f"{self.world} ranks > {L.EP_MAX_RANKS}")
        self.n_layers, self.k, self.hidden = n_layers, k, hidden
        self.device = device
        self.grid = L.ep_grid()
        self.wait_ns = int(wait_s * 1e9)
        self.recv = torch.zeros(2 * n_layers * (k + 1) * hidden,
                                dtype=torch.bfloat16, device=device)
        self.count = torch.zeros(max(64, 2 * n_layers), dtype=torch.int32,
                                 device=device)
        torch.cuda.synchronize(device)
        mine = (L.ipc_handle(self.recv), L.ipc_handle(self.count), self.grid)
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        grids = {g[2] for g in allh}
        if len(grids) != 1:
            raise RuntimeError(f"ranks disagree on the SwitchGLU grid: {grids}")
        self._opened: list[int] = []
        self.recv_ptr: list[int] = []
        self.count_ptr: list[int] = []
        for r, ((hr, offr), (hc, offc), _) in enumerate(allh):
            if r == self.rank:
                self.recv_ptr.append(self.recv.data_ptr())
                self.count_ptr.append(self.count.data_ptr())
                continue
            br = L.ipc_open(hr)
            self._opened.append(br)
            bc = br if hc == hr else L.ipc_open(hc)
            if bc != br:
                self._opened.append(bc)
            self.recv_ptr.append(br + offr)
            self.count_ptr.append(bc + offc)
        dist.barrier(group=group)

    def struct(self, layer: int, stamp_ptr: int, warmup: bool = False):
        L = self.L
        recv = (C_VOID * 8)(*(self.recv_ptr + [0] * (8 - self.world)))
        count = (C_VOID * 8)(*(self.count_ptr + [0] * (8 - self.world)))
        return L.slx_ep_exchange(self.rank, self.world, layer, self.n_layers,
                                 stamp_ptr, recv, count,
                                 0 if warmup else self.grid, self.wait_ns)

    def close(self) -> None:
        for b in self._opened:
            try:
                self.L.ipc_close(b)
            except Exception:   # noqa: BLE001 - best effort at teardown
                pass
        self._opened = []


import ctypes as _ctypes  # noqa: E402

C_VOID = _ctypes.c_void_p
