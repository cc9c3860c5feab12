"""Model integration: a pool-backed SwitchGLU replacement and the loader.

Mirrors ``streamlx/integrate.py``:

* ``StreamingSwitchGLU(pool)`` is call-compatible with
  ``SwitchGLU.__call__(x, indices) -> [B, T, k, H]`` (per-expert outputs
  before score weighting, integrate.py:234-298).  ``fused(x, scores,
  indices)`` additionally returns the score-weighted combine ``[B, T, H]``
  (+ shared expert) from the same fused kernel -- the path the decoder uses.
* Per call, the pool bookkeeping follows the reference exactly (it decides
  the hit/miss/eviction trace): decode = ``B*T == 1``; one host sync on the
  routed ids; ``prefetch_absorb`` first; then the hits of the call are
  touched before the misses are ensured when both exist
  (``_overlapped``, integrate.py:97-139), else ``ensure(uniq)``; then the
  next layer's prefetch is started with the predicted ids ordered by score
  (integrate.py:255-260).  Prediction gates itself off once 512 routed ids
  were tallied at < 55% agreement (integrate.py:76-77).
* Prefill whose expert union exceeds the pool runs the expert-major sweep
  (``STREAMLX_PREFILL=sweep``, default; integrate.py:141-232): pairs grouped
  by expert, ``STREAMLX_SWEEP_BATCH`` experts per batch in ascending id,
  read one batch ahead on a worker thread, the ``n_slots`` most-routed
  experts adopted into the pool (``STREAMLX_SWEEP_WARM``) and retouched so
  the most frequent ends most-recently-used.  ``STREAMLX_PREFILL=slice`` is
  the legacy token-slice path (integrate.py:269-298).
* ``load_streaming_model`` returns ``(model, tokenizer, pools, reader)``
  with the per-layer budget split ``max(k, budget_left / n_streamed /
  bytes_per_expert)`` (integrate.py:397-473); ``STREAMLX_PREFETCH=0``
  disables the next-layer prediction links.

The B200 difference is below the bookkeeping: every resident expert of a
call is computed by ONE fused kernel launch that maps expert ids to slots on
the device, after the misses of the call have landed in their slots.
"""

from __future__ import annotations

import os
import sys
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .pool import StreamingSwitchMLP
from .reader import ExpertReader
from .stindex import PARTS, PROJS, SafetensorsIndex

_PF_EX = None


def _pf_ex():
    global _PF_EX
    if _PF_EX is None:
        _PF_EX = ThreadPoolExecutor(max_workers=1,
                                    thread_name_prefix="streamlx-pf")
    return _PF_EX


class StreamingSwitchGLU:
    """Pool-backed replacement for one MoE layer's SwitchGLU."""

    def __init__(self, pool: StreamingSwitchMLP, shared=None):
        self.pool = pool
        self.shared = shared          # (slx_shared_expert, buffer, inter) or None
        self.record_sink = None
        self.prefill_mode = os.environ.get("STREAMLX_PREFILL", "sweep")
        self.sweep_batch = int(os.environ.get("STREAMLX_SWEEP_BATCH", "16"))
        self.sweep_warm = os.environ.get("STREAMLX_SWEEP_WARM", "1") != "0"
        self._sweep_ex = None
        # (next pool, predict(x) -> (ids, scores) numpy or None)
        self._pf_next = None
        self._mini = None

    # -------------------------------------------------------- bookkeeping --

    def pred_gate(self) -> bool:
        """Whether this call makes a next-layer prediction: a link exists
        and the next pool's agreement has not fallen below 55% over 512+
        routed ids (integrate.py:67-77)."""
        nxt = self._pf_next
        if nxt is None:
            return False
        pool_j = nxt[0]
        return not (pool_j.pf_agree_tot >= 512 and
                    pool_j.prefetch_agreement() < 0.55)

    def _pf_pred(self, x, k):
        if not self.pred_gate():
            return None
        predict = self._pf_next[1]
        try:
            return predict(x)
        except Exception:   # noqa: BLE001 - arch surprise: disable the link
            self._pf_next = None
            return None

    def start_prefetch(self, pred) -> None:
        """Start the next layer's prefetch from a prediction (ids, scores):
        ids ordered by score, stable (integrate.py:255-260)."""
        if pred is None or self._pf_next is None:
            return
        pi = np.asarray(pred[0]).reshape(-1)
        ps = np.asarray(pred[1]).reshape(-1)
        ordered = list(dict.fromkeys(
            int(pi[j]) for j in np.argsort(-ps, kind="stable")))
        self._pf_next[0].prefetch_start(ordered, _pf_ex())

    def route(self, idx: np.ndarray, pred=None,
              start_prefetch: bool = True) -> str:
        """Pool bookkeeping of one call (no device work except slot fills).
        idx: [B, T, k] routed expert ids (host).  pred: next-layer
        prediction (ids, scores) for decode, or None.  Returns "pool" when the
        call's experts are resident, else the prefill mode to run.
        ``start_prefetch=False``: the caller has already started this call's
        next-layer prefetch (it touches only the next pool, whose state no
        call in between changes)."""
        pool = self.pool
        decode = idx.shape[0] * idx.shape[1] == 1
        if self.record_sink is not None:
            self.record_sink.append((pool.layer, idx.copy()))
        flat = [int(e) for e in idx.reshape(-1).tolist()]
        uniq = list(dict.fromkeys(flat))
        pool.begin_call()
        if decode:
            pool.prefetch_absorb(uniq)
        if len(uniq) <= pool.n_slots:
            if decode and pool.hit_all(uniq):
                if start_prefetch:
                    self.start_prefetch(pred)
                return "pool"
            if decode:
                hits = [e for e in uniq if pool.resident(e)]
                miss = [e for e in uniq if not pool.resident(e)]
                if hits and miss:
                    pool.touch(hits)
                    pool.ensure(miss)
                else:
                    pool.ensure(uniq)
                if start_prefetch:
                    self.start_prefetch(pred)
            else:
                pool.ensure(uniq)
            return "pool"
        return self.prefill_mode

    # ------------------------------------------------------------ compute --

    def _host_ids(self, indices):
        import torch
        if isinstance(indices, torch.Tensor):
            return indices.detach().to("cpu").numpy()
        return np.asarray(indices)

    def __call__(self, x, indices):
        """Drop-in: per-expert outputs [B, T, k, H] (unweighted)."""
        return self._run(x, None, indices)

    def fused(self, x, scores, indices):
        """Score-weighted combine [B, T, H] (+ shared expert)."""
        return self._run(x, scores, indices)

    def _run(self, x, scores, indices):
        from . import ops
        B, T, k = indices.shape
        pred = self._pf_pred(x, k) if B * T == 1 else None
        idx = self._host_ids(indices)          # the per-layer host sync
        mode = self.route(idx, pred)
        if mode == "pool":
            return self._pool_compute(x, scores, indices, idx)
        if mode == "sweep":
            y = self._expert_sweep(x, idx)
        else:
            y = self._slice_prefill(x, idx)
        if scores is None:
            return y
        return self._combine(x, y, scores)

    def _pool_compute(self, x, scores, indices, idx):
        from . import ops
        pool = self.pool
        B, T, k = idx.shape
        x2d = ops.as_bf16_2d(x)
        if (B * T * k >= ops.PREFILL_MIN_PAIRS and
                pool.store.__class__.__name__ == "HbmSlotStore" and
                ops.prefill_supported(pool.hidden, pool.inter, pool.bits)):
            y = self._pool_prefill(x2d, idx)
            if scores is None:
                return y
            return self._combine(x, y, scores)
        pool.sync_device()
        ids = ops.as_ids_2d(indices, k, x2d.device)
        sh = self.shared
        y = ops.switchglu(pool.store.bank, x2d, ids, k,
                          scores=None if scores is None else
                          scores.reshape(-1, k).float().contiguous(),
                          table=pool.store.table_dev,
                          shared=sh[0] if sh else None, inter=pool.inter,
                          shared_inter=sh[2] if sh else 0)
        if scores is None:
            return y.reshape(B, T, k, -1)
        return y.reshape(B, T, -1)

    def _pool_prefill(self, x2d, idx):
        """Resident experts of a multi-token call on the tensor-core grouped
        prefill: pairs grouped by the slot of their expert (the host holds
        the id -> slot map after the call's bookkeeping), each output written
        at its (token, pick) row.  Returns [B, T, k, H]."""
        from . import ops
        pool = self.pool
        B, T, k = idx.shape
        flat = idx.reshape(-1).astype(np.int64)
        slot_of = np.array([pool.id2slot[int(e)] for e in flat], dtype=np.int64)
        order = np.argsort(slot_of, kind="stable")
        slots, counts = np.unique(slot_of[order], return_counts=True)
        row_of_pair = order // k
        y = ops.prefill_grouped(pool.store.bank, x2d, row_of_pair, slots,
                                counts, out_row=order, n_out=flat.size)
        return y.reshape(B, T, k, -1)

    def _combine(self, x, y, scores):
        """Score-weighted sum of per-expert outputs (+ shared expert) for the
        prefill paths."""
        import torch

        from . import ops
        B, T, k, H = y.shape
        acc = (y.float() * scores.reshape(B, T, k, 1).float()).sum(-2)
        if self.shared is not None:
            _, sh_buf, sh_inter = self.shared
            x2d = ops.as_bf16_2d(x)
            zero_ids = torch.zeros(x2d.shape[0], 1, dtype=torch.int32,
                                   device=x2d.device)
            ys = ops.switchglu(shared_bank(sh_buf, self.pool, sh_inter), x2d,
                               zero_ids, 1, inter=sh_inter)
            acc = acc + ys.reshape(B, T, H).float()
        return acc.to(torch.bfloat16)

    # ------------------------------------------------------ prefill paths --

    def _mini_pool(self, n: int):
        import torch

        from . import _lib as L
        pool = self.pool
        stride = L.slot_stride(pool.hidden, pool.inter, pool.bits)
        if self._mini is None or self._mini[0] < n:
            buf = torch.empty(n * stride, dtype=torch.uint8,
                              device=pool.store.pool.device)
            self._mini = (n, buf, stride)
        return self._mini

    def _expert_sweep(self, x, idx):
        """Expert-major prefill (streamlx/integrate.py:141-232)."""
        import torch

        from . import _lib as L
        from . import ops
        pool = self.pool
        b, t, k = idx.shape
        P = b * t
        on_gpu = pool.store.__class__.__name__ == "HbmSlotStore"
        x_rows = ops.as_bf16_2d(x) if on_gpu else None
        flat = idx.reshape(-1).astype(np.int64)
        row_of_pair = np.repeat(np.arange(P, dtype=np.int64), k)
        order = np.argsort(flat, kind="stable")
        sorted_e = flat[order]
        uniq, starts = np.unique(sorted_e, return_index=True)
        bounds = np.append(starts, sorted_e.size)
        counts = bounds[1:] - bounds[:-1]
        warm_ids: set = set()
        if self.sweep_warm:
            top = np.argsort(counts, kind="stable")[::-1][:pool.n_slots]
            warm_ids = {int(uniq[i]) for i in top}
        if self._sweep_ex is None:
            self._sweep_ex = ThreadPoolExecutor(max_workers=1)
        batches = [[int(e) for e in uniq[i0:i0 + self.sweep_batch]]
                   for i0 in range(0, len(uniq), self.sweep_batch)]
        fut = self._sweep_ex.submit(pool.reader.read_experts_raw,
                                    pool.triples_loc, batches[0])
        y = None
        if on_gpu:
            H = x_rows.shape[1]
            # per-pair outputs land at their (token, pick) rows directly
            y = torch.empty(sorted_e.size, H, dtype=torch.bfloat16,
                            device=x_rows.device)
            nb, mini, stride = self._mini_pool(self.sweep_batch)
        for bi, ids in enumerate(batches):
            t0 = time.perf_counter()
            raw = fut.result()
            pool.sweep_fetch_s += time.perf_counter() - t0
            if bi + 1 < len(batches):
                fut = self._sweep_ex.submit(pool.reader.read_experts_raw,
                                            pool.triples_loc, batches[bi + 1])
            pool.sweep_experts += len(ids)
            i0 = bi * self.sweep_batch
            i1 = min(i0 + self.sweep_batch, len(uniq))
            lo, hi = int(bounds[i0]), int(bounds[i1])
            adopt_items = []
            for e in ids:
                if e in warm_ids:
                    adopt_items.append((pool.adopt(e, None), e))
            if y is not None:
                store = pool.store
                store.write_to(pool.reader, raw,
                               [(mini.data_ptr() + j * stride, e)
                                for j, e in enumerate(ids)], release=False)
                sel = order[lo:hi]
                bank = L.bank_struct(mini, len(ids), pool.hidden, pool.inter,
                                     pool.bits, stride)
                if ops.prefill_supported(pool.hidden, pool.inter, pool.bits):
                    # tensor-core grouped GEMM over the batch's pairs, each
                    # output written at its (token, pick) row
                    ops.prefill_grouped(bank, x_rows, row_of_pair[sel],
                                        list(range(len(ids))),
                                        counts[i0:i1], out=y, out_row=sel)
                else:
                    slot = np.searchsorted(uniq[i0:i1], sorted_e[lo:hi])
                    xb = x_rows[torch.as_tensor(row_of_pair[sel],
                                                device=x_rows.device)]
                    sid = torch.as_tensor(slot.astype(np.int32),
                                          device=x_rows.device).reshape(-1, 1)
                    yb = ops.switchglu(bank, xb.contiguous(), sid, 1,
                                       inter=pool.inter).reshape(hi - lo, H)
                    y[torch.as_tensor(sel, device=y.device)] = yb
            pool.store.write(pool.reader, raw, adopt_items)
        if warm_ids:
            for i in np.argsort(counts, kind="stable"):
                e = int(uniq[i])
                if e in warm_ids and e in pool.id2slot:
                    pool.id2slot.move_to_end(e)
        if y is None:
            return None
        return y.reshape(b, t, k, H)

    def _slice_prefill(self, x, idx):
        """Legacy token-slice prefill (streamlx/integrate.py:269-298)."""
        import torch

        from . import ops
        pool = self.pool
        b, t, k = idx.shape
        flat = idx.reshape(-1, k)
        on_gpu = pool.store.__class__.__name__ == "HbmSlotStore"
        x_flat = ops.as_bf16_2d(x) if on_gpu else None
        outs = []
        s, P = 0, flat.shape[0]
        while s < P:
            union: set = set()
            e = s
            while e < P:
                nxt = union | set(flat[e].tolist())
                if len(nxt) > pool.n_slots:
                    break
                union = nxt
                e += 1
            if e == s:
                raise RuntimeError(f"k > n_slots (layer {pool.layer})")
            ids = list(dict.fromkeys(flat[s:e].reshape(-1).tolist()))
            pool.ensure(ids)
            if on_gpu:
                pool.sync_device()
                sl = ops.as_ids_2d(flat[s:e], k, x_flat.device)
                y = ops.switchglu(pool.store.bank, x_flat[s:e].contiguous(), sl,
                                  k, table=pool.store.table_dev,
                                  inter=pool.inter)
                torch.cuda.current_stream().synchronize()
                outs.append(y)
            s = e
        if not outs:
            return None
        return torch.cat(outs, 0).reshape(b, t, k, -1)


def shared_bank(sh_buf, pool, sh_inter):
    """Bank view of a shared expert buffer (one slot)."""
    from . import _lib as L
    return L.bank_struct(sh_buf, 1, pool.hidden, sh_inter, pool.bits,
                         L.slot_stride(pool.hidden, sh_inter, pool.bits))


def install_streaming(model, model_dir: str, n_slots: int):
    """Swap every MoE layer's switch_mlp for a streaming wrapper; returns
    (pools, reader), the reader shared by all pools (integrate.py:301-319)."""
    index = SafetensorsIndex(model_dir)
    reader = ExpertReader(index)
    pools: dict = {}
    for i, layer in enumerate(model.layers):
        mlp = getattr(layer, "mlp", None)
        if mlp is None or not hasattr(mlp, "switch_mlp"):
            continue
        pool = StreamingSwitchMLP(model_dir, i, n_slots, index=index,
                                  reader=reader)
        layer.mlp.switch_mlp = StreamingSwitchGLU(pool, mlp.shared_struct())
        pools[i] = pool
    if not pools:
        raise RuntimeError("no MoE layers found to wrap")
    if hasattr(model, "flush"):
        for pool in pools.values():
            pool.flush_hook = model.flush
    model.link_prefetch(pools)
    return pools, reader


def plan_residency(layers: list, bpe: dict, n_exp: dict, budget_bytes: int,
                   k: int) -> tuple[set, float]:
    """Which MoE layers hold ALL their experts (no pool, no streaming), and
    the budget left for the pools of the others (streamlx/integrate.py:
    322-346 decides the same way).

    Layers are visited from the smallest whole-layer size up.  A layer is
    made resident when its whole size fits the fair share of what is left
    (``left / still-streamed layers``) and, after paying for it, every other
    still-streamed layer can keep ``k`` slots.  Paying for a small layer
    raises the fair share of the rest, so on a budget near the total expert
    bytes the decision cascades to every layer; on a small budget none
    qualifies."""
    streamed = sorted(layers, key=lambda j: n_exp[j] * bpe[j])
    order = list(streamed)
    resident: set = set()
    left = float(budget_bytes)
    # k-slot floor of every still-streamed layer, kept as a running sum
    floor = float(sum(k * bpe[j] for j in streamed))
    for i in order:
        whole = n_exp[i] * bpe[i]
        others = floor - k * bpe[i]
        if whole <= left / len(streamed) and left - whole >= others:
            resident.add(i)
            streamed.remove(i)
            floor = others
            left -= whole
    return resident, left


class IdTokenizer:
    """Tokenizer of the synthetic checkpoints: ids are the text."""

    eos_token_ids: set = set()

    def encode(self, ids):
        return [int(i) for i in ids]

    def decode(self, ids):
        return " ".join(str(int(i)) for i in ids)


def load_streaming_model(model_dir: str, budget_bytes: int, k: int = 8,
                         trust_remote_code: bool = False,
                         tokenizer_config: dict | None = None,
                         resident: str | None = None, device=None,
                         expert_parallel: bool = False, ep_group=None):
    """Build the decoder with every MoE layer pool-backed.  Returns
    ``(model, tokenizer, pools, reader)`` (integrate.py:397-473).

    ``expert_parallel``: one process per GPU under torch.distributed; this
    rank keeps only its block of every layer's experts, all resident (the
    budget is not used), and decode steps exchange the experts' outputs
    over NVLink peer memory (no reference counterpart).  A group of one
    rank holds every expert and decodes without the exchange."""
    from .model import SynthDecoder
    index = SafetensorsIndex(model_dir)
    reader = ExpertReader(index)
    model = SynthDecoder.from_checkpoint(model_dir, index, device=device)
    moe_layers = list(range(model.cfg.layers))
    if expert_parallel:
        return _load_expert_parallel(model, model_dir, index, reader,
                                     moe_layers, ep_group)
    bpe = {i: index.layer_expert_bytes(i) for i in moe_layers}
    n_exp = {i: index.switch_triples(i)["gate_proj"]["weight"].shape[0]
             for i in moe_layers}
    mode = resident if resident is not None else os.environ.get(
        "STREAMLX_RESIDENT", "off")
    res_layers: set = set()
    budget_left = float(budget_bytes)
    if mode not in ("off", "0"):
        res_layers, budget_left = plan_residency(moe_layers, bpe, n_exp,
                                                 budget_bytes, k)
    streamed = [i for i in moe_layers if i not in res_layers]
    pools: dict = {}
    for i in moe_layers:
        if i in res_layers:
            slots = n_exp[i]
        else:
            slots = max(k, int(budget_left / len(streamed) / bpe[i]))
        pool = StreamingSwitchMLP(model_dir, i, slots, index=index,
                                  reader=reader, device=model.device)
        if i in res_layers:   # fully resident: fill every slot once
            for e0 in range(0, n_exp[i], 32):   # reads of <= 32 experts
                pool.begin_call()
                pool.ensure(list(range(e0, min(e0 + 32, n_exp[i]))))
        model.layers[i].mlp.switch_mlp = StreamingSwitchGLU(
            pool, model.layers[i].mlp.shared_struct())
        pool.flush_hook = model.flush   # stats first finish deferred steps
        if i in res_layers:
            # every expert in its slot for good: the reference runs these
            # layers on the stock path, outside the returned pools
            pool.sync_device()
            model.static_glu[i] = True
        else:
            pools[i] = pool
    if os.environ.get("STREAMLX_PREFETCH", "1") != "0":
        linked = model.link_prefetch({i: pools[i] for i in streamed})
        if linked:
            print(f"[streamlx] attention-window prefetch: {linked} layer "
                  f"links", file=sys.stderr)
    if res_layers:
        rb = sum(n_exp[i] * bpe[i] for i in res_layers) / 2**30
        print(f"[streamlx] {len(res_layers)} fully-resident MoE layers "
              f"({rb:.1f} GiB); {len(streamed)} streamed", file=sys.stderr)
    return model, IdTokenizer(), pools, reader


def _load_expert_parallel(model, model_dir, index, reader, moe_layers,
                          group):
    import torch.distributed as dist

    from .expert_parallel import local_range
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    pools: dict = {}
    for i in moe_layers:
        n_exp = index.switch_triples(i)["gate_proj"]["weight"].shape[0]
        e0, e1 = local_range(n_exp, world, rank)
        pool = StreamingSwitchMLP(model_dir, i, max(1, e1 - e0), index=index,
                                  reader=reader, device=model.device)
        for a in range(e0, e1, 32):
            pool.begin_call()
            pool.ensure(list(range(a, min(a + 32, e1))))
        pool.sync_device()
        model.layers[i].mlp.switch_mlp = StreamingSwitchGLU(
            pool, model.layers[i].mlp.shared_struct())
        pools[i] = pool
    for pool in pools.values():
        pool.flush_hook = model.flush
    model.static_glu = [True] * len(model.layers)
    if world > 1:
        model.enable_expert_parallel(group)
    # one rank holds every expert: no rows to exchange, so the step keeps
    # the single-GPU form (the SwitchGLU launch combines the experts itself)
    return model, IdTokenizer(), pools, reader


def preload_popular(pools: dict, trace_npz: str) -> int:
    """Warm-start every pool with the experts its layer routed to most often
    in a routing trace (``streamlx_b200.trace`` format; streamlx/integrate.py:
    476-506 reads the same file).

    The trace's axis of each model layer comes from the sidecar's
    ``layer_ids`` (identity when there is no sidecar); a layer absent from
    the trace is left cold.  Per pool the ``n_slots`` largest counts are
    taken in the order numpy's default argsort of the counts gives, reversed
    (the same call as the reference, so ties fall the same way), then loaded
    in ascending id order (one ``ensure``: file-ordered reads).  Pad entries
    (0xFFFF) are not counted.  Returns the number of experts loaded."""
    from .trace import PAD, read_trace
    arrays, meta = read_trace(trace_npz)
    routed = arrays["experts"]
    axes = (meta["layer_ids"] if meta is not None
            else list(range(routed.shape[1])))
    axis_of = {int(lid): a for a, lid in enumerate(axes)}
    loaded = 0
    for lid, pool in pools.items():
        a = axis_of.get(int(lid))
        if a is None:
            continue
        col = routed[:, a, :].reshape(-1)
        counts = np.bincount(col[col != PAD], minlength=pool.n_experts)
        pick = np.argsort(counts)[::-1][:pool.n_slots]
        pool.begin_call()
        pool.ensure(sorted(int(e) for e in pick))
        loaded += len(pick)
    return loaded


def aggregate_stats(pools: dict) -> dict:
    """Sum of the pool counters (integrate.py:509-526)."""
    tot = {"hits": 0, "misses": 0, "evictions": 0, "fetch_s": 0.0,
           "sweep_experts": 0, "sweep_fetch_s": 0.0, "adopted": 0,
           "pf_calls": 0, "pf_launched": 0, "pf_used": 0,
           "pf_agree_hit": 0, "pf_agree_tot": 0}
    for p in pools.values():
        s = p.stats
        for key in ("hits", "misses", "evictions", "sweep_experts", "adopted",
                    "pf_calls", "pf_launched", "pf_used", "pf_agree_hit",
                    "pf_agree_tot"):
            tot[key] += s.get(key, 0)
        tot["fetch_s"] += s["fetch_s"]
        tot["sweep_fetch_s"] += s.get("sweep_fetch_s", 0.0)
    acc = tot["hits"] + tot["misses"]
    tot["miss_rate"] = tot["misses"] / acc if acc else 0.0
    tot["fetch_s"] = round(tot["fetch_s"], 3)
    tot["sweep_fetch_s"] = round(tot["sweep_fetch_s"], 3)
    return tot
