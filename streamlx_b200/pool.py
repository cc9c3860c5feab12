"""Per-layer expert pool: HBM slot pool + the reference's slot policy.

Mirrors ``streamlx/pool.py`` (StreamingSwitchMLP, pool.py:53-332): same
attributes (``n_slots``, ``n_experts``, ``layer``, ``id2slot``, ``free``,
``slot_table``, ``SENTINEL``, S3-FIFO queues, counters), same methods
(``ensure``, ``touch``, ``resident``, ``adopt``, ``prefetch_start``,
``prefetch_absorb``, ``prefetch_agreement``, ``stats``, ``reset_stats``,
``__call__``) and the same decisions, pinned against the reference's own
code by tests/golden:

* LRU: hit -> ``move_to_end``; miss -> ``free.pop()`` (LIFO) or evict the
  ``id2slot`` head (pool.py:110-171);
* S3-FIFO (``STREAMLX_EVICT=s3fifo``): small FIFO of ``max(1, 0.1 n)``
  entries, main of ``max(1, n - small)``, frequency capped at 3, ghost
  queue; *plus* protection of every id touched or inserted during the current
  wrapper call (``begin_call``).  The reference evicts an id it inserted
  earlier in the same call and then fails with ``KeyError`` whenever one call
  inserts more misses than the small FIFO holds (pool.py:139-150, 195-196);
  here a protected small-queue head is promoted to main instead of being
  ghosted, and main eviction skips protected entries;
* misses are slot-assigned in order, then fetched as ONE coalesced read.

Where the weights live differs: slots are rows of one tile-format HBM buffer
(``HbmSlotStore``) and a device copy of ``slot_table`` lets the kernels map
expert ids to slots without a host round trip.  A slot fill is one
host->device copy of the pinned read region plus one pack kernel.
"""

from __future__ import annotations

import os
import time
from collections import OrderedDict

import numpy as np

from .reader import ExpertReader
from .stindex import PARTS, PROJS, SafetensorsIndex

SENTINEL = np.uint32(0xFFFFFFFF)


# --------------------------------------------------------------- storage --

class NullSlotStore:
    """Bookkeeping-only store (no device): records which expert went where.
    Used to replay pool traces on machines without a GPU."""

    def __init__(self, *args, **kw):
        self.writes: list[tuple[int, int]] = []

    def write(self, reader, raw, items) -> None:
        self.writes.extend((slot, e) for slot, e in items)
        reader.release_raw(raw)

    def write_to(self, reader, raw, items, release: bool = True) -> None:
        if release:
            reader.release_raw(raw)

    def sync_table(self, slot_table) -> None:
        pass


_STAGING: dict = {}


def _staging(torch, device, nbytes: int):
    """Device staging buffer shared by every store of a device (writes are
    ordered on one stream, so one buffer suffices); grows on demand."""
    key = str(device)
    t = _STAGING.get(key)
    if t is None or t.numel() < nbytes:
        t = torch.empty(max(nbytes, 64 << 20), dtype=torch.uint8,
                        device=device)
        _STAGING[key] = t
    return t


class HbmSlotStore:
    """n_slots experts in the tile format, plus the device slot table."""

    def __init__(self, n_slots: int, n_experts: int, hidden: int, inter: int,
                 bits: int, triples_loc: dict, device=None):
        import torch

        from . import _lib
        self.torch = torch
        self.L = _lib
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.hidden, self.inter, self.bits = hidden, inter, bits
        self.n_slots = n_slots
        self.stride = _lib.slot_stride(hidden, inter, bits)
        self.pool = torch.zeros(n_slots * self.stride, dtype=torch.uint8,
                                device=self.device)
        self.table_dev = torch.full((n_experts,), -1, dtype=torch.int32,
                                    device=self.device)
        self._table_host = torch.full((n_experts,), -1, dtype=torch.int32,
                                      pin_memory=True)
        self.triples_loc = triples_loc
        self.bank = _lib.bank_struct(self.pool, n_slots, hidden, inter, bits,
                                     self.stride)
        self._dirty = True
        # Deferred mode (the graph decoder, while a step runs): slot fills
        # and table pushes are recorded instead of issued, because the device
        # may be reading this pool's slots.  They are applied between steps
        # (flush_pending) or handed to a parked layer kernel (take_pending).
        self.deferred = False
        self._pending: list = []        # (reader, raw, [(slot, expert)])
        self._slot_table = None

    def slot_ptr(self, slot: int) -> int:
        return self.pool.data_ptr() + slot * self.stride

    def write(self, reader: ExpertReader, raw: dict, items) -> None:
        """Copy the experts of `items` [(slot, expert)] from a read result
        into their slots (recorded for later in deferred mode)."""
        self._dirty = True
        if self.deferred:
            self._pending.append((reader, raw, list(items)))
            return
        self.write_to(reader, raw, [(self.slot_ptr(s), e) for s, e in items])

    def take_pending(self, slot_table: np.ndarray) -> tuple[list, list]:
        """Coalesced recorded fills: the last fill of each slot whose expert
        still occupies that slot in `slot_table`, as [(slot, expert, raw,
        reader)], plus every (reader, raw) the records referenced (each to be
        released exactly once by the caller).  Clears the record."""
        last: dict = {}
        raws: dict = {}
        for reader, raw, items in self._pending:
            raws[id(raw)] = (reader, raw)
            for slot, e in items:
                last[slot] = (e, raw, reader)
        self._pending = []
        keep = [(slot, e, raw, rd) for slot, (e, raw, rd) in last.items()
                if int(slot_table[e]) == slot]
        return keep, list(raws.values())

    def has_pending(self) -> bool:
        return bool(self._pending) or self._dirty

    def flush_pending(self, slot_table: np.ndarray, stream=None) -> int:
        """Apply the recorded fills now, on `stream` (nothing may be reading
        this pool's slots meanwhile), then push the table.  Returns the
        number of experts packed."""
        keep, raws = self.take_pending(slot_table)
        by_raw: dict = {}
        for slot, e, raw, rd in keep:
            by_raw.setdefault(id(raw), (rd, raw, []))[2].append(
                (self.slot_ptr(slot), e))
        for rd, raw in raws:
            ent = by_raw.get(id(raw))
            if ent is not None:
                self.write_to(rd, raw, ent[2], release=True, stream=stream)
            else:
                rd.release_raw(raw)
        was, self.deferred = self.deferred, False
        try:
            self._dirty = True
            self.sync_table(slot_table, stream=stream)
        finally:
            self.deferred = was
        return len(keep)

    def write_to(self, reader: ExpertReader, raw: dict, items,
                 release: bool = True, stream=None) -> None:
        """Pack the experts of `items` [(device_ptr, expert)] from a read
        result: one host->device copy of the read's pinned region, one pack
        kernel.  With `release`, the region returns to the reader's arena
        once the copy has run.  Ordered on `stream` (default: current)."""
        torch = self.torch
        if not items:
            if release:
                reader.release_raw(raw)
            return
        base, total = raw["__arena__"]
        staging = _staging(torch, self.device, total)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        arena = reader.arena
        host0 = arena.base_ptr() + base
        self.L.copy_many([staging.data_ptr()], [host0], [total], stream)
        dev0 = staging.data_ptr()
        experts = []
        for slot, e in items:
            trip = []
            for proj in PROJS:
                ptrs = []
                for part in PARTS:
                    v = raw[(e, proj, part)]
                    addr = np.frombuffer(v, dtype=np.uint8).ctypes.data
                    ptrs.append(dev0 + (addr - host0))
                trip.append(tuple(_Ptr(p) for p in ptrs))
            experts.append(tuple(trip))
        self.L.pack_experts(experts, self.hidden, self.inter, self.bits,
                            [d for d, _ in items], stream)
        if release:
            ev = torch.cuda.Event()
            ev.record(stream)
            reader.release_raw(raw, ev)

    def sync_table(self, slot_table: np.ndarray, stream=None) -> None:
        """Push the host slot table (SENTINEL -> -1) to the device copy
        (deferred mode: only remembered)."""
        if not self._dirty:
            return
        if self.deferred:
            self._slot_table = slot_table
            return
        torch = self.torch
        t = self._table_host.numpy()
        t[:] = slot_table.astype(np.int64).astype(np.int32)
        if stream is None:
            self.table_dev.copy_(self._table_host, non_blocking=True)
        else:
            with torch.cuda.stream(stream):
                self.table_dev.copy_(self._table_host, non_blocking=True)
        self._dirty = False

    def table_words(self, slot_table: np.ndarray) -> np.ndarray:
        """The device form of a host slot table (int32, -1 = absent)."""
        return slot_table.astype(np.int64).astype(np.int32)

    def mark_clean(self) -> None:
        """The device table was installed another way (a parked kernel)."""
        self._dirty = False

    def mark_dirty(self) -> None:
        self._dirty = True


class _Ptr:
    """Minimal stand-in for a tensor in _lib.qmat (exposes data_ptr)."""

    __slots__ = ("p",)

    def __init__(self, p: int):
        self.p = p

    def data_ptr(self) -> int:
        return self.p


# ------------------------------------------------------------------ pool --

class StreamingSwitchMLP:
    SENTINEL = SENTINEL
    # Confidence cut for prefetch (streamlx/pool.py:218-221): read at import,
    # like the reference's class attribute.
    _PF_TOPM = int(os.environ.get("STREAMLX_PF_TOPM", "7"))

    def __init__(self, model_dir: str, layer: int, n_slots: int,
                 index: SafetensorsIndex | None = None,
                 reader: ExpertReader | None = None, store=None,
                 device=None):
        self.index = index or SafetensorsIndex(model_dir)
        self.reader = reader or ExpertReader(self.index)
        self.layer = layer
        self.triples_loc = self.index.switch_triples(layer)
        self.qparams = {p: self.index.quant_params(self.triples_loc[p])
                        for p in PROJS}
        self.n_experts = self.triples_loc["gate_proj"]["weight"].shape[0]
        if n_slots < 1:
            raise ValueError("n_slots must be >= 1")
        self.n_slots = n_slots
        hidden, inter, bits, gs = self.qparams["gate_proj"]
        if gs != 64 or {q[2] for q in self.qparams.values()} != {bits}:
            raise ValueError(f"layer {layer}: expert projections must share "
                             f"one bit width with group size 64 ({self.qparams})")
        self.hidden, self.inter, self.bits = hidden, inter, bits
        self.id2slot: OrderedDict[int, int] = OrderedDict()
        self.free = list(range(n_slots))
        self.policy = os.environ.get("STREAMLX_EVICT", "lru")
        self.n_small = max(1, int(n_slots * 0.1))
        self.n_main = max(1, n_slots - self.n_small)
        self.q_small: OrderedDict[int, int] = OrderedDict()
        self.q_main: OrderedDict[int, int] = OrderedDict()
        self.q_ghost: OrderedDict[int, bool] = OrderedDict()
        self.slot_table = np.full(self.n_experts, SENTINEL, dtype=np.uint32)
        self._protect: set = set()
        if store == "null":
            store = NullSlotStore()
        self.store = store if store is not None else HbmSlotStore(
            n_slots, self.n_experts, hidden, inter, bits, self.triples_loc,
            device=device)
        self.reset_stats()
        self._pf = None   # (pred_set, launch, future, rank_of)

    # -- policy (decisions identical to streamlx/pool.py:110-171) ----------

    def begin_call(self) -> None:
        """Start of one wrapper call: clears the S3-FIFO protection set."""
        self._protect = set()

    def _policy_hit(self, e: int) -> None:
        if self.policy == "s3fifo":
            q = self.q_small if e in self.q_small else self.q_main
            q[e] = min(3, q[e] + 1)
        else:
            self.id2slot.move_to_end(e)

    def _s3_evict_main(self) -> int:
        skipped = 0
        while self.q_main:
            e, f = self.q_main.popitem(last=False)
            if e in self._protect:            # in use by the current call
                self.q_main[e] = f
                skipped += 1
                if skipped > len(self.q_main):
                    break
                continue
            skipped = 0
            if f > 0:
                self.q_main[e] = f - 1
                continue
            return e
        raise RuntimeError("s3fifo: no evictable entry in main "
                           "(every entry is in use by this call)")

    def _s3_insert(self, e: int) -> int | None:
        if e in self.q_ghost:
            del self.q_ghost[e]
            victim = (self._s3_evict_main()
                      if len(self.q_main) >= self.n_main else None)
            self.q_main[e] = 0
            return victim
        victim = None
        if len(self.q_small) >= self.n_small:
            e2, f = self.q_small.popitem(last=False)
            if f > 0 or e2 in self._protect:
                if len(self.q_main) >= self.n_main:
                    victim = self._s3_evict_main()
                self.q_main[e2] = 0
            else:
                if len(self.q_ghost) >= self.n_main:
                    self.q_ghost.popitem(last=False)
                self.q_ghost[e2] = True
                victim = e2
        self.q_small[e] = 0
        return victim

    def _take_slot_for(self, e: int) -> int:
        if self.policy == "s3fifo":
            victim = self._s3_insert(e)
            if victim is not None:
                slot = self.id2slot.pop(victim)
                self.slot_table[victim] = SENTINEL
                self.evictions += 1
                self.free.append(slot)
            slot = self.free.pop()
        elif self.free:
            slot = self.free.pop()
        else:
            old_id, slot = self.id2slot.popitem(last=False)
            self.slot_table[old_id] = SENTINEL
            self.evictions += 1
        self.id2slot[e] = slot
        self.slot_table[e] = slot
        self.store_dirty()
        return slot

    def store_dirty(self) -> None:
        mark = getattr(self.store, "mark_dirty", None)
        if mark:
            mark()

    # -- residency ----------------------------------------------------------

    def ensure(self, ids: list[int]) -> list[int]:
        """Slots for `ids` in order; misses fetched as one coalesced read."""
        slots = []
        missing: list[int] = []
        for e in ids:
            e = int(e)
            self._protect.add(e)
            if e in self.id2slot:
                self._policy_hit(e)
                self.hits += 1
            else:
                self.misses += 1
                self._take_slot_for(e)
                missing.append(e)
            slots.append(self.id2slot[e])
        if missing:
            t0 = time.perf_counter()
            raw = self.reader.read_experts_raw(self.triples_loc, missing)
            self.store.write(self.reader, raw,
                             [(self.id2slot[e], e) for e in missing])
            self.fetch_s += time.perf_counter() - t0
        return slots

    def resident(self, e: int) -> bool:
        return e in self.id2slot

    def hit_all(self, ids: list[int]) -> bool:
        """``ensure(ids)`` when every id is resident -- the common decode
        call -- without building the slot list: the same policy hits, in
        order, and hit counts.  Returns False (and changes nothing) if any
        id is missing."""
        id2slot = self.id2slot
        for e in ids:
            if e not in id2slot:
                return False
        self._protect.update(ids)
        if self.policy == "s3fifo":
            for e in ids:
                self._policy_hit(e)
        else:
            mte = id2slot.move_to_end
            for e in ids:
                mte(e)
        self.hits += len(ids)
        return True

    def touch(self, ids: list[int]) -> None:
        for e in ids:
            e = int(e)
            self._protect.add(e)
            self._policy_hit(e)
            self.hits += 1

    def adopt(self, e: int, arrays) -> None:
        """Place expert e from already-read bytes without IO (prefill sweep
        warm-up, prefetch absorption).  ``arrays`` is (raw_read, keep_open):
        the raw read that holds e's bytes."""
        e = int(e)
        self._protect.add(e)
        if e in self.id2slot:
            self._policy_hit(e)
            slot = self.id2slot[e]
        else:
            slot = self._take_slot_for(e)
        self.adopted += 1
        return slot

    # -- prefetch (streamlx/pool.py:218-280) ---------------------------------

    def prefetch_start(self, pred: list[int], ex) -> None:
        rank_of = {e: r for r, e in enumerate(pred)}
        missing = [e for e in pred if e not in self.id2slot]
        launch = [e for e in missing if rank_of[e] < self._PF_TOPM]
        for e in launch:
            self.pf_rank.setdefault(rank_of[e], [0, 0])[0] += 1
        self._drop_pending_prefetch()
        if not launch:
            self._pf = (set(pred), [], None, rank_of)
            return
        self.pf_launched += len(launch)
        self._pf = (set(pred), launch,
                    ex.submit(self.reader.read_experts_raw, self.triples_loc,
                              launch), rank_of)

    def _drop_pending_prefetch(self) -> None:
        """An unconsumed prediction is dropped: its bytes go back."""
        if self._pf is None or self._pf[2] is None:
            return
        fut = self._pf[2]

        def _release(f, reader=self.reader):
            try:
                reader.release_raw(f.result())
            except Exception:   # noqa: BLE001 - failed read: nothing to free
                pass
        fut.add_done_callback(_release)

    def prefetch_absorb(self, wanted: list[int]) -> None:
        pf, self._pf = self._pf, None
        if pf is None:
            return
        pred_set, launch, fut, rank_of = pf
        self.pf_calls += 1
        self.pf_agree_hit += len(set(wanted) & pred_set)
        self.pf_agree_tot += len(wanted)
        if fut is None:
            return
        wanted_set = set(wanted)
        take = [e for e in launch if e in wanted_set and e not in self.id2slot]
        try:
            raw = fut.result()
        except Exception:   # noqa: BLE001 - the reference swallows it too
            return
        if not take:
            self.reader.release_raw(raw)
            return
        items = []
        for e in take:
            items.append((self.adopt(e, None), e))
            self.pf_rank.setdefault(rank_of[e], [0, 0])[1] += 1
        self.store.write(self.reader, raw, items)
        self.adopted -= len(take)       # keep sweep-adoption count pure
        self.pf_used += len(take)

    def prefetch_agreement(self) -> float:
        return (self.pf_agree_hit / self.pf_agree_tot
                if self.pf_agree_tot else 1.0)

    # -- misc ------------------------------------------------------------------

    def sync_device(self) -> None:
        """Make the device slot table match the host bookkeeping."""
        self.store.sync_table(self.slot_table)

    def reset_stats(self) -> None:
        self.hits = self.misses = self.evictions = 0
        self.fetch_s = 0.0
        self.sweep_experts = 0
        self.sweep_fetch_s = 0.0
        self.adopted = 0
        self.pf_calls = self.pf_launched = self.pf_used = 0
        self.pf_agree_hit = self.pf_agree_tot = 0
        self.pf_rank = {}

    @property
    def stats(self) -> dict:
        hook = getattr(self, "flush_hook", None)
        if hook is not None:        # a decoder with deferred bookkeeping
            hook()
        total = self.hits + self.misses
        return {"hits": self.hits, "misses": self.misses,
                "evictions": self.evictions,
                "miss_rate": self.misses / total if total else 0.0,
                "fetch_s": round(self.fetch_s, 4),
                "sweep_experts": self.sweep_experts,
                "sweep_fetch_s": round(self.sweep_fetch_s, 4),
                "adopted": self.adopted,
                "pf_calls": self.pf_calls,
                "pf_launched": self.pf_launched,
                "pf_used": self.pf_used,
                "pf_agree_hit": self.pf_agree_hit,
                "pf_agree_tot": self.pf_agree_tot,
                "bytes_read": self.reader.bytes_read,
                "reads": self.reader.reads}

    def __call__(self, x, expert_ids: list[int]):
        """Per-expert outputs [1, 1, k, H] for one token (streamlx/pool.py:
        299-304): ensure the experts, then run the fused kernel in drop-in
        (unweighted) mode."""
        if len(expert_ids) > self.n_slots:
            raise ValueError("n_slots must be >= k")
        self.begin_call()
        self.ensure(list(expert_ids))
        from .ops import switch_forward_ids
        return switch_forward_ids(self, x, expert_ids)
