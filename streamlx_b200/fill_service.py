"""Host half of the in-kernel slot fill (``slx_fill_service``,
include/streamlx_cuda.h) used by the graph-launched decoder.

The reference decides a layer's slots on the host between the router and
the expert math (streamlx/integrate.py:234-250) and overlaps the misses'
reads with the hits' compute (streamlx/integrate.py:97-139).  Here the whole
decode step is one CUDA graph; each layer's SwitchGLU launch reports the
layer's routed ids and next-layer prediction through host-mapped memory as
it starts, and parks only when one of its routed experts has no slot.  The
host follows the records in layer order, runs the pool bookkeeping of each
call exactly as the reference does, and serves a parked layer: it copies the
raw MLX bytes of that layer's pending fills and a descriptor into device
memory on a copy stream of its own, then the release ticket, and the parked
kernel repacks the experts into their slots and installs the new table.

Nothing in a service waits on the compute stream (the parked kernel holds
it): only copies on the service stream, whose sources are page-locked host
buffers.
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib as L
from .stindex import PARTS, PROJS

_ALIGN = 256


def _align(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


class FillService:
    """Mapped log / park words, the device descriptor and staging, and the
    service stream of one decoder."""

    def __init__(self, n_layers: int, n_table: int, max_items: int,
                 staging_bytes: int, device, wait_s: float = 30.0):
        self.device = device
        self.n_layers = n_layers
        self.n_table = n_table
        self.max_items = max_items
        self.wait_ns = int(wait_s * 1e9)
        W = L.FILL_LOG_WORDS
        self.log_host = torch.zeros(n_layers * W, dtype=torch.int32,
                                    pin_memory=True)
        self.log = self.log_host.numpy().reshape(n_layers, W)
        self.park_host = torch.zeros(16, dtype=torch.int32, pin_memory=True)
        self.park = self.park_host.numpy()
        self.log_dev = L.host_device_ptr(self.log_host.data_ptr())
        self.park_dev = L.host_device_ptr(self.park_host.data_ptr())
        self.desc_bytes = _align(L.FILL_HEADER_BYTES +
                                 max_items * L.FILL_ITEM_BYTES + 4 * n_table)
        self.desc_dev = torch.zeros(self.desc_bytes, dtype=torch.uint8,
                                    device=device)
        self.desc_host = torch.zeros(self.desc_bytes, dtype=torch.uint8,
                                     pin_memory=True)
        d = self.desc_host.numpy()
        self.h_head = d[:L.FILL_HEADER_BYTES].view(np.int32)
        self.h_items = d[L.FILL_HEADER_BYTES:L.FILL_HEADER_BYTES +
                         max_items * L.FILL_ITEM_BYTES].view(np.int64) \
            .reshape(max_items, L.FILL_ITEM_BYTES // 8)
        t0 = L.FILL_HEADER_BYTES + max_items * L.FILL_ITEM_BYTES
        self.h_table = d[t0:t0 + 4 * n_table].view(np.int32)
        # word 0: release ticket, word 32: the kernels' "go" word
        self.words_dev = torch.zeros(64, dtype=torch.int32, device=device)
        self.release_host = torch.zeros(16, dtype=torch.int32,
                                        pin_memory=True)
        self.staging = torch.empty(staging_bytes, dtype=torch.uint8,
                                   device=device)
        self.stream = torch.cuda.Stream(device=device)
        self.served = 0
        self.stats = {"parks": 0, "experts": 0, "bytes": 0}

    # ------------------------------------------------------------ launch --

    def svc(self, layer: int, stamp_ptr: int, pred_ids=None,
            pred_scores=None) -> L.slx_fill_service:
        W = L.FILL_LOG_WORDS
        return L.slx_fill_service(
            layer, self.max_items, stamp_ptr, self.log_dev + 4 * W * layer,
            L.ptr(pred_ids), L.ptr(pred_scores), self.park_dev,
            self.words_dev.data_ptr(), self.desc_dev.data_ptr(),
            self.words_dev.data_ptr() + 4 * 32, self.wait_ns)

    def reset_words(self) -> None:
        """Clear the log, park and release words (no step is running)."""
        self.log[:] = 0
        self.park[:] = 0
        self.words_dev.zero_()
        self.served = 0

    # ------------------------------------------------------------- serve --

    def pending_park(self, stamp: int):
        """(layer, ticket) of a parked layer of this step not yet served."""
        p = self.park
        t = int(p[0])
        if t == 0 or t == self.served or int(p[2]) != stamp:
            return None
        return int(p[1]), t

    def serve(self, layer: int, ticket: int, pool) -> int:
        """Hand pool `layer`'s pending fills and its table to the parked
        kernel.  Returns the number of experts sent."""
        store = pool.store
        keep, raws = store.take_pending(pool.slot_table)
        if len(keep) > self.max_items:
            self.abort(ticket)
            raise RuntimeError(f"layer {layer}: {len(keep)} slot fills exceed "
                               f"the service descriptor ({self.max_items})")
        regions: dict = {}
        dsts, srcs, sizes = [], [], []
        off = 0
        for slot, e, raw, rd in keep:
            if id(raw) in regions:
                continue
            base, total = raw["__arena__"]
            regions[id(raw)] = (rd.arena.base_ptr() + base, off)
            dsts.append(self.staging.data_ptr() + off)
            srcs.append(rd.arena.base_ptr() + base)
            sizes.append(total)
            off += _align(total)
        if off > self.staging.numel():
            self.abort(ticket)
            raise RuntimeError(f"layer {layer}: {off} bytes of fills exceed "
                               f"the {self.staging.numel()}-byte staging")
        h = self.h_head
        h[:] = 0
        h[0], h[1], h[2], h[3] = ticket, layer, len(keep), self.n_table
        for i, (slot, e, raw, rd) in enumerate(keep):
            host0, soff = regions[id(raw)]
            row = self.h_items[i]
            row[0] = slot                     # int32 slot + int32 pad
            j = 1
            for proj in PROJS:
                for part in PARTS:
                    v = raw[(e, proj, part)]
                    a = np.frombuffer(v, dtype=np.uint8).ctypes.data
                    row[j] = self.staging.data_ptr() + soff + (a - host0)
                    j += 1
        self.h_table[:] = store.table_words(pool.slot_table)
        self.release_host[0] = ticket
        dsts += [self.desc_dev.data_ptr(), self.words_dev.data_ptr()]
        srcs += [self.desc_host.data_ptr(), self.release_host.data_ptr()]
        sizes += [self.desc_bytes, 4]
        L.copy_many(dsts, srcs, sizes, self.stream)
        ev = torch.cuda.Event()
        ev.record(self.stream)
        for rd, raw in raws:
            rd.release_raw(raw, ev)
        store.mark_clean()
        self.served = ticket
        self.stats["parks"] += 1
        self.stats["experts"] += len(keep)
        self.stats["bytes"] += int(sum(sizes))
        return len(keep)

    def abort(self, ticket: int) -> None:
        """Release a parked kernel without fills (it reports the layer as
        SLX_ERR_UNMAPPED_EXPERT)."""
        self.release_host[0] = -ticket
        L.copy_many([self.words_dev.data_ptr()], [self.release_host.data_ptr()],
                    [4], self.stream)
        self.served = ticket
