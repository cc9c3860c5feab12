"""Span-merged ``pread`` of expert rows into pinned host memory.

Same public surface and IO accounting as the reference's
``streamlx/reader.py`` (ExpertReader, reader.py:34-152):

* ``_plan`` sorts requests by (path, offset) and merges a request into the
  previous span when it starts ``0 <= gap <= merge_gap`` bytes after it and
  the merged span stays within ``max_span`` (reader.py:64-78);
* spans are read concurrently on a small thread pool, a short read raises
  ``IOError`` (reader.py:80-100);
* ``bytes_read`` counts every byte off the file (gap bytes included),
  ``useful_bytes`` the requested ones, ``reads`` the preads issued;
* ``read_experts_raw`` returns ``{(expert, proj, part): memoryview}`` and is
  safe to call from any thread (prefetch and sweep read-ahead use it from
  worker threads, reader.py:112-123).

B200 difference: each span is read with ``os.preadv`` directly into a slot
of a pinned (page-locked) host arena, so the host->HBM copies that follow are
true DMA transfers on a copy stream.  The arena is a ring; a region is
reused only after the copies that read it have completed (``release``).
Without a CUDA device (unit tests of the bookkeeping) the arena is ordinary
host memory.
"""

from __future__ import annotations

import os
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .stindex import PARTS, PROJS, SafetensorsIndex, TensorLoc

def _native():
    """The library's batched pread, or None when it is not built."""
    try:
        from . import _lib
        _lib.lib()
        return _lib
    except (ImportError, OSError):
        return None


_NP_VIEW = {"U32": np.uint32, "BF16": np.uint16, "F16": np.float16,
            "F32": np.float32, "U16": np.uint16, "U8": np.uint8}


class _Arena:
    """Ring allocator over one host buffer.

    Every allocation stays *live* until ``release``; a released region is
    reusable once its CUDA event (the last copy that reads it) has completed.
    Wrapping onto a still-live region raises instead of overwriting it."""

    def __init__(self, nbytes: int, pinned: bool):
        self.pinned = pinned
        if pinned:
            import torch
            self._t = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
            self.buf = self._t.numpy()
        else:
            self._t = None
            self.buf = np.empty(nbytes, dtype=np.uint8)
        self.size = nbytes
        self.head = 0
        self._lock = threading.Lock()
        self._regions: dict[int, list] = {}   # start -> [end, live, event]

    def base_ptr(self) -> int:
        return self.buf.ctypes.data

    def alloc(self, n: int) -> int:
        n = (n + 255) // 256 * 256
        if n > self.size:
            raise MemoryError(f"read of {n} bytes exceeds the {self.size}-byte "
                              "staging arena")
        with self._lock:
            if self.head + n > self.size:
                self.head = 0
            start, end = self.head, self.head + n
            for s0 in list(self._regions):
                e0, live, ev = self._regions[s0]
                if s0 < end and start < e0:
                    if live:
                        raise MemoryError(
                            "staging arena exhausted: reads still in use "
                            f"overlap [{start}, {end}); raise arena_bytes")
                    if ev is not None:
                        ev.synchronize()
                    del self._regions[s0]
            self._regions[start] = [end, True, None]
            self.head = end
            return start

    def release(self, start: int, n: int, event=None) -> None:
        """Mark a region reusable once `event` (a CUDA event recorded after
        the last copy that reads it) has completed; None = immediately."""
        with self._lock:
            r = self._regions.get(start)
            if r is None:
                return
            if event is None:
                del self._regions[start]
            else:
                r[1], r[2] = False, event


class ExpertReader:
    """Reads expert rows of stacked switch tensors; batch-coalescing planner."""

    def __init__(self, index: SafetensorsIndex, workers: int = 6,
                 merge_gap: int = 64 * 1024, max_span: int = 16 * 1024 * 1024,
                 arena_bytes: int = 512 << 20, pinned: bool | None = None):
        self.index = index
        self.workers = workers
        self.merge_gap = merge_gap
        self.max_span = max_span
        self._fds: dict[str, int] = {}
        self._fd_lock = threading.Lock()
        self._ex = ThreadPoolExecutor(max_workers=workers,
                                      thread_name_prefix="streamlx-pread")
        if pinned is None:
            try:
                import torch
                pinned = torch.cuda.is_available()
            except Exception:   # noqa: BLE001 - torch optional for bookkeeping
                pinned = False
        self.arena = _Arena(arena_bytes, pinned)
        self.bytes_read = 0
        self.useful_bytes = 0
        self.reads = 0
        self._stat_lock = threading.Lock()

    def _fd(self, path: str) -> int:
        with self._fd_lock:
            fd = self._fds.get(path)
            if fd is None:
                fd = os.open(path, os.O_RDONLY)
                self._fds[path] = fd
            return fd

    # -- planning ------------------------------------------------------------

    def _plan(self, requests):
        """[(key, path, off, n)] -> [(path, off, n, [(key, rel_off, n)])]."""
        spans: list = []
        for key, path, off, n in sorted(requests, key=lambda r: (r[1], r[2])):
            if spans:
                s_path, s_off, s_n, members = spans[-1]
                gap = off - (s_off + s_n)
                if (path == s_path and 0 <= gap <= self.merge_gap
                        and (off + n) - s_off <= self.max_span):
                    members.append((key, off - s_off, n))
                    spans[-1] = (s_path, s_off, (off + n) - s_off, members)
                    continue
            spans.append((path, off, n, [(key, 0, n)]))
        return spans

    def read_ranges(self, requests) -> dict:
        """[(key, path, off, n)] -> {key: memoryview of exactly n bytes}
        (views into the staging arena; call ``release_raw`` when done)."""
        spans = self._plan(requests)
        # Each span sits at an arena offset congruent to its file offset
        # (mod 256), so every tensor piece keeps the file's alignment: a
        # whole read can then move to the GPU as one copy and the pieces are
        # still 16-byte aligned there.
        rel = []
        o = 0
        for s in spans:
            o += (s[1] - o) % 256
            rel.append(o)
            o += s[2]
        total = (o + 255) // 256 * 256
        base = self.arena.alloc(total) if total else 0
        buf = self.arena.buf
        offs = [base + r for r in rel]

        out: dict = {}
        try:
            done = self._read_spans(spans, offs, buf)
        except BaseException:
            if total:
                self.arena.release(base, total)
            raise
        for i in done:
            path, off, n, members = spans[i]
            with self._stat_lock:
                self.bytes_read += n
                self.reads += 1
            view = memoryview(buf[offs[i]:offs[i] + n])
            for key, rel, m in members:
                out[key] = view[rel:rel + m]
                with self._stat_lock:
                    self.useful_bytes += m
        out["__arena__"] = (base, total)
        return out

    def _read_spans(self, spans, offs, buf) -> range:
        """pread every span into the arena: one native call over a pool of
        threads when the library is built, else one os.preadv per span on
        the Python pool (host IO either way)."""
        n_sp = len(spans)
        if n_sp == 0:
            return range(0)
        L = _native()
        if L is not None:
            fds = np.array([self._fd(sp[0]) for sp in spans], dtype=np.int32)
            off = np.array([sp[1] for sp in spans], dtype=np.int64)
            size = np.array([sp[2] for sp in spans], dtype=np.int64)
            dst = np.array([buf.ctypes.data + o for o in offs],
                           dtype=np.uint64)
            rc, bad, err = L.pread_many(fds, off, size, dst, self.workers)
            if rc != 0:
                path, o, n, _ = spans[bad] if bad >= 0 else spans[0]
                raise IOError(f"short read at {o} (+{n}) of {path}"
                              + (f": {os.strerror(err)}" if err else ""))
            return range(n_sp)

        def read_span(i):
            path, off, n, _ = spans[i]
            view = memoryview(buf[offs[i]:offs[i] + n])
            got = os.preadv(self._fd(path), [view], off)
            if got != n:
                raise IOError(f"short read {got}/{n} at {off} of {path}")
            return i

        futs = [self._ex.submit(read_span, i) for i in range(n_sp)]
        try:
            return [f.result() for f in futs]
        except BaseException:
            for f in futs:
                f.cancel()
            for f in futs:
                try:
                    f.result()
                except BaseException:   # noqa: BLE001 - first error re-raised
                    pass
            raise

    def release_raw(self, raw: dict, event=None) -> None:
        """Return a read's staging region to the arena (after `event`)."""
        base, total = raw.get("__arena__", (0, 0))
        if total:
            self.arena.release(base, total, event)

    # -- expert-level API ----------------------------------------------------

    def read_experts_raw(self, layer_triples: dict, ids: list[int]) -> dict:
        """{(e, proj, part): memoryview} -- raw bytes only, one coalesced
        batch.  Safe from any thread."""
        requests = []
        for e in ids:
            for proj in PROJS:
                for part in PARTS:
                    path, off, n = layer_triples[proj][part].expert_range(e)
                    requests.append(((e, proj, part), path, off, n))
        return self.read_ranges(requests)

    def experts_from_raw(self, layer_triples: dict, ids: list[int],
                         raw: dict) -> dict:
        """{e: {proj: {part: memoryview}}} from a read_experts_raw result."""
        return {e: {proj: {part: raw[(e, proj, part)] for part in PARTS}
                    for proj in PROJS} for e in ids}

    def read_experts(self, layer_triples: dict, ids: list[int]) -> dict:
        return self.experts_from_raw(layer_triples, ids,
                                     self.read_experts_raw(layer_triples, ids))

    def read_expert(self, layer_triples: dict, e: int) -> dict:
        return self.read_experts(layer_triples, [e])[e]

    @staticmethod
    def as_array(view: memoryview, loc: TensorLoc) -> np.ndarray:
        """numpy view of one expert row (uint16 for bf16 parts)."""
        return np.frombuffer(view, dtype=_NP_VIEW[loc.dtype]).reshape(
            loc.shape[1:])

    def reset_stats(self) -> None:
        self.bytes_read = 0
        self.useful_bytes = 0
        self.reads = 0

    def close(self) -> None:
        self._ex.shutdown(wait=True)
        for fd in self._fds.values():
            os.close(fd)
        self._fds.clear()
