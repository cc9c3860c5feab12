"""Routing traces: capture the routed expert ids of a run and write them in
the warm-start format that ``preload_popular`` reads.

File format (the one streamlx's capture tool writes and its loader reads,
examples/capture_trace.py:34,98-139 and streamlx/integrate.py:476-506):

* ``<out>.npz`` (numpy ``savez_compressed``):
  ``experts`` uint16 ``[tokens, moe_layers, k]`` -- routed ids, ``0xFFFF``
  where a slot holds no id; ``seq_id`` uint32 ``[tokens]`` -- which input
  sequence a row came from; ``pos`` uint32 ``[tokens]`` -- its position in
  that sequence; ``prompt_class`` uint8 ``[tokens]`` (0).
* ``<out stem>.meta.json``: ``schema_version`` 1, ``model``, ``n_experts``,
  ``k``, ``n_moe_layers``, ``layer_ids`` (model layer of each trace axis --
  models with dense layers are not axis-identity), ``bytes_per_expert``
  (per layer, as a string-keyed map), ``tokens``, ``sequences``.

Capture uses the wrappers' ``record_sink`` (every pool call appends
``(layer, ids [B, T, k])``), so it sees exactly the ids the pools were asked
for, in call order, whether the decoder runs eagerly or as CUDA graphs.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

PAD = 0xFFFF
SCHEMA_VERSION = 1


class TraceRecorder:
    """Attach to a model's pool wrappers and collect per-token routing rows.

    ``rec = TraceRecorder(model, pools)``; run sequences, calling
    ``rec.end_sequence()`` after each; then ``rec.write(path)``."""

    def __init__(self, model, pools: dict):
        self.model = model
        self.pools = pools
        self.layer_ids = sorted(pools)
        self._sink: list = []
        self._blocks: list[np.ndarray] = []
        self._seq: list[np.ndarray] = []
        self._pos: list[np.ndarray] = []
        self.k = None
        for lid in self.layer_ids:
            self._wrapper(lid).record_sink = self._sink

    def _wrapper(self, lid: int):
        return self.model.layers[lid].mlp.switch_mlp

    def detach(self) -> None:
        for lid in self.layer_ids:
            self._wrapper(lid).record_sink = None

    def end_sequence(self) -> int:
        """Close the current sequence: its rows become one block of the
        trace.  Returns the sequence's token count."""
        flush = getattr(self.model, "flush", None)
        if flush is not None:
            flush()             # a graph decoder's deferred bookkeeping
        rows: dict[int, list] = {lid: [] for lid in self.layer_ids}
        for lid, idx in self._sink:
            if lid in rows:
                arr = np.asarray(idx)
                rows[lid].append(arr.reshape(-1, arr.shape[-1]))
        self._sink.clear()
        if not rows[self.layer_ids[0]]:
            return 0
        per = {lid: np.concatenate(r, 0) for lid, r in rows.items()}
        T = per[self.layer_ids[0]].shape[0]
        k = max(a.shape[1] for a in per.values())
        self.k = k if self.k is None else max(self.k, k)
        block = np.full((T, len(self.layer_ids), k), PAD, dtype=np.uint16)
        for ax, lid in enumerate(self.layer_ids):
            a = per[lid]
            if a.shape[0] != T:
                raise RuntimeError(f"layer {lid}: {a.shape[0]} routed rows "
                                   f"for {T} tokens")
            block[:, ax, :a.shape[1]] = a.astype(np.uint16)
        seq = len(self._blocks)
        self._blocks.append(block)
        self._seq.append(np.full(T, seq, dtype=np.uint32))
        self._pos.append(np.arange(T, dtype=np.uint32))
        return T

    def write(self, out: str, model_name: str = "") -> tuple[Path, Path]:
        """Write ``out`` (.npz) and its ``.meta.json`` sidecar."""
        if self._sink:
            self.end_sequence()
        if not self._blocks:
            raise RuntimeError("no routed tokens recorded")
        k = self.k
        blocks = []
        for b in self._blocks:
            if b.shape[2] < k:
                pad = np.full(b.shape[:2] + (k - b.shape[2],), PAD,
                              dtype=np.uint16)
                b = np.concatenate([b, pad], 2)
            blocks.append(b)
        p0 = self.pools[self.layer_ids[0]]
        return write_trace(
            out, np.concatenate(blocks, 0), np.concatenate(self._seq),
            np.concatenate(self._pos), self.layer_ids,
            n_experts=int(p0.n_experts),
            bytes_per_expert={lid: int(self.pools[lid].index
                                       .layer_expert_bytes(lid))
                              for lid in self.layer_ids},
            model_name=model_name)


def write_trace(out: str, experts: np.ndarray, seq_id: np.ndarray,
                pos: np.ndarray, layer_ids: list, n_experts: int,
                bytes_per_expert: dict, model_name: str = "",
                prompt_class: np.ndarray | None = None
                ) -> tuple[Path, Path]:
    """Write a routing trace and its sidecar (format in the module doc)."""
    experts = np.asarray(experts)
    if experts.ndim != 3 or experts.shape[1] != len(layer_ids):
        raise ValueError(f"experts must be [tokens, {len(layer_ids)}, k], "
                         f"got {experts.shape}")
    T = experts.shape[0]
    if prompt_class is None:
        prompt_class = np.zeros(T, dtype=np.uint8)
    out_p = Path(out)
    if out_p.suffix != ".npz":
        out_p = out_p.with_suffix(".npz")
    np.savez_compressed(out_p, experts=experts.astype(np.uint16),
                        seq_id=np.asarray(seq_id, dtype=np.uint32),
                        pos=np.asarray(pos, dtype=np.uint32),
                        prompt_class=np.asarray(prompt_class, dtype=np.uint8))
    meta = {
        "schema_version": SCHEMA_VERSION,
        "model": model_name,
        "n_experts": int(n_experts),
        "k": int(experts.shape[2]),
        "n_moe_layers": len(layer_ids),
        "layer_ids": [int(i) for i in layer_ids],
        "bytes_per_expert": {str(int(i)): int(bytes_per_expert[i])
                             for i in layer_ids},
        "tokens": int(T),
        "sequences": int(len(np.unique(seq_id))) if T else 0,
    }
    side = out_p.parent / (out_p.stem + ".meta.json")
    side.write_text(json.dumps(meta, indent=2))
    return out_p, side


def read_trace(path: str) -> tuple[dict, dict | None]:
    """(arrays, meta or None) of a trace file."""
    p = Path(path)
    with np.load(p) as d:
        arrays = {k: d[k] for k in d.files}
    side = p.parent / (p.stem + ".meta.json")
    meta = json.loads(side.read_text()) if side.exists() else None
    return arrays, meta


def capture_trace(model, pools: dict, sequences, out: str,
                  model_name: str = "") -> tuple[Path, Path]:
    """Run each token-id sequence through the decoder one token at a time
    (the synthetic models' ids are their text) and write the routing trace."""
    import torch
    rec = TraceRecorder(model, pools)
    try:
        for seq in sequences:
            if hasattr(model, "reset"):
                model.reset()
            for tok in seq:
                model.step(torch.tensor([int(tok)], dtype=torch.int32,
                                        device=model.device))
            rec.end_sequence()
        return rec.write(out, model_name=model_name)
    finally:
        rec.detach()
