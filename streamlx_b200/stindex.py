"""Header-only safetensors index: tensor name -> byte range, and the byte range
of one expert's row inside a stacked ``[n_experts, ...]`` tensor.

Same public surface as the reference's ``streamlx/stindex.py``:
``TensorLoc`` (stindex.py:22-39), ``SafetensorsIndex`` with
``switch_triples`` / ``layer_expert_bytes`` / ``quant_params``
(stindex.py:43-119).  Behaviour kept identical because the expert reader, the
slot pool and the budget split all key off these ranges:

* only shards matching ``model-*.safetensors`` are indexed, in sorted order;
* absolute data offset = 8 + header length + ``data_offsets[0]``;
* bits / group_size come from ``config.json``'s ``quantization`` table
  (per-path override, then top level, then inference at group 64), with the
  ``language_model.`` prefix stripped from keys;
* errors: ``IndexError`` (expert out of range), ``KeyError`` (missing switch
  tensors), ``ValueError`` (packing mismatch), ``FileNotFoundError`` (no
  shards).
"""

from __future__ import annotations

import glob
import json
import os
import struct
from dataclasses import dataclass
from math import prod

DTYPE_SIZE = {"U32": 4, "BF16": 2, "F16": 2, "F32": 4, "U16": 2, "U8": 1}
PROJS = ("gate_proj", "up_proj", "down_proj")
PARTS = ("weight", "scales", "biases")
_VLM_PREFIX = "language_model."


@dataclass(frozen=True)
class TensorLoc:
    path: str
    abs_start: int
    nbytes: int
    dtype: str
    shape: tuple
    name: str = ""

    @property
    def row_stride(self) -> int:
        """Bytes of one leading-axis row (one expert of a stacked tensor)."""
        return DTYPE_SIZE[self.dtype] * prod(self.shape[1:])

    def expert_range(self, e: int) -> tuple[str, int, int]:
        """(path, absolute offset, nbytes) of row ``e``."""
        n = self.shape[0]
        if e < 0 or e >= n:
            raise IndexError(f"expert {e} out of range {n}")
        stride = self.row_stride
        return self.path, self.abs_start + e * stride, stride


def _read_header(path: str) -> tuple[int, dict]:
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        return 8 + hlen, json.loads(f.read(hlen))


class SafetensorsIndex:
    def __init__(self, model_dir: str):
        self.model_dir = str(model_dir)
        self.tensors: dict[str, TensorLoc] = {}
        pattern = os.path.join(self.model_dir, "model-*.safetensors")
        for shard in sorted(glob.glob(pattern)):
            base, hdr = _read_header(shard)
            for name, info in hdr.items():
                if name == "__metadata__":
                    continue
                lo, hi = info["data_offsets"]
                self.tensors[name] = TensorLoc(shard, base + lo, hi - lo,
                                               info["dtype"],
                                               tuple(info["shape"]), name)
        if not self.tensors:
            raise FileNotFoundError(f"no shards under {model_dir}")
        qtab: dict = {}
        cfg_path = os.path.join(self.model_dir, "config.json")
        if os.path.exists(cfg_path):
            with open(cfg_path) as f:
                qtab = json.load(f).get("quantization") or {}
        self._quant_default = {k: v for k, v in qtab.items()
                               if not isinstance(v, dict)}
        self._quant_by_path = {self._norm(k): v for k, v in qtab.items()
                               if isinstance(v, dict)}

    @staticmethod
    def _norm(key: str) -> str:
        return key[len(_VLM_PREFIX):] if key.startswith(_VLM_PREFIX) else key

    def switch_triples(self, layer: int) -> dict[str, dict[str, TensorLoc]]:
        """{proj: {part: TensorLoc}} of one MoE layer's stacked experts."""
        tag = f"layers.{layer}.mlp.switch_mlp."
        found: dict[str, dict[str, TensorLoc]] = {}
        for name, loc in self.tensors.items():
            if tag not in name:
                continue
            for proj in PROJS:
                for part in PARTS:
                    if name.endswith(f"{proj}.{part}"):
                        found.setdefault(proj, {})[part] = loc
        missing = [(p, q) for p in PROJS for q in PARTS
                   if q not in found.get(p, {})]
        if missing:
            raise KeyError(f"layer {layer}: missing switch tensors {missing}")
        return found

    def layer_expert_bytes(self, layer: int) -> int:
        """Bytes of ONE expert of ``layer`` (3 projections x W/S/B)."""
        return sum(loc.row_stride for parts in self.switch_triples(layer)
                   .values() for loc in parts.values())

    def quant_params(self, triple: dict[str, TensorLoc]
                     ) -> tuple[int, int, int, int]:
        """(in_features, out_features, bits, group_size) of one projection."""
        w, s = triple["weight"], triple["scales"]
        n_groups, packed = s.shape[-1], w.shape[-1]
        key = self._norm(w.name)
        if key.endswith(".weight"):
            key = key[: -len(".weight")]
        ov = self._quant_by_path.get(key, {})
        bits = ov.get("bits", self._quant_default.get("bits"))
        gs = ov.get("group_size", self._quant_default.get("group_size"))
        if gs is None:
            gs = 64
        in_features = n_groups * gs
        if bits is None:
            bits = packed * 32 // in_features
        if packed * 32 != in_features * bits or bits not in (2, 3, 4, 5, 6, 8):
            raise ValueError(f"quant mismatch for {w.name}: W{w.shape} "
                             f"S{s.shape} with bits={bits} group_size={gs}")
        return in_features, w.shape[1], bits, gs

    def get(self, name: str) -> TensorLoc:
        return self.tensors[name]

    def read_tensor(self, name: str) -> bytes:
        """Whole tensor bytes (trunk weights; experts go through the reader)."""
        loc = self.tensors[name]
        with open(loc.path, "rb") as f:
            f.seek(loc.abs_start)
            data = f.read(loc.nbytes)
        if len(data) != loc.nbytes:
            raise IOError(f"short read of {name}")
        return data
