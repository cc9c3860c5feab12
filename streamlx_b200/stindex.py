"""Byte-range index over a safetensors checkpoint, built from the shard
headers alone.

Format facts this module relies on (the safetensors container and MLX's
quantized-checkpoint conventions, not any particular loader):

* a shard is ``u64 little-endian header length N`` + ``N`` bytes of JSON +
  the raw tensor bytes; each JSON entry gives ``dtype``, ``shape`` and
  ``data_offsets = [begin, end)`` relative to the first byte after the
  header, so a tensor's absolute file offset is ``8 + N + begin``;
  the optional ``__metadata__`` entry is not a tensor;
* tensors are row-major, so row ``e`` of a stacked ``[E, ...]`` expert
  tensor is the contiguous range ``start + e * (bytes per row)``;
* an MLX affine-quantized matrix ``[out, in]`` is stored as ``weight``
  uint32 ``[out, in * bits / 32]`` plus ``scales`` / ``biases``
  ``[out, in / group_size]``; ``config.json``'s ``quantization`` object holds
  the default ``bits`` / ``group_size`` and, as nested objects keyed by module
  path, per-module overrides (mlx-vlm exports prefix paths with
  ``language_model.``, which is ignored when matching);
* an mlx-vlm export of a text-only model (every key of
  ``model.safetensors.index.json``'s ``weight_map`` starting with
  ``language_model.``) also names the router matrix ``….mlp.gate.proj.…``
  where mlx-lm has ``….mlp.gate.…``.  ``get`` / ``read_tensor`` resolve the
  mlx-lm name against such an export, the remap streamlx installs as a
  sanitize hook (streamlx/integrate.py:349-394, ``_vlm_export_shim``);
  native exports are untouched.

The public surface is the one streamlx's loader, reader and pool call
(streamlx/stindex.py:22-119): ``TensorLoc`` with ``row_stride`` /
``expert_range``; ``SafetensorsIndex(model_dir)`` with ``tensors``,
``switch_triples(layer)``, ``layer_expert_bytes(layer)`` and
``quant_params(triple)``; only shards named ``model-*.safetensors`` are
indexed (in name order, a later shard's entry replacing an earlier one's);
the exception types are ``FileNotFoundError`` (no shard), ``IndexError``
(expert row out of range), ``KeyError`` (a layer lacks one of its nine
stacked switch tensors) and ``ValueError`` (shapes that do not pack at the
configured bit width).  The byte ranges are checked against the reference's
own output by tests/golden.
"""

from __future__ import annotations

import fnmatch
import json
import os
import re
import struct
from dataclasses import dataclass

DTYPE_SIZE = {"U32": 4, "BF16": 2, "F16": 2, "F32": 4, "U16": 2, "U8": 1}
PROJS = ("gate_proj", "up_proj", "down_proj")
PARTS = ("weight", "scales", "biases")
SUPPORTED_BITS = frozenset((2, 3, 4, 5, 6, 8))
DEFAULT_GROUP = 64
_VLM_PREFIX = "language_model."
# "...layers.<L>.mlp.switch_mlp.<anything>" -- the stacked expert tensors
_SWITCH_RE = re.compile(r"layers\.(\d+)\.mlp\.switch_mlp\.(.+)$")


@dataclass(frozen=True)
class TensorLoc:
    """Where one tensor's bytes live: shard path, absolute file offset,
    byte count, safetensors dtype tag, shape, and its key."""
    path: str
    abs_start: int
    nbytes: int
    dtype: str
    shape: tuple
    name: str = ""

    @property
    def row_stride(self) -> int:
        """Bytes of one slice along the leading axis."""
        n = DTYPE_SIZE[self.dtype]
        for d in self.shape[1:]:
            n *= d
        return n

    def expert_range(self, e: int) -> tuple[str, int, int]:
        """(path, absolute offset, nbytes) of leading-axis row ``e``."""
        rows = self.shape[0]
        if not (0 <= e < rows):
            raise IndexError(f"row {e} outside 0..{rows - 1} of {self.name}")
        step = self.row_stride
        return self.path, self.abs_start + step * e, step


def parse_shard_header(path: str) -> list[TensorLoc]:
    """Every tensor entry of one shard, located in absolute file offsets."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: not a safetensors file")
        n = struct.unpack("<Q", head)[0]
        meta = json.loads(f.read(n))
    data0 = 8 + n
    locs = []
    for key, ent in meta.items():
        if key == "__metadata__":
            continue
        begin, end = ent["data_offsets"]
        locs.append(TensorLoc(path, data0 + begin, end - begin, ent["dtype"],
                              tuple(ent["shape"]), key))
    return locs


def _module_key(name: str) -> str:
    """Module path of a tensor key for quantization lookups."""
    if name.startswith(_VLM_PREFIX):
        name = name[len(_VLM_PREFIX):]
    if name.endswith(".weight"):
        name = name[:-len(".weight")]
    return name


def _mlx_lm_name(key: str) -> str:
    """mlx-lm's name for a tensor key of an mlx-vlm export."""
    return key[len(_VLM_PREFIX):].replace(".mlp.gate.proj.", ".mlp.gate.")


def vlm_aliases(model_dir: str, keys) -> dict[str, str]:
    """{mlx-lm name: stored key} when ``model_dir`` is an mlx-vlm export
    (its index's weight map non-empty and every key prefixed), else {}."""
    p = os.path.join(model_dir, "model.safetensors.index.json")
    if not os.path.exists(p):
        return {}
    with open(p) as f:
        wm = json.load(f).get("weight_map") or {}
    if not wm or not all(k.startswith(_VLM_PREFIX) for k in wm):
        return {}
    return {_mlx_lm_name(k): k for k in keys if k.startswith(_VLM_PREFIX)}


class QuantTable:
    """``config.json``'s quantization object: defaults plus per-module
    overrides (keys compared without the ``language_model.`` prefix)."""

    def __init__(self, table: dict | None):
        table = table or {}
        self.default_bits = None
        self.default_group = None
        self.modules: dict[str, dict] = {}
        for key, val in table.items():
            if isinstance(val, dict):
                mk = key[len(_VLM_PREFIX):] if key.startswith(_VLM_PREFIX) \
                    else key
                self.modules[mk] = val
            elif key == "bits":
                self.default_bits = val
            elif key == "group_size":
                self.default_group = val

    @classmethod
    def from_model_dir(cls, model_dir: str) -> "QuantTable":
        p = os.path.join(model_dir, "config.json")
        if not os.path.exists(p):
            return cls(None)
        with open(p) as f:
            return cls(json.load(f).get("quantization"))

    def lookup(self, tensor_name: str) -> tuple:
        """(bits or None, group size or None) for a weight tensor."""
        over = self.modules.get(_module_key(tensor_name), {})
        return (over.get("bits", self.default_bits),
                over.get("group_size", self.default_group))


class SafetensorsIndex:
    """Tensor name -> TensorLoc over the ``model-*.safetensors`` shards of a
    checkpoint directory, plus the per-layer stacked-expert view."""

    def __init__(self, model_dir: str):
        self.model_dir = str(model_dir)
        shards = sorted(f for f in os.listdir(self.model_dir)
                        if fnmatch.fnmatch(f, "model-*.safetensors")) \
            if os.path.isdir(self.model_dir) else []
        self.tensors: dict[str, TensorLoc] = {}
        for fn in shards:
            for loc in parse_shard_header(os.path.join(self.model_dir, fn)):
                self.tensors[loc.name] = loc
        if not self.tensors:
            raise FileNotFoundError(
                f"{self.model_dir}: no model-*.safetensors shard with tensors")
        self.quant = QuantTable.from_model_dir(self.model_dir)
        self.aliases = vlm_aliases(self.model_dir, self.tensors)
        # layer -> {(proj, part): TensorLoc}, in tensor order (a later key
        # with the same (proj, part) suffix replaces an earlier one)
        self._switch: dict[int, dict] = {}
        for key, loc in self.tensors.items():
            m = _SWITCH_RE.search(key)
            if m is None:
                continue
            tail = m.group(2)
            for proj in PROJS:
                for part in PARTS:
                    if tail.endswith(f"{proj}.{part}"):
                        self._switch.setdefault(int(m.group(1)), {})[
                            (proj, part)] = loc

    def switch_triples(self, layer: int) -> dict[str, dict[str, TensorLoc]]:
        """{proj: {part: TensorLoc}} of one layer's stacked expert tensors."""
        have = self._switch.get(int(layer), {})
        absent = [(proj, part) for proj in PROJS for part in PARTS
                  if (proj, part) not in have]
        if absent:
            raise KeyError(f"layer {layer} has no stacked expert tensor for "
                           f"{absent}")
        return {proj: {part: have[(proj, part)] for part in PARTS}
                for proj in PROJS}

    def layer_expert_bytes(self, layer: int) -> int:
        """Bytes of one expert of ``layer``: its row of all nine tensors."""
        tri = self.switch_triples(layer)
        return sum(tri[proj][part].row_stride for proj in PROJS
                   for part in PARTS)

    def quant_params(self, triple: dict[str, TensorLoc]
                     ) -> tuple[int, int, int, int]:
        """(in_features, out_features, bits, group_size) of one quantized
        projection: bits and group size from the quantization table (the
        module's override, else the default; group size 64 and bits inferred
        from the packed width when the table is silent), then checked
        against the stored shapes."""
        w, s = triple["weight"], triple["scales"]
        bits, group = self.quant.lookup(w.name)
        group = DEFAULT_GROUP if group is None else group
        words, groups = w.shape[-1], s.shape[-1]
        in_features = groups * group
        if bits is None:
            bits = (32 * words) // in_features if in_features else 0
        if bits not in SUPPORTED_BITS or 32 * words != bits * in_features:
            raise ValueError(
                f"{w.name}: weight {tuple(w.shape)} / scales "
                f"{tuple(s.shape)} do not pack {bits}-bit codes in groups "
                f"of {group}")
        return in_features, w.shape[1], bits, group

    def get(self, name: str) -> TensorLoc:
        """The tensor stored as ``name``, or under the mlx-vlm key that
        mlx-lm calls ``name``."""
        loc = self.tensors.get(name)
        if loc is None:
            alias = self.aliases.get(name)
            if alias is None:
                raise KeyError(name)
            loc = self.tensors[alias]
        return loc

    def read_tensor(self, name: str) -> bytes:
        """All bytes of one tensor (trunk weights; experts go through the
        reader)."""
        loc = self.get(name)
        buf = bytearray(loc.nbytes)
        view = memoryview(buf)
        done = 0
        with open(loc.path, "rb") as f:
            while done < loc.nbytes:
                n = os.preadv(f.fileno(), [view[done:]], loc.abs_start + done)
                if n <= 0:
                    raise IOError(f"{name}: read {done} of {loc.nbytes} bytes")
                done += n
        return bytes(buf)
