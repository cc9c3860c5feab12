"""Test helper: rewrite a checkpoint directory the way mlx-vlm exports a
text-only model -- every tensor key and every per-module quantization key
prefixed with ``language_model.``, the router matrix named
``….mlp.gate.proj.…`` -- plus the ``model.safetensors.index.json`` weight map
those exports carry.  Tensor bytes are copied unchanged."""

from __future__ import annotations

import json
import os
import shutil
import struct

PREFIX = "language_model."


def vlm_key(key: str) -> str:
    return PREFIX + key.replace(".mlp.gate.", ".mlp.gate.proj.")


def write_vlm_copy(src: str, dst: str) -> str:
    os.makedirs(dst, exist_ok=True)
    weight_map = {}
    for fn in sorted(os.listdir(src)):
        p = os.path.join(src, fn)
        if fn.endswith(".safetensors"):
            with open(p, "rb") as f:
                n = struct.unpack("<Q", f.read(8))[0]
                meta = json.loads(f.read(n))
                new = {}
                for k, v in meta.items():
                    if k == "__metadata__":
                        new[k] = v
                    else:
                        new[vlm_key(k)] = v
                        weight_map[vlm_key(k)] = fn
                head = json.dumps(new).encode()
                head += b" " * (-len(head) % 8)
                with open(os.path.join(dst, fn), "wb") as g:
                    g.write(struct.pack("<Q", len(head)))
                    g.write(head)
                    shutil.copyfileobj(f, g, 1 << 24)
        elif fn == "config.json":
            with open(p) as f:
                cfg = json.load(f)
            q = cfg.get("quantization") or {}
            cfg["quantization"] = {(PREFIX + k if isinstance(v, dict) else k): v
                                   for k, v in q.items()}
            with open(os.path.join(dst, fn), "w") as f:
                json.dump(cfg, f)
        elif os.path.isfile(p):
            shutil.copy(p, os.path.join(dst, fn))
    with open(os.path.join(dst, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)
    return dst
