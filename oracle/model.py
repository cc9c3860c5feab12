"""ORACLE — test infrastructure only; never imported by the product path.

numpy restatement of one batch-1 decode step of the synthetic MoE decoders
(the same computation the library runs on the GPU), reading the safetensors
checkpoint directly.  Built from oracle/affine.py (expert path: router,
gather_qmm, SwiGLU, combine -- streamlx/pool.py:30-50 plus the mlx-lm block
around it) and oracle/trunk.py (RMSNorm, RoPE, attention).
"""

from __future__ import annotations

import glob
import json
import os
import struct

import numpy as np

from . import affine as A
from . import trunk as TR


def read_checkpoint(model_dir: str) -> dict:
    """All tensors of model-*.safetensors as numpy arrays (uint32 codes,
    uint16 bf16 bits, float32)."""
    out = {}
    dt = {"U32": np.uint32, "BF16": np.uint16, "F32": np.float32}
    for shard in sorted(glob.glob(os.path.join(model_dir,
                                               "model-*.safetensors"))):
        with open(shard, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            hdr = json.loads(f.read(hlen))
            base = 8 + hlen
            for name, info in hdr.items():
                if name == "__metadata__":
                    continue
                a, b = info["data_offsets"]
                f.seek(base + a)
                out[name] = np.frombuffer(f.read(b - a),
                                          dtype=dt[info["dtype"]]).reshape(
                                              info["shape"])
    return out


class OracleDecoder:
    def __init__(self, model_dir: str, max_len: int = 256):
        with open(os.path.join(model_dir, "config.json")) as f:
            self.cfg = json.load(f)["streamlx_synthetic"]
        c = self.cfg
        self.t = read_checkpoint(model_dir)
        self.ebits, self.tbits = c["expert_bits"], c["trunk_bits"]
        self.L = c["layers"]
        self.kc = [np.zeros((max_len, c["kv_heads"], c["head_dim"]), np.float32)
                   for _ in range(self.L)]
        self.vc = [np.zeros_like(k) for k in self.kc]
        self.inv = TR.rope_inv_freq(c["head_dim"], c["rope_theta"])
        self._deq: dict = {}
        self.pos = 0

    def deq(self, prefix: str, bits: int) -> np.ndarray:
        if prefix not in self._deq:
            t = self.t
            self._deq[prefix] = A.dequant(t[prefix + ".weight"],
                                          t[prefix + ".scales"],
                                          t[prefix + ".biases"], bits, 64)
        return self._deq[prefix]

    def bf(self, name: str) -> np.ndarray:
        return A.bf16_from_bits(self.t[name])

    def expert(self, layer: int, e: int) -> dict:
        key = (layer, e)
        if key not in self._deq:
            p = f"model.layers.{layer}.mlp.switch_mlp"
            t = self.t
            self._deq[key] = {
                proj: A.dequant(t[f"{p}.{proj}.weight"][e],
                                t[f"{p}.{proj}.scales"][e],
                                t[f"{p}.{proj}.biases"][e], self.ebits, 64)
                for proj in ("gate_proj", "up_proj", "down_proj")}
        return self._deq[key]

    def moe(self, layer: int, m: np.ndarray, forced_ids=None):
        """m [1, H] -> (combined [1, H], ids [k], scores [k])."""
        c = self.cfg
        p = f"model.layers.{layer}.mlp"
        ids, sc, _ = A.router(m, self.t[f"{p}.gate.weight"],
                              self.t[f"{p}.gate.bias"], c["top_k"],
                              c["norm_topk_prob"], forced_ids=forced_ids)
        y = np.stack([A.expert_forward(m, self.expert(layer, int(e)))[0]
                      for e in ids[0]])[None]
        sh = None
        if c["shared_inter"]:
            d = {proj: self.deq(f"{p}.shared_expert.{proj}", self.tbits)
                 for proj in ("gate_proj", "up_proj", "down_proj")}
            sh = A.expert_forward(m, d)
        return A.moe_combine(y, sc, sh), ids[0], sc[0]

    def step(self, token: int, forced: dict | None = None):
        """One decode step; returns (logits [V], routed ids per layer).
        forced: {layer: ids} for the temporal-reuse routing override."""
        c = self.cfg
        H, hd, nq, nkv = c["hidden"], c["head_dim"], c["heads"], c["kv_heads"]
        eps = c["rms_eps"]
        h = A.bf16_round(self.deq("model.embed_tokens", self.tbits)[token][None])
        delta = None
        routed = []
        for i in range(self.L):
            p = f"model.layers.{i}"
            h, x = TR.add_rmsnorm(h, delta, self.bf(f"{p}.input_layernorm.weight"),
                                  eps)
            wq = np.concatenate([self.deq(f"{p}.self_attn.{n}_proj", self.tbits)
                                 for n in ("q", "k", "v")], 0)
            qkv = A.qmv(x, wq)[0]
            q = qkv[:nq * hd].reshape(nq, hd)
            k = qkv[nq * hd:(nq + nkv) * hd].reshape(nkv, hd)
            v = qkv[(nq + nkv) * hd:].reshape(nkv, hd)
            qn = self.bf(f"{p}.self_attn.q_norm.weight")
            kn = self.bf(f"{p}.self_attn.k_norm.weight")
            qr = np.stack([TR.qk_norm_rope(q[j], qn, eps, self.pos, self.inv)
                           for j in range(nq)])
            self.kc[i][self.pos] = np.stack(
                [TR.qk_norm_rope(k[j], kn, eps, self.pos, self.inv)
                 for j in range(nkv)])
            self.vc[i][self.pos] = v
            att = TR.attn_decode(qr, self.kc[i], self.vc[i], self.pos + 1, nq,
                                 nkv).reshape(1, -1)
            o = A.qmv(att, self.deq(f"{p}.self_attn.o_proj", self.tbits))
            h, m = TR.add_rmsnorm(h, o,
                                  self.bf(f"{p}.post_attention_layernorm.weight"),
                                  eps)
            fi = None if forced is None else forced.get(i)
            delta, ids, _ = self.moe(i, m, None if fi is None else fi[None])
            routed.append(ids)
        h, x = TR.add_rmsnorm(h, delta, self.bf("model.norm.weight"), eps)
        logits = A.qmv(x, self.deq("lm_head", self.tbits))[0]
        self.pos += 1
        return logits, routed
