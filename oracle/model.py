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
    """All tensors of model-*.safetensors as read-only memory-mapped numpy
    arrays (uint32 codes, uint16 bf16 bits, float32)."""
    out = {}
    dt = {"U32": np.uint32, "BF16": np.uint16, "F32": np.float32}
    for shard in sorted(glob.glob(os.path.join(model_dir,
                                               "model-*.safetensors"))):
        with open(shard, "rb") as f:
            (hlen,) = struct.unpack("<Q", f.read(8))
            hdr = json.loads(f.read(hlen))
        base = 8 + hlen
        mm = np.memmap(shard, dtype=np.uint8, mode="r")
        for name, info in hdr.items():
            if name == "__metadata__":
                continue
            a, b = info["data_offsets"]
            out[name] = mm[base + a:base + b].view(
                dt[info["dtype"]]).reshape(info["shape"])
    return out


class OracleDecoder:
    """exact=True: fp64 accumulation (the parity reference); exact=False:
    fp32 BLAS accumulation like an fp32 CPU implementation would use (the
    timed CPU baseline)."""

    def __init__(self, model_dir: str, max_len: int = 256, exact: bool = True):
        self.exact = exact
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
        # smallest logit gap that decided each layer's routed / predicted
        # ids at the last step (how far an input perturbation must move a
        # logit to change the decision)
        self.route_margin = np.full(self.L, np.inf)
        self.pred_margin = np.full(self.L, np.inf)
        self.route_own = [None] * self.L
        self.own_margin = np.full(self.L, np.inf)
        self.route_scores = [None] * self.L

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
        """Dequantised expert (cached for small models only)."""
        key = (layer, e)
        hit = self._deq.get(key)
        if hit is not None:
            return hit
        p = f"model.layers.{layer}.mlp.switch_mlp"
        t = self.t
        d = {proj: A.dequant(t[f"{p}.{proj}.weight"][e],
                             t[f"{p}.{proj}.scales"][e],
                             t[f"{p}.{proj}.biases"][e], self.ebits, 64)
             for proj in ("gate_proj", "up_proj", "down_proj")}
        if self.cfg["n_experts"] * self.L <= 4096:
            self._deq[key] = d
        return d

    def embed_row(self, token: int) -> np.ndarray:
        t = self.t
        return A.dequant(t["model.embed_tokens.weight"][token],
                         t["model.embed_tokens.scales"][token],
                         t["model.embed_tokens.biases"][token], self.tbits,
                         64)[None]

    def mv(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        if self.exact:
            return A.qmv(x, w)
        return A.bf16_round(x.astype(np.float32) @ w.T)

    def expert_fwd(self, x: np.ndarray, d: dict) -> np.ndarray:
        if self.exact:
            return A.expert_forward(x, d)
        up = self.mv(x, d["up_proj"])
        gate = self.mv(x, d["gate_proj"])
        return self.mv(A.swiglu(gate, up), d["down_proj"])

    def qkv_weight(self, p: str) -> np.ndarray:
        key = p + ".qkv"
        if key not in self._deq:
            self._deq[key] = np.concatenate(
                [self.deq(f"{p}.self_attn.{n}_proj", self.tbits)
                 for n in ("q", "k", "v")], 0)
        return self._deq[key]

    def moe(self, layer: int, m: np.ndarray, forced_ids=None):
        """m [1, H] -> (combined [1, H], ids [k], scores [k])."""
        c = self.cfg
        p = f"model.layers.{layer}.mlp"
        ids, sc, lg = A.router(m, self.t[f"{p}.gate.weight"],
                               self.t[f"{p}.gate.bias"], c["top_k"],
                               c["norm_topk_prob"], forced_ids=forced_ids)
        self.route_margin[layer] = (A.topk_margin(lg[0], c["top_k"])
                                    if forced_ids is None else np.inf)
        # the router's own ordered pick and its margin even when the ids
        # are forced, and the combine weights used
        self.route_own[layer] = A.topk_ids(lg, c["top_k"])[0]
        self.own_margin[layer] = A.topk_margin(lg[0], c["top_k"])
        self.route_scores[layer] = sc[0]
        y = np.stack([self.expert_fwd(m, self.expert(layer, int(e)))[0]
                      for e in ids[0]])[None]
        sh = None
        if c["shared_inter"]:
            d = {proj: self.deq(f"{p}.shared_expert.{proj}", self.tbits)
                 for proj in ("gate_proj", "up_proj", "down_proj")}
            sh = self.expert_fwd(m, d)
        return A.moe_combine(y, sc, sh), ids[0], sc[0]

    def predict_next(self, layer: int, m: np.ndarray):
        """Next-layer routing prediction made at ``layer`` from its MoE input
        m [1, H] (streamlx/integrate.py:60-88): the next layer's gate on
        bf16(m * bf16(w_post(layer+1) / w_post(layer))).  Returns (ids [k],
        scores [k])."""
        c = self.cfg
        wa = self.bf(f"model.layers.{layer}.post_attention_layernorm.weight")
        wb = self.bf(f"model.layers.{layer + 1}.post_attention_layernorm"
                     ".weight")
        ratio = A.bf16_round(wb.astype(np.float32) / wa.astype(np.float32))
        xr = A.bf16_round(m.astype(np.float32) * ratio)
        p = f"model.layers.{layer + 1}.mlp"
        ids, sc, lg = A.router(xr, self.t[f"{p}.gate.weight"],
                               self.t[f"{p}.gate.bias"], c["top_k"],
                               c["norm_topk_prob"])
        self.pred_margin[layer] = A.topk_margin(lg[0], c["top_k"])
        return ids[0], sc[0]

    def step(self, token: int, forced: dict | None = None,
             predict: bool = False, n_layers: int | None = None):
        """One decode step; returns (logits [V], routed ids per layer), and
        with ``predict`` also the next-layer predictions [(ids, scores) or
        None per layer].  forced: {layer: ids} for the temporal-reuse
        routing override.  ``n_layers`` runs only the first layers before
        the final norm and head (a timing sample; logits then meaningless)."""
        c = self.cfg
        H, hd, nq, nkv = c["hidden"], c["head_dim"], c["heads"], c["kv_heads"]
        eps = c["rms_eps"]
        h = A.bf16_round(self.embed_row(token))
        delta = None
        routed = []
        preds: list = []
        for i in range(self.L if n_layers is None else min(n_layers, self.L)):
            p = f"model.layers.{i}"
            h, x = TR.add_rmsnorm(h, delta, self.bf(f"{p}.input_layernorm.weight"),
                                  eps)
            qkv = self.mv(x, self.qkv_weight(p))[0]
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
            o = self.mv(att, self.deq(f"{p}.self_attn.o_proj", self.tbits))
            h, m = TR.add_rmsnorm(h, o,
                                  self.bf(f"{p}.post_attention_layernorm.weight"),
                                  eps)
            fi = None if forced is None else forced.get(i)
            if predict:
                preds.append(self.predict_next(i, m) if i + 1 < self.L
                             else None)
            delta, ids, _ = self.moe(i, m, None if fi is None else fi[None])
            routed.append(ids)
        h, x = TR.add_rmsnorm(h, delta, self.bf("model.norm.weight"), eps)
        logits = self.mv(x, self.deq("lm_head", self.tbits))[0]
        self.pos += 1
        if predict:
            return logits, routed, preds
        return logits, routed
