"""Synthetic MoE decoder that runs on the B200 kernels (the trunk around the
expert path).

The reference is an add-on to mlx-lm and brings no trunk of its own; the
workloads' decoders are Qwen3-MoE-shaped: per layer RMSNorm -> GQA
attention (q/k RMSNorm, rotate-half RoPE, KV cache) -> residual ->
RMSNorm -> router top-k -> SwitchGLU experts (+ optional shared expert) ->
residual; final RMSNorm and a quantized LM head, greedy argmax.  Every op is
one of the library's kernels (slx_*), inputs and positions live in device
memory.  ``layers[i].mlp.switch_mlp`` is the swappable SwitchGLU slot the
loader replaces with a pool-backed wrapper (streamlx/integrate.py:436-439).
"""

from __future__ import annotations

import json
import os

import numpy as np
import torch

from . import _lib as L
from . import ops
from .stindex import SafetensorsIndex
from .synth import SynthConfig


def _tensor(index: SafetensorsIndex, name: str, device) -> torch.Tensor:
    loc = index.get(name)
    raw = np.frombuffer(index.read_tensor(name), dtype=np.uint8)
    dt = {"U32": torch.int32, "BF16": torch.bfloat16, "F32": torch.float32,
          "F16": torch.float16}[loc.dtype]
    t = torch.from_numpy(raw.copy()).view(dt).reshape(loc.shape)
    return t.to(device)


def _qmat(index, prefix, device):
    return tuple(_tensor(index, f"{prefix}.{p}", device)
                 for p in ("weight", "scales", "biases"))


def _pack_dense(w3, out_f, in_f, bits, device) -> torch.Tensor:
    buf = torch.zeros(L.dense_tiled_bytes(out_f, in_f, bits), dtype=torch.uint8,
                      device=device)
    L.pack_dense(w3, out_f, in_f, bits, buf)
    return buf


class _Buf:
    """Per-layer device buffers reused every step."""


class MoEBlock:
    def __init__(self, layer: int, cfg: SynthConfig, index, device):
        self.layer = layer
        self.cfg = cfg
        self.device = device
        p = f"model.layers.{layer}.mlp"
        self.w_gate = _tensor(index, f"{p}.gate.weight", device).contiguous()
        self.bias = _tensor(index, f"{p}.gate.bias", device).contiguous()
        self.switch_mlp = None            # installed by the loader
        self.shared = None
        if cfg.shared_inter:
            H, Is, bits = cfg.hidden, cfg.shared_inter, cfg.trunk_bits
            trip = [_qmat(index, f"{p}.shared_expert.{n}", device)
                    for n in ("gate_proj", "up_proj", "down_proj")]
            buf = torch.zeros(L.slot_stride(H, Is, bits), dtype=torch.uint8,
                              device=device)
            L.pack_experts([tuple(trip)], H, Is, bits, [buf.data_ptr()])
            self.shared = (L.shared_struct(buf, Is), buf, Is)
        k, E = cfg.top_k, cfg.n_experts
        self.ids = torch.zeros(1, k, dtype=torch.int32, device=device)
        self.scores = torch.zeros(1, k, dtype=torch.float32, device=device)
        self.force = torch.zeros(1, dtype=torch.int32, device=device)
        self.scratch = torch.zeros(L.router_scratch_bytes(1, E),
                                   dtype=torch.uint8, device=device)
        # predictor (next layer's gate on this layer's input, rescaled)
        self.pf_ids = torch.zeros(1, k, dtype=torch.int32, device=device)
        self.pf_scores = torch.zeros(1, k, dtype=torch.float32, device=device)
        self.pf_scratch = torch.zeros(L.router_scratch_bytes(1, E),
                                      dtype=torch.uint8, device=device)

    def shared_struct(self):
        return self.shared

    def route(self, x2d, status, forced: bool = False):
        L.router_topk(x2d, self.w_gate, self.bias, self.cfg.top_k,
                      self.cfg.norm_topk_prob, self.ids, self.scores,
                      self.scratch, status,
                      force=self.force if forced else None,
                      forced_ids=self.ids if forced else None)
        return self.ids, self.scores


class DecoderLayer:
    def __init__(self, layer: int, cfg: SynthConfig, index, device):
        self.layer = layer
        H, hd, bits = cfg.hidden, cfg.head_dim, cfg.trunk_bits
        p = f"model.layers.{layer}"
        self.has_attn = cfg.has_trunk
        if self.has_attn:
            self.w_in = _tensor(index, f"{p}.input_layernorm.weight", device)
            self.post_attention_layernorm = _tensor(
                index, f"{p}.post_attention_layernorm.weight", device)
            q = _qmat(index, f"{p}.self_attn.q_proj", device)
            k = _qmat(index, f"{p}.self_attn.k_proj", device)
            v = _qmat(index, f"{p}.self_attn.v_proj", device)
            qkv = tuple(torch.cat([q[i], k[i], v[i]], 0).contiguous()
                        for i in range(3))
            self.n_qkv = (cfg.heads + 2 * cfg.kv_heads) * hd
            self.w_qkv = _pack_dense(qkv, self.n_qkv, H, bits, device)
            o = _qmat(index, f"{p}.self_attn.o_proj", device)
            self.w_o = _pack_dense(o, H, cfg.heads * hd, bits, device)
            self.q_norm = _tensor(index, f"{p}.self_attn.q_norm.weight", device)
            self.k_norm = _tensor(index, f"{p}.self_attn.k_norm.weight", device)
        self.mlp = MoEBlock(layer, cfg, index, device)


class SynthDecoder:
    """Batch-1 decoder over the library kernels."""

    def __init__(self, cfg: SynthConfig, index, device=None,
                 max_len: int = 1024):
        self.cfg = cfg
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        self.layers = [DecoderLayer(i, cfg, index, dev)
                       for i in range(cfg.layers)]
        H = cfg.hidden
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        if cfg.has_trunk:
            hd = cfg.head_dim
            self.embed = _qmat(index, "model.embed_tokens", dev)
            self.norm = _tensor(index, "model.norm.weight", dev)
            lm = _qmat(index, "lm_head", dev)
            self.w_lm = _pack_dense(lm, cfg.vocab, H, cfg.trunk_bits, dev)
            inv = (cfg.rope_theta ** (-2.0 * np.arange(hd // 2) / hd))
            self.inv_freq = torch.from_numpy(inv.astype(np.float32)).to(dev)
            self.max_len = max_len
            self.k_cache = [torch.zeros(max_len, cfg.kv_heads, hd,
                                        dtype=torch.bfloat16, device=dev)
                            for _ in range(cfg.layers)]
            self.v_cache = [torch.zeros_like(c) for c in self.k_cache]
            self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
            self.tok = torch.zeros(1, dtype=torch.int32, device=dev)
            self.h = torch.zeros(1, H, dtype=torch.bfloat16, device=dev)
            self.x = torch.zeros(1, H, dtype=torch.bfloat16, device=dev)
            self.qkv = torch.zeros(1, (cfg.heads + 2 * cfg.kv_heads) * hd,
                                   dtype=torch.bfloat16, device=dev)
            self.att = torch.zeros(1, cfg.heads * hd, dtype=torch.bfloat16,
                                   device=dev)
            self.o = torch.zeros(1, H, dtype=torch.bfloat16, device=dev)
            self.logits = torch.zeros(1, cfg.vocab, dtype=torch.bfloat16,
                                      device=dev)
        self.n_pos = 0
        # temporal-reuse routing override of the workloads: per (token,
        # layer) a seeded coin decides whether the previous token's expert
        # set is kept (applied identically to the CPU oracle)
        self.repeat_p = cfg.repeat_p
        self._rng = np.random.default_rng(12345)

    @classmethod
    def from_checkpoint(cls, model_dir: str, index=None, device=None,
                        max_len: int = 1024) -> "SynthDecoder":
        with open(os.path.join(model_dir, "config.json")) as f:
            cfg = SynthConfig(**json.load(f)["streamlx_synthetic"])
        index = index or SafetensorsIndex(model_dir)
        return cls(cfg, index, device=device, max_len=max_len)

    # ------------------------------------------------------ prefetch links --

    def link_prefetch(self, pools: dict) -> int:
        """Attention-window prefetch (streamlx/integrate.py:440-459): layer a
        predicts layer a+1's routing from its own MoE input rescaled by
        w_post(a+1) / w_post(a); adjacent streamed layers only."""
        linked = 0
        ordered = sorted(pools)
        for a, b in zip(ordered, ordered[1:]):
            if b != a + 1 or not self.cfg.has_trunk:
                continue
            la, lb = self.layers[a], self.layers[b]
            ratio = (lb.post_attention_layernorm.float() /
                     la.post_attention_layernorm.float()).to(torch.bfloat16)
            blk = la.mlp

            def predict(x, ratio=ratio.contiguous(), nxt=lb.mlp, blk=blk):
                x2d = ops.as_bf16_2d(x)
                L.router_topk(x2d, nxt.w_gate, nxt.bias, self.cfg.top_k,
                              self.cfg.norm_topk_prob, blk.pf_ids,
                              blk.pf_scores, blk.pf_scratch, self.status,
                              ratio=ratio)
                return (blk.pf_ids.cpu().numpy()[0],
                        blk.pf_scores.cpu().numpy()[0])

            la.mlp.switch_mlp._pf_next = (pools[b], predict)
            linked += 1
        return linked

    # -------------------------------------------------------------- decode --

    def reset(self) -> None:
        self.n_pos = 0
        self._rng = np.random.default_rng(12345)

    def _moe(self, layer: DecoderLayer, x2d: torch.Tensor) -> torch.Tensor:
        blk = layer.mlp
        forced = bool(self.repeat_p) and self.n_pos > 0 and \
            self._rng.random() < self.repeat_p
        if forced:
            blk.force.fill_(1)
        ids, scores = blk.route(x2d, self.status, forced=forced)
        return blk.switch_mlp.fused(x2d[None], scores[None], ids[None])[0]

    @torch.no_grad()
    def step(self, token: torch.Tensor) -> torch.Tensor:
        """One decode step for the token id in `token` (device int32 [1]);
        returns the greedy next token (device int32 [1])."""
        cfg = self.cfg
        if self.n_pos >= self.max_len:
            raise RuntimeError("KV cache full")
        self.pos.fill_(self.n_pos)
        L.dequant_rows(self.embed, cfg.hidden, cfg.trunk_bits, token, 1,
                       cfg.vocab, self.h, self.status)
        delta = None
        for i, layer in enumerate(self.layers):
            L.add_rmsnorm(self.h, delta, layer.w_in, cfg.rms_eps, self.x)
            L.qlinear(layer.w_qkv, layer.n_qkv, cfg.hidden, cfg.trunk_bits,
                      self.x, self.qkv, self.status)
            L.qk_norm_rope_cache(self.qkv, cfg.heads, cfg.kv_heads,
                                 cfg.head_dim, layer.q_norm, layer.k_norm,
                                 cfg.rms_eps, self.inv_freq, self.pos,
                                 self.k_cache[i], self.v_cache[i],
                                 self.status)
            L.attn_decode(self.qkv, cfg.heads, cfg.kv_heads, cfg.head_dim,
                          self.k_cache[i], self.v_cache[i], self.pos,
                          self.att)
            L.qlinear(layer.w_o, cfg.hidden, cfg.heads * cfg.head_dim,
                      cfg.trunk_bits, self.att, self.o, self.status)
            L.add_rmsnorm(self.h, self.o, layer.post_attention_layernorm,
                          cfg.rms_eps, self.x)
            delta = self._moe(layer, self.x)
        L.add_rmsnorm(self.h, delta, self.norm, cfg.rms_eps, self.x)
        L.qlinear(self.w_lm, cfg.vocab, cfg.hidden, cfg.trunk_bits, self.x,
                  self.logits, self.status)
        nxt = torch.empty(1, dtype=torch.int32, device=self.device)
        L.argmax(self.logits, nxt)
        self.n_pos += 1
        return nxt

    @torch.no_grad()
    def generate(self, prompt_ids, max_new: int) -> list[int]:
        """Token-by-token prompt feed, then greedy decode
        (examples/generate.py:67-89 of the reference)."""
        tok = None
        for pid in prompt_ids:
            tok = self.step(torch.tensor([int(pid)], dtype=torch.int32,
                                         device=self.device))
        out = []
        for _ in range(max_new):
            out.append(int(tok.item()))
            tok = self.step(tok)
        return out

    @torch.no_grad()
    def moe_forward(self, layer: int, x: torch.Tensor) -> torch.Tensor:
        """MoE block of one layer on hidden rows x [T, H] (router, experts,
        combine) -- the bare-MoE-layer workload."""
        x2d = ops.as_bf16_2d(x)
        blk = self.layers[layer].mlp
        T = x2d.shape[0]
        if T == 1:
            return self._moe(self.layers[layer], x2d)
        ids = torch.zeros(T, self.cfg.top_k, dtype=torch.int32,
                          device=self.device)
        scores = torch.zeros(T, self.cfg.top_k, dtype=torch.float32,
                             device=self.device)
        scr = torch.zeros(L.router_scratch_bytes(T, self.cfg.n_experts),
                          dtype=torch.uint8, device=self.device)
        L.router_topk(x2d, blk.w_gate, blk.bias, self.cfg.top_k,
                      self.cfg.norm_topk_prob, ids, scores, scr, self.status)
        return blk.switch_mlp.fused(x2d[None], scores[None], ids[None])[0]
