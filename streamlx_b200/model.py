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

import time

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
        self.pf_link = None         # (ratio, next layer's MoEBlock)

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
        self.use_graphs = cfg.has_trunk
        self.pdl = True             # captured kernels chain with PDL
        # time sampled SwitchGLU launches with event pairs in the step graph
        # (a measurement aid: the event nodes cost the step a few us)
        self.glu_events = False
        self._graphs = None
        self.glu_times: list | None = None
        # host seconds per phase of the graph-launched step (launch, the
        # previous step's deferred bookkeeping, waiting for the device log)
        self.host_times = {"launch": 0.0, "serve": 0.0, "bookkeeping": 0.0,
                           "park_serve": 0.0, "flush": 0.0, "steps": 0,
                           "parks": 0, "park_steps": 0}
        self._step_active = False
        self.ep = None              # EpExchange when experts are sharded
        # layers whose pool holds every expert for good (fully resident):
        # their launch needs no slot fill and the host no bookkeeping
        self.static_glu = [False] * cfg.layers
        # with every layer static, launch a step's graph before checking the
        # previous one (its device errors are raised one step late)
        self.overlap_steps = True
        self._inflight = None       # log buffer of an unchecked step
        self._all_pooled = None     # cached layer-set facts, set on first use
        self._store_list = None
        self._pf_layers = None
        # temporal-reuse routing override of the workloads: per (token,
        # layer) a seeded coin decides whether the previous token's expert
        # set is kept (applied identically to the CPU oracle)
        self.repeat_p = cfg.repeat_p
        self._rng = np.random.default_rng(12345)

    @classmethod
    def from_checkpoint(cls, model_dir: str, index=None, device=None,
                        max_len: int = 2048) -> "SynthDecoder":
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
            la.mlp.pf_link = (ratio.contiguous(), lb.mlp)
            linked += 1
        self._graphs = None          # links changed: capture again
        return linked

    def enable_expert_parallel(self, group=None, wait_s: float = 10.0):
        """Shard the experts over the ranks of a process group: this rank's
        pools hold only its experts, and each decode step exchanges the
        owned experts' output rows over NVLink peer memory
        (expert_parallel.EpExchange).  Graph decode only."""
        from .expert_parallel import EpExchange
        self.ep = EpExchange(self.cfg.layers, self.cfg.top_k, self.cfg.hidden,
                             self.device, group=group, wait_s=wait_s)
        self.use_graphs = True
        self._graphs = None
        return self.ep

    # -------------------------------------------------------------- decode --

    def reset(self) -> None:
        self.flush()
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
        """One decode step for the token id in `token` (int32 [1], on the
        device or in host memory); returns the greedy next token (device
        int32 [1]).

        With ``use_graphs`` the step runs as one captured CUDA graph whose
        layers report their routing to the host as they run; the host keeps
        the pool bookkeeping in step and serves layers that park on a miss
        (_step_graph).  Otherwise the step runs layer by layer with one host
        sync on the routed ids per layer (_step_eager)."""
        if self.ep is not None or (self.use_graphs and self._pooled()):
            return self._step_graph(token)
        self.flush()
        if token.device != self.device or token.dtype != torch.int32:
            token = token.to(device=self.device, dtype=torch.int32)
        return self._step_eager(token)

    @torch.no_grad()
    def _step_eager(self, token: torch.Tensor) -> torch.Tensor:
        """Layer by layer, one host sync on the routed ids per layer."""
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
            L.attn_rope_decode(self.qkv, cfg.heads, cfg.kv_heads,
                               cfg.head_dim, layer.q_norm, layer.k_norm,
                               cfg.rms_eps, self.inv_freq, self.pos,
                               self.k_cache[i], self.v_cache[i], self.att,
                               self.status)
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
        ops.check_status(self.device)   # the kernels' device-side errors
        if int(self.status.item()) != 0:
            code = int(self.status.item())
            self.status.zero_()
            raise L.SlxError("device", code, "decode step device error")
        return nxt

    # ----------------------------------------------------- graph decode --
    #
    # A decode step is one CUDA graph of every layer plus the tail.  Each
    # layer's SwitchGLU launch (slx_switchglu_serviced) first reports the
    # layer's routed ids and its next-layer prediction through host-mapped
    # memory; if one of its routed experts has no slot it parks until the
    # host has served it (fill_service.py).  The host follows the records in
    # layer order while the step runs: it starts each layer's next-layer
    # prefetch, replays the layer's pool bookkeeping through the wrapper's
    # route() -- the same calls, in the same order, as the eager path, so the
    # hit/miss/eviction trace is the reference's -- and serves parked layers
    # with their slot fills.  Fills of layers that did not park (the device
    # already computed them with slots that were still valid) are recorded
    # and applied between steps.  A layer is computed correctly because its
    # kernel only reads slots whose table entry and bytes were installed
    # together (between steps, or by the kernel itself after a park).

    WAIT_S = 30.0       # bound of a parked layer's wait for its service

    def _graph_buffers(self) -> None:
        from .fill_service import FillService
        cfg, dev = self.cfg, self.device
        n, k, H = cfg.layers, cfg.top_k, cfg.hidden
        if k > L.FILL_MAX_K:
            raise ValueError(f"top_k {k} > {L.FILL_MAX_K}: graph decode "
                             "needs the eager path")
        bf = torch.bfloat16
        self.g_s = torch.zeros(n, 1, H, dtype=bf, device=dev)
        self.g_m = torch.zeros(n, 1, H, dtype=bf, device=dev)
        self.g_d = torch.zeros(n, 1, H, dtype=bf, device=dev)
        self.g_xm = torch.zeros(n, 1, H, dtype=bf, device=dev)  # MoE input
        self.g_emb = torch.zeros(1, H, dtype=bf, device=dev)
        self.g_fin = torch.zeros(1, H, dtype=bf, device=dev)
        self.g_ids = torch.zeros(n, 1, k, dtype=torch.int32, device=dev)
        self.g_pf_ids = torch.zeros(n, 1, k, dtype=torch.int32, device=dev)
        self.g_pf_scores = torch.zeros(n, 1, k, dtype=torch.float32,
                                       device=dev)
        # device log read back once per step: layer status [n] | status |
        # next token
        self.g_log = torch.zeros(n + 2, dtype=torch.int32, device=dev)
        # host copies of the log and of the control words alternate between
        # two buffers, so a step can be launched while the previous one's
        # copies are still pending (overlapped steps)
        self._log_host = [torch.zeros(n + 2, dtype=torch.int32).pin_memory()
                          for _ in range(2)]
        self.g_log_host = self._log_host[0]
        self.g_lstatus = self.g_log[0:n]
        self.g_status = self.g_log[n:n + 1]
        self.g_tok_out = self.g_log[n + 1:n + 2]
        self.g_scores = torch.zeros(n, 1, k, dtype=torch.float32, device=dev)
        self.g_prev_ids = torch.zeros(n, 1, k, dtype=torch.int32, device=dev)
        # control, written with one copy per step:
        # pos | force[n] | token | stamp
        self.g_ctrl = torch.zeros(n + 3, dtype=torch.int32, device=dev)
        self._ctrl_host = [torch.zeros(n + 3, dtype=torch.int32).pin_memory()
                           for _ in range(2)]
        self.g_ctrl_host = self._ctrl_host[0]
        sh = [la.mlp.switch_mlp.shared for la in self.layers]
        s_inter = max([x[2] for x in sh if x] or [0])
        self.g_glu_scratch = torch.zeros(
            L.switchglu_scratch_bytes(1, k, cfg.inter, s_inter),
            dtype=torch.uint8, device=dev)
        pools = [la.mlp.switch_mlp.pool for la in self.layers]
        max_slots = max(p.n_slots for p in pools)
        topm = max(p._PF_TOPM for p in pools)
        # a parked layer receives its pool's fills since the last step: its
        # own misses and prefetch adoptions (bounded by the pool size)
        max_items = min(max_slots, max(4 * (k + topm), 32))
        stride = max(p.store.stride for p in pools)
        staging = min(max_items * stride * 2, 2 << 30)
        self.svc = FillService(n, cfg.n_experts, max_items, staging, dev,
                               wait_s=self.WAIT_S)
        self._stamp = 0
        self.g_ev = [(torch.cuda.Event(enable_timing=True),
                      torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for pair in self.g_ev:      # torch creates the CUDA event on first use
            for e in pair:
                e.record()
        self._ev_step = [torch.cuda.Event(), torch.cuda.Event()]
        self._ev_done = self._ev_step[0]

    def _pred_on(self, i: int) -> bool:
        """Layer i computes the next-layer prediction in its router launch:
        it has a prefetch link and the next pool's agreement gate is open
        (the reference stops predicting below 55% agreement,
        streamlx/integrate.py:76-77)."""
        blk = self.layers[i].mlp
        return blk.pf_link is not None and blk.switch_mlp.pred_gate()

    def _record_layer(self, i: int, serviced: bool = True) -> None:
        cfg = self.cfg
        n, k, H, bits = cfg.layers, cfg.top_k, cfg.hidden, cfg.trunk_bits
        la = self.layers[i]
        blk = la.mlp
        w = blk.switch_mlp
        eps = cfg.rms_eps
        stamp = self.g_ctrl.data_ptr() + 4 * (n + 2)
        if i == 0:
            L.dequant_rows(self.embed, H, bits, self.g_ctrl[n + 1:n + 2], 1,
                           cfg.vocab, self.g_emb, self.g_status)
            L.add_rmsnorm_out(self.g_emb, None, la.w_in, eps, self.g_s[i],
                              self.x)
        elif self.ep is not None:
            # the previous layer's experts, combined from every rank's rows
            L.ep_combine_rmsnorm(
                self.ep.struct(i - 1, stamp, warmup=not serviced),
                self.g_scores[i - 1], k, H,
                self.layers[i - 1].mlp.switch_mlp.shared is not None,
                self.g_m[i - 1], la.w_in, eps, self.g_s[i], self.x,
                self.g_status)
        else:
            L.add_rmsnorm_out(self.g_m[i - 1], self.g_d[i - 1], la.w_in, eps,
                              self.g_s[i], self.x)
        L.qlinear(la.w_qkv, la.n_qkv, H, bits, self.x, self.qkv,
                  self.g_status)
        L.attn_rope_decode(self.qkv, cfg.heads, cfg.kv_heads, cfg.head_dim,
                           la.q_norm, la.k_norm, eps, self.inv_freq,
                           self.g_ctrl[0:1], self.k_cache[i], self.v_cache[i],
                           self.att, self.g_status)
        L.qlinear(la.w_o, H, cfg.heads * cfg.head_dim, bits, self.att,
                  self.o, self.g_status)
        xm = self.g_xm[i]
        heads = [L.router_head(blk.w_gate, blk.bias, self.g_ids[i],
                               self.g_scores[i], blk.scratch,
                               force=self.g_ctrl[1 + i:2 + i],
                               forced_ids=self.g_prev_ids[i])]
        pred = self._pred_on(i)
        if pred:
            # the next-layer predictor shares the router launch (same input)
            ratio, nxt = blk.pf_link
            heads.append(L.router_head(nxt.w_gate, nxt.bias,
                                       self.g_pf_ids[i], self.g_pf_scores[i],
                                       blk.pf_scratch, ratio=ratio))
        # the post-attention residual add + RMSNorm runs inside the router
        # launch (g_m[i] = g_s[i] + o, xm = the MoE input)
        L.router_topk_multi_norm(heads, self.g_s[i], self.o,
                                 la.post_attention_layernorm, eps,
                                 self.g_m[i], xm, cfg.n_experts, k,
                                 cfg.norm_topk_prob, self.g_status)
        pool = w.pool
        sh = w.shared
        ev = self.g_ev[i]
        timed = self._glu_timed(i)
        if timed:
            L.event_record_external(ev[0])
        if serviced and self.ep is not None:
            L.switchglu_ep(pool.store.bank, xm, self.g_ids[i],
                           self.g_scores[i], pool.store.table_dev,
                           self.g_glu_scratch, self.g_lstatus[i:i + 1],
                           self.ep.struct(i, stamp),
                           shared=sh[0] if sh else None)
        elif serviced:
            svc = self.svc.svc(i, stamp,
                               self.g_pf_ids[i] if pred else None,
                               self.g_pf_scores[i] if pred else None)
            L.switchglu_serviced(pool.store.bank, xm, self.g_ids[i],
                                 self.g_scores[i], pool.store.table_dev,
                                 self.g_d[i], self.g_glu_scratch,
                                 self.g_lstatus[i:i + 1], svc,
                                 shared=sh[0] if sh else None)
        else:
            ops.switchglu(pool.store.bank, xm, self.g_ids[i], k,
                          scores=self.g_scores[i], table=pool.store.table_dev,
                          shared=sh[0] if sh else None, out=self.g_d[i],
                          inter=pool.inter, shared_inter=sh[2] if sh else 0,
                          scratch_buf=self.g_glu_scratch,
                          status=self.g_lstatus[i:i + 1])
        if timed:
            L.event_record_external(ev[1])

    def _record_tail(self, serviced: bool = True) -> None:
        cfg = self.cfg
        n = cfg.layers
        if self.ep is not None:
            stamp = self.g_ctrl.data_ptr() + 4 * (n + 2)
            L.ep_combine_rmsnorm(
                self.ep.struct(n - 1, stamp, warmup=not serviced),
                self.g_scores[n - 1], cfg.top_k, cfg.hidden,
                self.layers[n - 1].mlp.switch_mlp.shared is not None,
                self.g_m[n - 1], self.norm, cfg.rms_eps, self.g_fin, self.x,
                self.g_status)
        else:
            L.add_rmsnorm_out(self.g_m[n - 1], self.g_d[n - 1], self.norm,
                              cfg.rms_eps, self.g_fin, self.x)
        L.qlinear(self.w_lm, cfg.vocab, cfg.hidden, cfg.trunk_bits, self.x,
                  self.logits, self.g_status)
        L.argmax(self.logits, self.g_tok_out)
        # a plain async copy (no allocator event) so it captures as a node:
        # the step's ids become the next step's reuse candidates (not in the
        # capture's initialising pass, which must not replace them)
        if serviced:
            L.copy_many([self.g_prev_ids.data_ptr()], [self.g_ids.data_ptr()],
                        [self.g_ids.numel() * 4])

    def _capture(self) -> None:
        """Capture the graph of one whole step."""
        if not hasattr(self, "g_log"):
            self._graph_buffers()
        self.flush()
        n = self.cfg.layers
        # the initialising pass below really runs (without the slot fill):
        # point it at the position the next step overwrites anyway, not
        # forced, token 0
        ch = self.g_ctrl_host.numpy()
        ch[:] = 0
        ch[0] = min(self.n_pos, self.max_len - 1)
        L.copy_many([self.g_ctrl.data_ptr()], [self.g_ctrl_host.data_ptr()],
                    [self.g_ctrl.numel() * 4])
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        prev_pdl = L.set_pdl(self.pdl)
        try:
            # one eager pass on the side stream initialises every launcher
            # (function attributes, lazy module loads, the launch-attribute
            # choices) outside the capture
            with torch.cuda.stream(s):
                for i in range(n):
                    self._record_layer(i, serviced=False)
                self._record_tail(serviced=False)
            s.synchronize()
            self._pred_flags = [self._pred_on(i) for i in range(n)]
            self._pf_layers = [i for i in range(n)
                               if self.layers[i].mlp.pf_link is not None]
            self._store_list = None
            full = torch.cuda.CUDAGraph()
            c0 = L.LAUNCHES[0]
            with torch.cuda.graph(full, stream=s,
                                  capture_error_mode="thread_local"):
                self.g_lstatus.zero_()
                for i in range(n):
                    self._record_layer(i, serviced=not self.static_glu[i]
                                       or self.ep is not None)
                self._record_tail()
            self._kernels_full = L.LAUNCHES[0] - c0
        finally:
            L.set_pdl(prev_pdl)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self._graphs = full
        self.g_status.zero_()
        self.g_lstatus.zero_()
        self.svc.reset_words()

    def _glu_timed(self, i: int) -> bool:
        """Layers whose SwitchGLU launch is bracketed by timing events: one in
        eight (an event node costs a few microseconds of the step)."""
        return self.glu_events and i % 8 == 3

    def _glu_timing(self) -> None:
        if self.glu_times is None or not self.glu_events:
            return
        ev = [self.g_ev[i] for i in range(self.cfg.layers)
              if self._glu_timed(i)]
        if ev:
            self.glu_times.extend(
                L.event_elapsed_many([e[0] for e in ev], [e[1] for e in ev])
                .tolist())

    def _pooled(self) -> bool:
        """Every layer's SwitchGLU is pool-backed (the graph step's
        condition; the layers are fixed once the loader returns)."""
        if self._all_pooled is None:
            self._all_pooled = all(hasattr(la.mlp.switch_mlp, "route")
                                   for la in self.layers)
        return self._all_pooled

    def _stores(self):
        """Pools whose fills a step may defer: the static layers' pools
        never fill."""
        if self._store_list is None:
            self._store_list = [
                la.mlp.switch_mlp.pool for i, la in enumerate(self.layers)
                if not self.static_glu[i]
                and hasattr(la.mlp.switch_mlp, "pool")
                and hasattr(la.mlp.switch_mlp.pool.store, "deferred")]
        return self._store_list

    def flush(self) -> None:
        """Apply every recorded slot fill and table push now (on the current
        stream); nothing of a decode step is left pending after it."""
        if self._step_active:
            return
        self._drain()
        stream = torch.cuda.current_stream(self.device)
        for pool in self._stores():
            if pool.store.has_pending():
                pool.store.flush_pending(pool.slot_table, stream)

    def _on_record(self, i: int, rec: np.ndarray) -> None:
        """Host side of layer i's record: start the next layer's prefetch
        from the prediction (gate checked as the reference does), then the
        pool bookkeeping of the call."""
        k = self.cfg.top_k
        w = self.layers[i].mlp.switch_mlp
        if self._pred_flags[i] and w.pred_gate():
            w.start_prefetch((rec[20:20 + k].copy(),
                              rec[36:36 + k].view(np.float32).copy()))
        ids = rec[4:4 + k].astype(np.int64).reshape(1, 1, k)
        if w.route(ids, None, start_prefetch=False) != "pool":
            raise RuntimeError("decode call routed more experts than the "
                               "pool has slots")
        w.pool.sync_device()

    def _serve_step(self, stamp: int) -> None:
        """Follow the running step's layer records and serve parked layers
        until the step's graph has completed."""
        n = self.cfg.layers
        svc = self.svc
        log = svc.log
        ht = self.host_times
        nxt = 0
        idle = 0
        while True:
            busy = False
            while nxt < n and (self.static_glu[nxt] or
                               int(log[nxt, 0]) == stamp):
                if not self.static_glu[nxt]:    # static layers write none
                    t0 = time.perf_counter()
                    self._on_record(nxt, log[nxt].copy())
                    ht["bookkeeping"] += time.perf_counter() - t0
                nxt += 1
                busy = True
            pk = svc.pending_park(stamp)
            if pk is not None and pk[0] < nxt:
                t0 = time.perf_counter()
                layer, ticket = pk
                svc.serve(layer, ticket, self.layers[layer].mlp.switch_mlp.pool)
                ht["park_serve"] += time.perf_counter() - t0
                ht["parks"] += 1
                busy = True
            if busy:
                idle = 0
                continue
            if nxt == n and self._ev_done.query():
                break
            idle += 1
            if idle > 64:
                time.sleep(0)       # let the prefetch thread run
            if idle > 64 and self._ev_done.query() and nxt < n:
                # the graph finished: every record it wrote is visible
                if int(log[nxt, 0]) != stamp:
                    raise RuntimeError(f"decode step ended without layer "
                                       f"{nxt}'s record")

    def _overlapped(self) -> bool:
        """Steps are launched before the previous one is checked: every
        layer static (no slot service, no bookkeeping; the expert-parallel
        form is, its exchange is ordered on the device by the step stamp)
        and no per-step timing events."""
        return (self.overlap_steps and not self.glu_events and
                (self.ep is not None or all(self.static_glu)))

    def _check_log(self, b: int) -> None:
        """Raise the device errors a step's log (host copy b) reports."""
        n = self.cfg.layers
        log = self._log_host[b].numpy()
        st = int(log[n])
        bad = [int(v) for v in log[:n] if int(v) != 0]
        if st != 0 or bad:
            self.g_status.zero_()
            self.g_lstatus.zero_()
            raise L.SlxError("device", st or bad[0], "decode step device error")

    def _drain(self) -> None:
        """Wait for an overlapped step still unchecked and check it."""
        prev, self._inflight = self._inflight, None
        if prev is not None:
            self._ev_step[prev].synchronize()
            self._check_log(prev)

    def sync(self) -> None:
        """Finish every launched step: with overlapped steps a step's device
        errors are raised by the next step, or here."""
        self._drain()
        torch.cuda.current_stream(self.device).synchronize()

    def _abort_step(self, stamp: int) -> None:
        """After a host-side failure: release any parked layer without
        fills, let the step finish and put the stores back in direct mode."""
        t_end = time.perf_counter() + self.WAIT_S + 5
        while not self._ev_done.query() and time.perf_counter() < t_end:
            pk = self.svc.pending_park(stamp)
            if pk is not None:
                self.svc.abort(pk[1])
            time.sleep(1e-4)
        torch.cuda.current_stream(self.device).synchronize()
        self.svc.stream.synchronize()
        for pool in self._stores():
            pool.store.deferred = False

    def _step_graph(self, token: torch.Tensor) -> torch.Tensor:
        n = self.cfg.layers
        if self.n_pos >= self.max_len:
            raise RuntimeError("KV cache full")
        if self._graphs is not None and any(
                self._pred_flags[i] != self._pred_on(i)
                for i in self._pf_layers):
            self._graphs = None     # a prediction gate closed: recapture
        if self._graphs is None:
            self._capture()
        self._stamp += 1
        stamp = self._stamp & 0x7FFFFF
        if stamp == 0:
            self._stamp += 1
            stamp = 1
        b = stamp & 1
        ctrl = self._ctrl_host[b]   # its copy two steps ago has run
        ch = ctrl.numpy()
        ch[0] = self.n_pos
        if self.repeat_p and self.n_pos > 0:
            # one draw per layer, in layer order (the eager path's sequence)
            ch[1:1 + n] = self._rng.random(n) < self.repeat_p
        else:
            ch[1:1 + n] = 0
        ch[n + 2] = stamp
        tok = token.reshape(1)
        cur = torch.cuda.current_stream(self.device)
        if tok.device.type == "cpu":
            # a host token travels with the control words: one copy
            ch[n + 1] = int(tok[0])
            L.copy_many([self.g_ctrl.data_ptr()], [ctrl.data_ptr()],
                        [4 * (n + 3)])
        else:
            if tok.dtype != torch.int32 or tok.device != self.device:
                tok = tok.to(device=self.device, dtype=torch.int32)
            L.copy_many([self.g_ctrl.data_ptr(),
                         self.g_ctrl.data_ptr() + 4 * (n + 1),
                         self.g_ctrl.data_ptr() + 4 * (n + 2)],
                        [ctrl.data_ptr(), tok.data_ptr(),
                         ctrl.data_ptr() + 4 * (n + 2)],
                        [4 * (n + 1), 4, 4])
        ht = self.host_times
        t0 = time.perf_counter()
        for pool in self._stores():
            pool.store.deferred = True
        self._step_active = True
        self._graphs.replay()
        L._count(self._kernels_full)
        L.copy_many([self._log_host[b].data_ptr()], [self.g_log.data_ptr()],
                    [self.g_log.numel() * 4])
        self._ev_done = self._ev_step[b]
        self._ev_done.record(cur)
        t1 = time.perf_counter()
        if self._overlapped():
            # nothing for the host to serve: check the previous step (long
            # finished or about to) while this one runs
            self._step_active = False
            prev, self._inflight = self._inflight, b
            if prev is not None:
                self._ev_step[prev].synchronize()
                try:
                    self._check_log(prev)
                except L.SlxError:
                    # the step just launched ran on the same (sticky) status
                    # words: its log goes with the error
                    self._inflight = None
                    raise
            ht["launch"] += t1 - t0
            ht["serve"] += time.perf_counter() - t1
            ht["steps"] += 1
            self.n_pos += 1
            nxt = torch.empty(1, dtype=torch.int32, device=self.device)
            nxt.copy_(self.g_tok_out)
            return nxt
        self._drain()
        parks0 = ht["parks"]
        try:
            if self.ep is not None or all(self.static_glu):
                self._ev_done.synchronize()     # resident experts: no service
            else:
                self._serve_step(stamp)
        except BaseException:
            self._step_active = False
            self._abort_step(stamp)
            raise
        t2 = time.perf_counter()
        self._step_active = False
        for pool in self._stores():
            pool.store.deferred = False
        self.flush()                 # fills of layers that did not park
        t3 = time.perf_counter()
        ht["launch"] += t1 - t0
        ht["serve"] += t2 - t1
        ht["flush"] += t3 - t2
        ht["steps"] += 1
        ht["park_steps"] += int(ht["parks"] > parks0)
        self._check_log(b)
        self._glu_timing()
        self.n_pos += 1
        nxt = torch.empty(1, dtype=torch.int32, device=self.device)
        nxt.copy_(self.g_tok_out)
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
        self.flush()
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
