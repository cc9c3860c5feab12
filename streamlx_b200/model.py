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
        self.pipeline = True
        self.pdl = True             # captured kernels chain with PDL
        self.glu_events = True      # time sampled SwitchGLU pairs in graphs
        self._graphs = None
        self._pending = None
        self._pf_done = 0
        self.glu_times: list | None = None
        # host seconds per phase of the graph-launched step (launch, the
        # previous step's deferred bookkeeping, waiting for the device log)
        self.host_times = {"launch": 0.0, "bookkeeping": 0.0, "wait": 0.0,
                           "miss_path": 0.0, "miss_replay": 0.0,
                           "miss_relaunch": 0.0, "miss_wait": 0.0,
                           "tail": 0.0, "steps": 0, "miss_steps": 0}
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
            la.mlp.pf_link = (ratio.contiguous(), lb.mlp)
            linked += 1
        self._graphs = None          # links changed: capture again
        return linked

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
        """One decode step for the token id in `token` (device int32 [1]);
        returns the greedy next token (device int32 [1]).

        With ``use_graphs`` the step runs as captured CUDA graphs and the
        pool bookkeeping follows from the device log (_step_graph); with
        ``pipeline`` the bookkeeping of a step that needed no slot fill is
        deferred to the next call (or flush()), where it overlaps that
        call's device work."""
        if self.use_graphs and all(
                hasattr(la.mlp.switch_mlp, "route") for la in self.layers):
            return self._step_graph(token)
        self.flush()
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
        ops.check_status(self.device)   # the kernels' device-side errors
        if int(self.status.item()) != 0:
            code = int(self.status.item())
            self.status.zero_()
            raise L.SlxError("device", code, "decode step device error")
        return nxt

    # ----------------------------------------------------- graph decode --
    #
    # A decode step runs as one CUDA graph per layer plus a tail graph, with
    # no host sync between layers.  The host then replays every layer's pool
    # bookkeeping from a device log (routed ids, next-layer prediction), in
    # layer order, through the wrapper's route() -- the same calls, in the
    # same order, as the eager path, so the hit/miss/eviction trace is the
    # same.  A layer computed correctly iff every routed expert had a slot
    # when its SwitchGLU ran (the kernel reads only routed experts, and a
    # resident expert never changes slot); otherwise the kernel reported
    # SLX_ERR_UNMAPPED_EXPERT for that layer, and after its replay has
    # filled the slots that layer and every later one run again.  Each
    # layer reads the previous layer's residual and MoE output from
    # per-layer buffers, so a rerun from layer l sees exactly its inputs.

    _UNMAPPED = -5

    def _graph_buffers(self) -> None:
        cfg, dev = self.cfg, self.device
        n, k, H = cfg.layers, cfg.top_k, cfg.hidden
        bf = torch.bfloat16
        self.g_s = torch.zeros(n, 1, H, dtype=bf, device=dev)
        self.g_m = torch.zeros(n, 1, H, dtype=bf, device=dev)
        self.g_d = torch.zeros(n, 1, H, dtype=bf, device=dev)
        self.g_xm = torch.zeros(n, 1, H, dtype=bf, device=dev)  # MoE input
        self.g_emb = torch.zeros(1, H, dtype=bf, device=dev)
        self.g_fin = torch.zeros(1, H, dtype=bf, device=dev)
        # device log, read back with one copy per launch cycle:
        # ids [n,k] | pred ids [n,k] | pred scores [n,k] f32 | layer status
        # [n] | status | next token
        words = 3 * n * k + n + 2
        self.g_log = torch.zeros(words, dtype=torch.int32, device=dev)
        self.g_log_host = torch.zeros(words, dtype=torch.int32).pin_memory()
        o = 0
        self.g_ids = self.g_log[o:o + n * k].view(n, 1, k)
        o += n * k
        self.g_pf_ids = self.g_log[o:o + n * k].view(n, 1, k)
        o += n * k
        self.g_pf_scores = self.g_log[o:o + n * k].view(torch.float32) \
            .view(n, 1, k)
        o += n * k
        self._lst_off = o
        self.g_lstatus = self.g_log[o:o + n]
        o += n
        self.g_status = self.g_log[o:o + 1]
        self.g_tok_out = self.g_log[o + 1:o + 2]
        self.g_scores = torch.zeros(n, 1, k, dtype=torch.float32, device=dev)
        self.g_prev_ids = torch.zeros(n, 1, k, dtype=torch.int32, device=dev)
        # control, written with one copy per step: pos | force[n] | token
        self.g_ctrl = torch.zeros(n + 2, dtype=torch.int32, device=dev)
        self.g_ctrl_host = torch.zeros(n + 2, dtype=torch.int32).pin_memory()
        sh = [la.mlp.switch_mlp.shared for la in self.layers]
        s_inter = max([x[2] for x in sh if x] or [0])
        self.g_glu_scratch = torch.zeros(
            L.switchglu_scratch_bytes(1, k, cfg.inter, s_inter),
            dtype=torch.uint8, device=dev)
        self._side = torch.cuda.Stream(device=dev)   # predictor branch
        self.g_ev = [(torch.cuda.Event(enable_timing=True),
                      torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for pair in self.g_ev:      # torch creates the CUDA event on first use
            for e in pair:
                e.record()

    def _record_layer(self, i: int, join: bool = True) -> None:
        cfg = self.cfg
        n, k, H, bits = cfg.layers, cfg.top_k, cfg.hidden, cfg.trunk_bits
        la = self.layers[i]
        blk = la.mlp
        w = blk.switch_mlp
        eps = cfg.rms_eps
        if i == 0:
            L.dequant_rows(self.embed, H, bits, self.g_ctrl[n + 1:n + 2], 1,
                           cfg.vocab, self.g_emb, self.g_status)
            h_in, d_in = self.g_emb, None
        else:
            h_in, d_in = self.g_m[i - 1], self.g_d[i - 1]
        L.add_rmsnorm_out(h_in, d_in, la.w_in, eps, self.g_s[i], self.x)
        L.qlinear(la.w_qkv, la.n_qkv, H, bits, self.x, self.qkv,
                  self.g_status)
        L.qk_norm_rope_cache(self.qkv, cfg.heads, cfg.kv_heads, cfg.head_dim,
                             la.q_norm, la.k_norm, eps, self.inv_freq,
                             self.g_ctrl[0:1], self.k_cache[i],
                             self.v_cache[i], self.g_status)
        L.attn_decode(self.qkv, cfg.heads, cfg.kv_heads, cfg.head_dim,
                      self.k_cache[i], self.v_cache[i], self.g_ctrl[0:1],
                      self.att)
        L.qlinear(la.w_o, H, cfg.heads * cfg.head_dim, bits, self.att,
                  self.o, self.g_status)
        xm = self.g_xm[i]
        L.add_rmsnorm_out(self.g_s[i], self.o, la.post_attention_layernorm,
                          eps, self.g_m[i], xm)
        L.router_topk_multi(
            xm, [L.router_head(blk.w_gate, blk.bias, self.g_ids[i],
                               self.g_scores[i], blk.scratch,
                               force=self.g_ctrl[1 + i:2 + i],
                               forced_ids=self.g_prev_ids[i])],
            cfg.n_experts, k, cfg.norm_topk_prob, self.g_status)
        if blk.pf_link is not None:
            # the next-layer predictor only feeds the host's prefetch: it
            # runs on a side branch, off the layer's critical path
            ratio, nxt = blk.pf_link
            cur = torch.cuda.current_stream(self.device)
            self._side.wait_stream(cur)
            self._forked = True
            prev = L.set_pdl(False)
            try:
                with torch.cuda.stream(self._side):
                    L.router_topk_multi(
                        xm, [L.router_head(nxt.w_gate, nxt.bias,
                                           self.g_pf_ids[i],
                                           self.g_pf_scores[i],
                                           blk.pf_scratch, ratio=ratio)],
                        cfg.n_experts, k, cfg.norm_topk_prob, self.g_status)
            finally:
                L.set_pdl(prev)
        pool = w.pool
        sh = w.shared
        ev = self.g_ev[i]
        timed = self._glu_timed(i)
        if timed:
            L.event_record_external(ev[0])
        ops.switchglu(pool.store.bank, xm, self.g_ids[i], k,
                      scores=self.g_scores[i], table=pool.store.table_dev,
                      shared=sh[0] if sh else None, out=self.g_d[i],
                      inter=pool.inter, shared_inter=sh[2] if sh else 0,
                      scratch_buf=self.g_glu_scratch,
                      status=self.g_lstatus[i:i + 1])
        if timed:
            L.event_record_external(ev[1])
        if join:
            self._join_side()

    def _join_side(self) -> None:
        """Rejoin the predictor branch (only if this recording forked it:
        a capture may not wait on work from outside itself)."""
        if getattr(self, "_forked", False):
            torch.cuda.current_stream(self.device).wait_stream(self._side)
            self._forked = False

    def _record_tail(self) -> None:
        cfg = self.cfg
        n = cfg.layers
        L.add_rmsnorm_out(self.g_m[n - 1], self.g_d[n - 1], self.norm,
                          cfg.rms_eps, self.g_fin, self.x)
        L.qlinear(self.w_lm, cfg.vocab, cfg.hidden, cfg.trunk_bits, self.x,
                  self.logits, self.g_status)
        L.argmax(self.logits, self.g_tok_out)
        # a plain async copy (no allocator event) so it captures as a node
        L.copy_many([self.g_log_host.data_ptr()], [self.g_log.data_ptr()],
                    [self.g_log.numel() * 4])

    def _capture(self) -> None:
        """Capture the per-layer graphs, the tail graph and one graph of the
        whole step (used when a step starts at layer 0)."""
        if not hasattr(self, "g_log"):
            self._graph_buffers()
        n = self.cfg.layers
        # the initialising pass below really runs: point it at the position
        # the next step overwrites anyway, not forced, token 0
        ch = self.g_ctrl_host.numpy()
        ch[:] = 0
        ch[0] = min(self.n_pos, self.max_len - 1)
        L.copy_many([self.g_ctrl.data_ptr()], [self.g_ctrl_host.data_ptr()],
                    [self.g_ctrl.numel() * 4])
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        # one eager pass on the side stream initialises every launcher
        # (function attributes, lazy module loads) outside the capture
        with torch.cuda.stream(s):
            for i in range(n):
                self._record_layer(i)
            self._record_tail()
        s.synchronize()
        mode = "thread_local"
        prev_pdl = L.set_pdl(self.pdl)
        try:
            graphs, tail, full = self._capture_graphs(s, mode)
        finally:
            L.set_pdl(prev_pdl)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self._graphs = (graphs, tail, full)
        self.g_status.zero_()
        self.g_lstatus.zero_()

    def _capture_graphs(self, s, mode):
        """Capture the graphs; the library kernels each one launches are
        counted while it is recorded (launch accounting of replays)."""
        n = self.cfg.layers
        graphs = []
        self._kernels_layer = []
        for i in range(n):
            g = torch.cuda.CUDAGraph()
            c0 = L.LAUNCHES[0]
            with torch.cuda.graph(g, stream=s, capture_error_mode=mode):
                self._record_layer(i)
            self._kernels_layer.append(L.LAUNCHES[0] - c0)
            graphs.append(g)
        tail = torch.cuda.CUDAGraph()
        c0 = L.LAUNCHES[0]
        with torch.cuda.graph(tail, stream=s, capture_error_mode=mode):
            self._record_tail()
        self._kernels_tail = L.LAUNCHES[0] - c0
        full = torch.cuda.CUDAGraph()
        c0 = L.LAUNCHES[0]
        with torch.cuda.graph(full, stream=s, capture_error_mode=mode):
            self.g_lstatus.zero_()
            for i in range(n):
                self._record_layer(i, join=False)
            self._join_side()
            self._record_tail()
        self._kernels_full = L.LAUNCHES[0] - c0
        # suffix graphs: layers i..n-1 and the tail as one launch, for the
        # re-run after a slot fill (one graph launch instead of n - i + 1)
        self._suffix = [None] * n
        self._kernels_suffix = [0] * n
        for i in range(1, n):
            g = torch.cuda.CUDAGraph()
            c0 = L.LAUNCHES[0]
            with torch.cuda.graph(g, stream=s, capture_error_mode=mode):
                self.g_lstatus[i:].zero_()
                for j in range(i, n):
                    self._record_layer(j, join=False)
                self._join_side()
                self._record_tail()
            self._kernels_suffix[i] = L.LAUNCHES[0] - c0
            self._suffix[i] = g
        return graphs, tail, full

    def _graph_kernels(self, start: int) -> int:
        """Library kernels one launch from layer `start` runs."""
        if start == 0:
            return self._kernels_full
        return self._kernels_suffix[start]

    def _launch(self, start: int) -> None:
        graphs, tail, full = self._graphs
        if start == 0:
            full.replay()
        else:
            self._suffix[start].replay()
        L._count(self._graph_kernels(start))

    def _read_log(self) -> np.ndarray:
        torch.cuda.current_stream(self.device).synchronize()
        log = self.g_log_host.numpy().copy()
        st = int(log[self._lst_off + self.cfg.layers])
        if st != 0:
            self.g_status.zero_()
            raise L.SlxError("device", st, "decode step device error")
        return log

    def _glu_timed(self, i: int) -> bool:
        """Layers whose SwitchGLU pair is bracketed by timing events: one in
        eight (an event node costs a few microseconds of the step)."""
        return self.glu_events and i % 8 == 3

    def _glu_timing(self, start: int) -> None:
        if self.glu_times is None or not self.glu_events:
            return
        ev = [self.g_ev[i] for i in range(start, self.cfg.layers)
              if self._glu_timed(i)]
        if not ev:
            return
        self.glu_times.extend(
            L.event_elapsed_many([e[0] for e in ev], [e[1] for e in ev])
            .tolist())

    def _prefetch_upto(self, log: np.ndarray) -> None:
        """Start the next-layer prefetches of this step's layers whose logged
        prediction is final (every layer up to and including the first
        unmapped one), in layer order.  Layer i's prefetch touches only pool
        i+1, and nothing changes pool i+1 between the previous step's call of
        layer i+1 (already replayed) and this step's, so starting them here,
        before this step's bookkeeping, gives the reference's per-pool order
        while the reads overlap the bookkeeping and the next step."""
        n, k = self.cfg.layers, self.cfg.top_k
        lst = log[self._lst_off:self._lst_off + n]
        bad = np.flatnonzero(lst == self._UNMAPPED)
        upto = n if bad.size == 0 else int(bad[0]) + 1
        pf_ids = log[n * k:2 * n * k].reshape(n, k)
        pf_sc = log[2 * n * k:3 * n * k].view(np.float32).reshape(n, k)
        for i in range(self._pf_done, upto):
            w = self.layers[i].mlp.switch_mlp
            if self.layers[i].mlp.pf_link is not None and w.pred_gate():
                w.start_prefetch((pf_ids[i].copy(), pf_sc[i].copy()))
        self._pf_done = max(self._pf_done, upto)

    def _replay(self, log: np.ndarray, start: int) -> int | None:
        """Pool bookkeeping of layers start.. from a log; returns the first
        layer that must run again (its slots are now filled) or None.  The
        layers' prefetches were started by _prefetch_upto."""
        n, k = self.cfg.layers, self.cfg.top_k
        ids = log[:n * k].reshape(n, 1, 1, k)
        lst = log[self._lst_off:self._lst_off + n]
        for i in range(start, n):
            code = int(lst[i])
            if code not in (0, self._UNMAPPED):
                raise L.SlxError("device", code, f"layer {i} SwitchGLU")
            w = self.layers[i].mlp.switch_mlp
            if w.route(ids[i].copy(), None, start_prefetch=False) != "pool":
                raise RuntimeError("decode call routed more experts than "
                                   "the pool has slots")
            w.pool.sync_device()
            if code == self._UNMAPPED:
                return i
        return None

    def flush(self) -> None:
        """Finish the deferred bookkeeping of the last step, if any: start
        its next-layer prefetches not yet started, then replay its pool
        calls from the first layer not yet replayed."""
        pend, self._pending = self._pending, None
        if pend is None:
            return
        log, start, pf_done = pend
        self._pf_done = pf_done
        self._prefetch_upto(log)
        if self._replay(log, start) is not None:
            raise RuntimeError("deferred step had an unmapped expert")

    def _step_graph(self, token: torch.Tensor) -> torch.Tensor:
        n = self.cfg.layers
        if self.n_pos >= self.max_len:
            raise RuntimeError("KV cache full")
        if self._graphs is None:
            self.flush()
            self._capture()
        ch = self.g_ctrl_host.numpy()
        ch[0] = self.n_pos
        for i in range(n):
            ch[1 + i] = int(bool(self.repeat_p) and self.n_pos > 0 and
                            self._rng.random() < self.repeat_p)
        tok = token.reshape(1)
        if tok.dtype != torch.int32 or tok.device != self.device:
            tok = tok.to(device=self.device, dtype=torch.int32)
        L.copy_many([self.g_ctrl.data_ptr(), self.g_ctrl.data_ptr() + 4 * (n + 1)],
                    [self.g_ctrl_host.data_ptr(), tok.data_ptr()],
                    [4 * (n + 1), 4])
        # this step's device work is queued before the host replays the
        # previous step: that replay's slot fills and table pushes run after
        # it on the stream, and this step is judged by its own log
        ht = self.host_times
        t0 = time.perf_counter()
        self._launch(0)
        t1 = time.perf_counter()
        self.flush()
        t2 = time.perf_counter()
        log = self._read_log()
        t3 = time.perf_counter()
        ht["launch"] += t1 - t0
        ht["bookkeeping"] += t2 - t1
        ht["wait"] += t3 - t2
        ht["steps"] += 1
        self._glu_timing(0)
        lst = log[self._lst_off:self._lst_off + n]
        t4 = time.perf_counter()
        if self.pipeline and not (lst == self._UNMAPPED).any():
            # bookkeeping (and the prefetch reads it starts) waits for the
            # next call, where it overlaps that step's device work
            self._pending = (log, 0, 0)
        else:
            self._pf_done = 0
            self._prefetch_upto(log)
            start = 0
            while True:
                r0 = time.perf_counter()
                redo = self._replay(log, start)
                r1 = time.perf_counter()
                ht["miss_replay"] += r1 - r0
                if redo is None:
                    break
                self._launch(redo)
                r2 = time.perf_counter()
                log = self._read_log()
                ht["miss_relaunch"] += r2 - r1
                ht["miss_wait"] += time.perf_counter() - r2
                self._glu_timing(redo)
                self._prefetch_upto(log)
                if int(log[self._lst_off + redo]) != 0:
                    raise RuntimeError(f"layer {redo} still unmapped after "
                                       "its slots were filled")
                start = redo + 1
                rest = log[self._lst_off + start:self._lst_off + n]
                if self.pipeline and not (rest == self._UNMAPPED).any():
                    # the layers after the refilled one all ran on resident
                    # experts: their bookkeeping waits for the next call,
                    # like a miss-free step's
                    self._pending = (log, start, self._pf_done)
                    break
            ht["miss_path"] += time.perf_counter() - t4
            ht["miss_steps"] += 1
        t5 = time.perf_counter()
        self.g_prev_ids.copy_(self.g_ids)
        self.n_pos += 1
        nxt = torch.empty(1, dtype=torch.int32, device=self.device)
        nxt.copy_(self.g_tok_out)
        ht["tail"] += time.perf_counter() - t5
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
