"""Seeded synthetic checkpoints in the MLX quantized MoE layout.

No real checkpoint is available, so every workload runs on a model written
here from a seed.  The on-disk format is the one the reference reads
(streamlx/stindex.py:43-71, 77-119):

* shards named ``model-XXXXX-of-YYYYY.safetensors`` (8-byte little-endian
  header length, JSON header, raw data);
* stacked expert tensors ``model.layers.{L}.mlp.switch_mlp.{gate,up,down}_proj
  .{weight,scales,biases}`` with shapes ``[E, out, in*bits/32]`` (U32) and
  ``[E, out, in/group_size]`` (BF16);
* ``config.json`` with a ``quantization`` table (top-level bits/group_size and
  per-path overrides, e.g. 2-bit experts under a 4-bit trunk).

Quantisation is MLX "affine": per group of ``group_size`` input columns,
``w ~= scale * q + bias`` with ``q`` packed low-bits-first into uint32 words.
The quantiser below is the plain min/max affine scheme (``scale = (max-min) /
(2^bits-1)``, ``bias = min``); only the dequantisation semantics matter to the
expert path, and those are fixed by the format.

Generation runs in torch on any device (``device="cuda"`` makes the 18-30 GB
benchmark models in seconds); the files are the same format either way.
"""

from __future__ import annotations

import json
import math
import os
import struct
from dataclasses import asdict, dataclass, field

import numpy as np
import torch

__all__ = ["SynthConfig", "PRESETS", "quantize_affine", "write_model",
           "zipf_bias", "expert_bytes"]


@dataclass
class SynthConfig:
    """Shape of a synthetic MoE decoder (or a bare MoE layer stack)."""
    name: str = "tiny"
    hidden: int = 256
    layers: int = 2
    n_experts: int = 16
    top_k: int = 4
    inter: int = 128                 # routed expert intermediate size
    shared_inter: int = 0            # 0: no shared expert
    expert_bits: int = 4
    trunk_bits: int = 4
    group_size: int = 64
    # trunk (attention decoder); heads == 0 means "MoE layers only"
    heads: int = 0
    kv_heads: int = 0
    head_dim: int = 128
    vocab: int = 0
    rope_theta: float = 1_000_000.0
    rms_eps: float = 1e-6
    norm_topk_prob: bool = True
    zipf_s: float = 1.0              # router logit bias: popularity ~ 1/(rank+1)^s
    repeat_p: float = 0.0            # harness-side routing override (temporal reuse)
    weight_std: float = 0.02
    # "normal": N(0, weight_std) weights quantized with the min/max affine
    # scheme; "codes": the routed experts' codes, scales and biases drawn
    # directly (numpy, identical on every machine, ~1 GB/s) with the
    # statistics of quantized N(0, weight_std) groups -- for the large
    # 2-bit models, whose expert bytes dominate the checkpoint
    expert_init: str = "normal"
    extra: dict = field(default_factory=dict)

    @property
    def has_trunk(self) -> bool:
        return self.heads > 0

    def to_hf(self) -> dict:
        """config.json contents (mlx-lm style keys + quantization table)."""
        quant = {"group_size": self.group_size, "bits": self.trunk_bits}
        for L in range(self.layers):
            for p in ("gate_proj", "up_proj", "down_proj"):
                quant[f"model.layers.{L}.mlp.switch_mlp.{p}"] = {
                    "group_size": self.group_size, "bits": self.expert_bits}
        return {
            "model_type": "streamlx_synthetic_moe",
            "hidden_size": self.hidden,
            "num_hidden_layers": self.layers,
            "num_attention_heads": self.heads,
            "num_key_value_heads": self.kv_heads,
            "head_dim": self.head_dim,
            "vocab_size": self.vocab,
            "num_experts": self.n_experts,
            "num_experts_per_tok": self.top_k,
            "moe_intermediate_size": self.inter,
            "shared_expert_intermediate_size": self.shared_inter,
            "norm_topk_prob": self.norm_topk_prob,
            "rms_norm_eps": self.rms_eps,
            "rope_theta": self.rope_theta,
            "quantization": quant,
            "streamlx_synthetic": asdict(self),
        }


# Workload presets.  "moe_c1" is the single MoE layer the reference can run on
# its CPU path; "qwen3moe_c2" and "laguna_c3" are full decoders.
PRESETS: dict[str, SynthConfig] = {
    "moe_c1": SynthConfig(name="moe_c1", hidden=1024, layers=1, n_experts=32,
                          top_k=4, inter=512, expert_bits=4, zipf_s=1.0),
    "qwen3moe_c2": SynthConfig(name="qwen3moe_c2", hidden=2048, layers=40,
                               n_experts=256, top_k=8, inter=512,
                               shared_inter=512, expert_bits=4, trunk_bits=4,
                               heads=16, kv_heads=2, head_dim=128,
                               vocab=151936, zipf_s=1.0),
    "laguna_c3": SynthConfig(name="laguna_c3", hidden=2560, layers=48,
                             n_experts=256, top_k=10, inter=1024,
                             expert_bits=2, trunk_bits=4, heads=24,
                             kv_heads=4, head_dim=128, vocab=151936,
                             zipf_s=1.1, repeat_p=0.6),
    # the 117B-shaped decoder cut to 4 layers and a 4096-token vocabulary
    # (expert shapes, top-k, routing statistics unchanged): trace tests
    "laguna_c3_4l": SynthConfig(name="laguna_c3_4l", hidden=2560, layers=4,
                                n_experts=256, top_k=10, inter=1024,
                                expert_bits=2, trunk_bits=4, heads=24,
                                kv_heads=4, head_dim=128, vocab=4096,
                                zipf_s=1.1, repeat_p=0.6,
                                expert_init="codes"),
    # small decoders for parity tests
    "tiny_dec": SynthConfig(name="tiny_dec", hidden=512, layers=3,
                            n_experts=16, top_k=4, inter=512, shared_inter=512,
                            expert_bits=4, trunk_bits=4, heads=4, kv_heads=2,
                            head_dim=128, vocab=1024, zipf_s=1.0),
    "tiny_dec2": SynthConfig(name="tiny_dec2", hidden=512, layers=3,
                             n_experts=16, top_k=4, inter=512,
                             expert_bits=2, trunk_bits=4, heads=4, kv_heads=2,
                             head_dim=128, vocab=1024, zipf_s=1.1,
                             repeat_p=0.6),
}


def random_codes(rng: np.random.Generator, lead: tuple, out: int, inp: int,
                 bits: int, gs: int, std: float):
    """Quantized weights drawn directly: uniform codes, and per group a
    scale ~ (range of gs N(0, std) samples) / (2^bits - 1) and a bias near
    -(2^bits - 1) / 2 * scale, so s*q + b is centred with the spread of the
    quantized normal weights.  Returns (int32 words [..., out, inp*bits/32],
    bf16 scales, bf16 biases) as numpy arrays (bf16 as uint16 bits)."""
    import ml_dtypes
    shape = (*lead, out, inp * bits // 32)
    n = int(np.prod(shape))
    words = rng.bit_generator.random_raw((n + 1) // 2).view(np.int32)[:n] \
        .reshape(shape)
    g = inp // gs
    nb = (1 << bits) - 1
    spread = 2.0 * std * np.sqrt(2.0 * np.log(gs))      # ~ max - min
    scale = (spread / nb) * (0.85 + 0.3 * rng.random((*lead, out, g),
                                                    dtype=np.float32))
    bias = -0.5 * nb * scale * (0.9 + 0.2 * rng.random((*lead, out, g),
                                                     dtype=np.float32))
    s16 = scale.astype(ml_dtypes.bfloat16).view(np.uint16)
    b16 = bias.astype(ml_dtypes.bfloat16).view(np.uint16)
    return words, s16, b16


def expert_bytes(hidden: int, inter: int, bits: int, gs: int) -> int:
    """Bytes of one expert (gate+up+down, packed weights + bf16 scales/biases)."""
    def proj(inp, out):
        return out * inp * bits // 8 + 2 * 2 * out * (inp // gs)
    return 2 * proj(hidden, inter) + proj(inter, hidden)


def zipf_bias(n_experts: int, s: float, seed: int) -> np.ndarray:
    """Per-expert router logit bias log(p_e) with p_e ~ 1/(rank_e+1)^s over a
    seeded permutation of expert ids (fp32)."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(n_experts)
    rank = np.empty(n_experts, dtype=np.int64)
    rank[perm] = np.arange(n_experts)
    p = 1.0 / np.power(rank + 1.0, s)
    p /= p.sum()
    return np.log(p).astype(np.float32)


@torch.no_grad()
def quantize_affine(w: torch.Tensor, bits: int, gs: int):
    """Affine-quantise ``w[..., in]`` (float) along its last axis.

    Returns (packed int32 view of uint32 words [..., in*bits/32],
    scales bf16 [..., in/gs], biases bf16 [..., in/gs]).
    """
    if bits not in (2, 4, 8):
        raise ValueError(f"bits={bits}: the synthetic writer packs 2/4/8-bit")
    *lead, n = w.shape
    if n % gs or (n * bits) % 32:
        raise ValueError(f"in_features {n} not divisible by group {gs}")
    g = w.float().reshape(*lead, n // gs, gs)
    wmin = g.amin(-1)
    wmax = g.amax(-1)
    nb = (1 << bits) - 1
    scale = ((wmax - wmin) / nb).clamp_min(1e-8)
    s_bf = scale.to(torch.bfloat16)
    b_bf = wmin.to(torch.bfloat16)
    q = torch.round((g - b_bf.float()[..., None]) / s_bf.float()[..., None])
    q = q.clamp_(0, nb).to(torch.int64)
    per = 32 // bits
    q = q.reshape(*lead, n // per, per)
    shifts = (torch.arange(per, device=w.device, dtype=torch.int64) * bits)
    packed = (q << shifts).sum(-1)
    packed = torch.where(packed >= 2**31, packed - 2**32, packed)
    return packed.to(torch.int32), s_bf, b_bf


class _ShardWriter:
    """Streams tensors into one safetensors file whose layout is fixed up
    front (so the header can be written before any data is generated)."""

    _DT = {"U32": 4, "BF16": 2, "F32": 4, "F16": 2, "U16": 2, "U8": 1}

    def __init__(self, path: str, specs: list[tuple[str, str, tuple]]):
        self.path = path
        hdr = {}
        off = 0
        self.order = []
        for name, dt, shape in specs:
            n = int(np.prod(shape)) * self._DT[dt]
            hdr[name] = {"dtype": dt, "shape": list(shape),
                         "data_offsets": [off, off + n]}
            self.order.append((name, n))
            off += n
        hdr["__metadata__"] = {"format": "mlx"}
        raw = json.dumps(hdr, separators=(",", ":")).encode()
        # pad so tensor data starts 256-byte aligned in the file (safetensors
        # allows trailing spaces in the header)
        raw += b" " * ((-(len(raw) + 8)) % 256)
        self.f = open(path, "wb")
        self.f.write(struct.pack("<Q", len(raw)))
        self.f.write(raw)
        self.i = 0

    def put(self, name: str, t: torch.Tensor | np.ndarray) -> None:
        want, n = self.order[self.i]
        if want != name:
            raise RuntimeError(f"shard writer: expected {want}, got {name}")
        if isinstance(t, torch.Tensor):
            t = t.detach().contiguous()
            if t.dtype == torch.bfloat16:
                t = t.view(torch.int16)
            arr = t.cpu().numpy()
        else:
            arr = np.ascontiguousarray(t)
        if arr.nbytes != n:
            raise RuntimeError(f"{name}: {arr.nbytes} bytes, header says {n}")
        self.f.write(memoryview(arr.reshape(-1)).cast("B"))
        self.i += 1

    def close(self) -> None:
        if self.i != len(self.order):
            raise RuntimeError(f"{self.path}: wrote {self.i}/{len(self.order)}")
        self.f.close()


def _qspecs(prefix: str, out: int, inp: int, bits: int, gs: int, lead=()):
    return [(f"{prefix}.weight", "U32", (*lead, out, inp * bits // 32)),
            (f"{prefix}.scales", "BF16", (*lead, out, inp // gs)),
            (f"{prefix}.biases", "BF16", (*lead, out, inp // gs))]


def _layer_specs(cfg: SynthConfig, L: int):
    H, E, I, gs = cfg.hidden, cfg.n_experts, cfg.inter, cfg.group_size
    p = f"model.layers.{L}"
    sp = []
    if cfg.has_trunk:
        hd = cfg.head_dim
        sp += [(f"{p}.input_layernorm.weight", "BF16", (H,)),
               (f"{p}.post_attention_layernorm.weight", "BF16", (H,))]
        for nm, o, i in (("q_proj", cfg.heads * hd, H),
                         ("k_proj", cfg.kv_heads * hd, H),
                         ("v_proj", cfg.kv_heads * hd, H),
                         ("o_proj", H, cfg.heads * hd)):
            sp += _qspecs(f"{p}.self_attn.{nm}", o, i, cfg.trunk_bits, gs)
        sp += [(f"{p}.self_attn.q_norm.weight", "BF16", (hd,)),
               (f"{p}.self_attn.k_norm.weight", "BF16", (hd,))]
    sp += [(f"{p}.mlp.gate.weight", "BF16", (E, H)),
           (f"{p}.mlp.gate.bias", "F32", (E,))]
    for nm, o, i in (("gate_proj", I, H), ("up_proj", I, H),
                     ("down_proj", H, I)):
        sp += _qspecs(f"{p}.mlp.switch_mlp.{nm}", o, i, cfg.expert_bits, gs,
                      lead=(E,))
    if cfg.shared_inter:
        Is = cfg.shared_inter
        for nm, o, i in (("gate_proj", Is, H), ("up_proj", Is, H),
                         ("down_proj", H, Is)):
            sp += _qspecs(f"{p}.mlp.shared_expert.{nm}", o, i,
                          cfg.trunk_bits, gs)
    return sp


def write_model(out_dir: str, cfg: SynthConfig, seed: int = 0,
                device: str = "cpu", layers_per_shard: int = 8) -> str:
    """Write a seeded synthetic checkpoint; returns ``out_dir``.

    Re-running with the same (cfg, seed, device) reproduces the same bytes.
    """
    os.makedirs(out_dir, exist_ok=True)
    gen = torch.Generator(device=device)
    H, gs = cfg.hidden, cfg.group_size

    def randn(*shape, std=1.0):
        return torch.randn(*shape, generator=gen, device=device) * std

    def qput(w: _ShardWriter, prefix: str, t: torch.Tensor, bits: int):
        pk, s, b = quantize_affine(t, bits, gs)
        w.put(f"{prefix}.weight", pk)
        w.put(f"{prefix}.scales", s)
        w.put(f"{prefix}.biases", b)

    groups = [list(range(a, min(a + layers_per_shard, cfg.layers)))
              for a in range(0, cfg.layers, layers_per_shard)]
    n_shards = len(groups) + (1 if cfg.has_trunk else 0)
    for si, grp in enumerate(groups):
        specs = [s for L in grp for s in _layer_specs(cfg, L)]
        path = os.path.join(out_dir,
                            f"model-{si + 1:05d}-of-{n_shards:05d}.safetensors")
        w = _ShardWriter(path, specs)
        for L in grp:
            gen.manual_seed(seed * 1_000_003 + L)
            p = f"model.layers.{L}"
            std = cfg.weight_std
            if cfg.has_trunk:
                hd = cfg.head_dim
                w.put(f"{p}.input_layernorm.weight",
                      (1.0 + randn(H, std=0.05)).to(torch.bfloat16))
                w.put(f"{p}.post_attention_layernorm.weight",
                      (1.0 + randn(H, std=0.05)).to(torch.bfloat16))
                for nm, o, i in (("q_proj", cfg.heads * hd, H),
                                 ("k_proj", cfg.kv_heads * hd, H),
                                 ("v_proj", cfg.kv_heads * hd, H),
                                 ("o_proj", H, cfg.heads * hd)):
                    qput(w, f"{p}.self_attn.{nm}", randn(o, i, std=std),
                         cfg.trunk_bits)
                w.put(f"{p}.self_attn.q_norm.weight",
                      (1.0 + randn(hd, std=0.05)).to(torch.bfloat16))
                w.put(f"{p}.self_attn.k_norm.weight",
                      (1.0 + randn(hd, std=0.05)).to(torch.bfloat16))
            w.put(f"{p}.mlp.gate.weight",
                  randn(cfg.n_experts, H, std=1.0 / math.sqrt(H))
                  .to(torch.bfloat16))
            w.put(f"{p}.mlp.gate.bias",
                  zipf_bias(cfg.n_experts, cfg.zipf_s, seed * 7919 + L))
            E, I = cfg.n_experts, cfg.inter
            nrng = np.random.default_rng(seed * 1_000_003 + L * 7 + 1)
            for nm, o, i in (("gate_proj", I, H), ("up_proj", I, H),
                             ("down_proj", H, I)):
                pre = f"{p}.mlp.switch_mlp.{nm}"
                if cfg.expert_init == "codes":
                    for arr, part in zip(random_codes(nrng, (E,), o, i,
                                                      cfg.expert_bits, gs,
                                                      std),
                                         ("weight", "scales", "biases")):
                        w.put(f"{pre}.{part}", arr)
                else:
                    qput(w, pre, randn(E, o, i, std=std), cfg.expert_bits)
            if cfg.shared_inter:
                Is = cfg.shared_inter
                for nm, o, i in (("gate_proj", Is, H), ("up_proj", Is, H),
                                 ("down_proj", H, Is)):
                    qput(w, f"{p}.mlp.shared_expert.{nm}",
                         randn(o, i, std=std), cfg.trunk_bits)
        w.close()
    if cfg.has_trunk:
        path = os.path.join(out_dir,
                            f"model-{n_shards:05d}-of-{n_shards:05d}.safetensors")
        specs = (_qspecs("model.embed_tokens", cfg.vocab, H, cfg.trunk_bits, gs)
                 + [("model.norm.weight", "BF16", (H,))]
                 + _qspecs("lm_head", cfg.vocab, H, cfg.trunk_bits, gs))
        w = _ShardWriter(path, specs)
        gen.manual_seed(seed * 1_000_003 + 999_983)
        qput(w, "model.embed_tokens", randn(cfg.vocab, H, std=1.0),
             cfg.trunk_bits)
        w.put("model.norm.weight", (1.0 + randn(H, std=0.05))
              .to(torch.bfloat16))
        qput(w, "lm_head", randn(cfg.vocab, H, std=cfg.weight_std),
             cfg.trunk_bits)
        w.close()
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg.to_hf(), f, indent=1)
    return out_dir


def load_config(model_dir: str) -> SynthConfig:
    with open(os.path.join(model_dir, "config.json")) as f:
        d = json.load(f)["streamlx_synthetic"]
    return SynthConfig(**d)
