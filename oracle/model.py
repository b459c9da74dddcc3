"""Qwen3 / Qwen3-MoE decoder and its token loop, restated (test infrastructure only).

Follows mlx-lm ``models/qwen3.py`` and ``models/qwen3_moe.py`` (third-party,
mlx-lm==0.31.3 per requirements.txt:4, not vendored) as the reference calls it:

* config keys read at m5engine/context.py:76-87 and 162-170;
* every Linear / Embedding is an MLX affine-quantized layer (w4 g64, bf16
  scale/bias) and computes ``y = x @ dequant(W).T`` with an fp32 accumulator and
  a bf16 result;
* RMSNorm (``mx.fast.rms_norm``): fp32 ``x * rsqrt(mean(x^2) + eps)``, rounded to
  bf16, times the bf16 weight, rounded again;
* attention: q/k/v proj -> per-head q_norm/k_norm -> RoPE/YaRN at the cache
  offset (split-half rotation; YaRN multiplies q and k by mscale first) ->
  cache append -> SDPA (``oracle.sdpa``) -> o_proj;
* MLP: ``down(silu(gate(x)) * up(x))``; MoE: softmax router (fp32 math, bf16
  out), top-k, renormalise, per-expert SwiGLU, score-weighted sum;
* the loop (m5engine/engine.py:396-423 -> mlx-lm ``generate_step``): the prompt
  minus its last token in chunks of ``prefill_step``, KV quantized after a model
  call once ``offset >= quantized_kv_start`` (m5engine/attention.py:106-112),
  then greedy argmax decoding (engine.py:384-386, temperature 0).

Activations are torch CPU fp32 tensors holding bf16 values; ``rb`` marks each
point where MLX produces a bf16 array.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from .quant import affine_dequantize_torch, affine_quantize, bf16_bits_to_f32, f32_to_bf16_bits
from .rope import rope_table
from .sdpa import blocked_quantized_sdpa, dense_quantized_sdpa, rb


@dataclass
class Config:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 40960
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    norm_topk_prob: bool = True
    group_size: int = 64
    bits: int = 4

    @classmethod
    def from_dict(cls, d: dict) -> "Config":
        q = d.get("quantization") or {}
        kw = {k: d[k] for k in cls.__dataclass_fields__ if k in d}
        kw["group_size"] = int(q.get("group_size", 64))
        kw["bits"] = int(q.get("bits", 4))
        return cls(**kw)

    @property
    def moe(self) -> bool:
        return self.num_experts > 0


# ------------------------------------------------------------ weight generation
def _linear_names(cfg: Config, i: int) -> List[tuple]:
    p = f"model.layers.{i}."
    H, D = cfg.hidden_size, cfg.head_dim
    out = [
        (p + "self_attn.q_proj", (cfg.num_attention_heads * D, H)),
        (p + "self_attn.k_proj", (cfg.num_key_value_heads * D, H)),
        (p + "self_attn.v_proj", (cfg.num_key_value_heads * D, H)),
        (p + "self_attn.o_proj", (H, cfg.num_attention_heads * D)),
    ]
    if cfg.moe:
        E, I = cfg.num_experts, cfg.moe_intermediate_size
        out += [
            (p + "mlp.gate", (E, H)),
            (p + "mlp.switch_mlp.gate_proj", (E, I, H)),
            (p + "mlp.switch_mlp.up_proj", (E, I, H)),
            (p + "mlp.switch_mlp.down_proj", (E, H, I)),
        ]
    else:
        I = cfg.intermediate_size
        out += [
            (p + "mlp.gate_proj", (I, H)),
            (p + "mlp.up_proj", (I, H)),
            (p + "mlp.down_proj", (H, I)),
        ]
    return out


def weight_specs(cfg: Config) -> List[tuple]:
    """(name, shape, kind) in generation order; kind is "q" (quantized) or "norm"."""
    H, D = cfg.hidden_size, cfg.head_dim
    specs = [("model.embed_tokens", (cfg.vocab_size, H), "q")]
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        specs.append((p + "input_layernorm", (H,), "norm"))
        specs.append((p + "post_attention_layernorm", (H,), "norm"))
        specs.append((p + "self_attn.q_norm", (D,), "norm"))
        specs.append((p + "self_attn.k_norm", (D,), "norm"))
        specs += [(n, s, "q") for n, s in _linear_names(cfg, i)]
    specs.append(("model.norm", (H,), "norm"))
    if not cfg.tie_word_embeddings:
        specs.append(("lm_head", (cfg.vocab_size, H), "q"))
    return specs


def generate_weights(cfg: Config, seed: int, std: float = 0.02,
                     layers: Optional[List[int]] = None) -> Dict[str, np.ndarray]:
    """Random-init weights in the MLX safetensors layout.

    Linear/embedding weights: N(0, std) -> bf16 -> affine quantize (``.weight``
    uint32, ``.scales`` / ``.biases`` bf16 bits).  Norm weights: 1 + N(0, std) in
    bf16 (``.weight`` bf16 bits).  Every tensor draws from its own
    ``default_rng([seed, index])`` stream so a subset of layers can be generated
    alone (``layers``) with identical values.
    """
    out: Dict[str, np.ndarray] = {}
    for idx, (name, shape, kind) in enumerate(weight_specs(cfg)):
        if layers is not None and name.startswith("model.layers."):
            if int(name.split(".")[2]) not in layers:
                continue
        rng = np.random.default_rng([seed, idx])
        if kind == "norm":
            w = 1.0 + std * rng.standard_normal(shape, dtype=np.float32)
            out[name + ".weight"] = f32_to_bf16_bits(w.astype(np.float32))
            continue
        w = (std * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        w = bf16_bits_to_f32(f32_to_bf16_bits(w))
        wq, s, b = affine_quantize(w, cfg.group_size, cfg.bits)
        out[name + ".weight"], out[name + ".scales"], out[name + ".biases"] = wq, s, b
    return out


# ---------------------------------------------------------------- primitives
def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    inv = torch.rsqrt((x * x).mean(dim=-1, keepdim=True) + eps)
    return rb(w * rb(x * inv))


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    return rb(rb(g * rb(torch.sigmoid(g))) * u)


def apply_rope(x: torch.Tensor, offset: int, inv_freq: torch.Tensor, mscale: float) -> torch.Tensor:
    """x [H, L, D] bf16 values -> rotated (split-half), bf16 values."""
    if mscale != 1.0:
        x = rb(x * mscale)
    L, D = x.shape[-2], x.shape[-1]
    pos = torch.arange(offset, offset + L, dtype=torch.float32)[:, None]
    theta = pos * inv_freq[None, :]                           # fp32 product
    c = torch.cos(theta.double()).float()
    s = torch.sin(theta.double()).float()
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    return rb(torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1))


# --------------------------------------------------------------------- caches
class KVCache:
    """Unquantized (bf16) cache: K/V [Hkv, S, D]."""

    def __init__(self):
        self.keys: Optional[torch.Tensor] = None
        self.values: Optional[torch.Tensor] = None
        self.offset = 0

    def update_and_fetch(self, k, v):
        self.keys = k if self.keys is None else torch.cat([self.keys, k], dim=-2)
        self.values = v if self.values is None else torch.cat([self.values, v], dim=-2)
        self.offset += k.shape[-2]
        return self.keys, self.values

    def to_quantized(self, group_size: int, bits: int) -> "QuantizedKVCache":
        qc = QuantizedKVCache(group_size, bits)
        if self.keys is not None:
            qc.update_and_fetch(self.keys, self.values)
        return qc


class QuantizedKVCache:
    """MLX QuantizedKVCache: K/V each as (packed uint32, scales, biases) along D."""

    def __init__(self, group_size: int = 64, bits: int = 8):
        self.group_size, self.bits = group_size, bits
        self.k_parts: List[tuple] = []
        self.v_parts: List[tuple] = []
        self.offset = 0

    def _q(self, x: torch.Tensor):
        return affine_quantize(x.numpy().astype(np.float32), self.group_size, self.bits)

    def update_and_fetch(self, k, v):
        self.k_parts.append(self._q(k))
        self.v_parts.append(self._q(v))
        self.offset += k.shape[-2]
        return self.keys, self.values

    @staticmethod
    def _cat(parts):
        return tuple(np.concatenate([p[i] for p in parts], axis=-2) for i in range(3))

    @property
    def keys(self):
        return self._cat(self.k_parts)

    @property
    def values(self):
        return self._cat(self.v_parts)


def maybe_quantize(cache: list, quantized_kv_start: int, group_size: int, bits: Optional[int]):
    """m5engine/attention.py:106-112: convert plain caches once offset >= start."""
    if not bits:
        return
    for i, c in enumerate(cache):
        if type(c) is KVCache and c.offset >= quantized_kv_start:
            cache[i] = c.to_quantized(group_size, bits)


# ---------------------------------------------------------------------- model
class Model:
    def __init__(self, cfg: Config, weights: Dict[str, np.ndarray], yarn_factor: float = 1.0,
                 native_ctx: int = 32768):
        self.cfg = cfg
        self.w = weights
        self._deq: Dict[str, torch.Tensor] = {}
        self.route_log: Optional[list] = None  # set to a list to record router margins
        # attention in key blocks of this size at every length (the blocked
        # loop of attention.py:29-103 without its dense fallback); None = as
        # the reference dispatches
        self.attn_block: Optional[int] = None
        self.set_rope(yarn_factor, native_ctx)

    def set_rope(self, factor: float, native: int = 32768):
        inv, ms = rope_table(self.cfg.head_dim, self.cfg.rope_theta, factor, native)
        self.inv_freq = torch.from_numpy(inv)
        self.mscale = ms

    def deq(self, name: str) -> torch.Tensor:
        t = self._deq.get(name)
        if t is None:
            w = self.w
            t = affine_dequantize_torch(w[name + ".weight"], w[name + ".scales"], w[name + ".biases"],
                                        self.cfg.group_size, self.cfg.bits)
            self._deq[name] = t
        return t

    def deq_expert(self, name: str, e: int) -> torch.Tensor:
        """Expert ``e`` of a stacked [E, rows, K] projection, dequantized alone
        (a whole stack of a large MoE would not fit in host memory)."""
        t = self._deq.get(name)
        if t is not None:
            return t[e]
        w = self.w
        return affine_dequantize_torch(w[name + ".weight"][e], w[name + ".scales"][e], w[name + ".biases"][e],
                                       self.cfg.group_size, self.cfg.bits)

    def norm_w(self, name: str) -> torch.Tensor:
        return torch.from_numpy(bf16_bits_to_f32(self.w[name + ".weight"]))

    def linear(self, x: torch.Tensor, name: str) -> torch.Tensor:
        return rb(x @ self.deq(name).T)

    def embed(self, tokens: List[int]) -> torch.Tensor:
        return rb(self.deq("model.embed_tokens")[torch.as_tensor(tokens, dtype=torch.long)])

    def attention(self, i: int, x: torch.Tensor, cache) -> torch.Tensor:
        cfg = self.cfg
        p = f"model.layers.{i}.self_attn."
        L, D, Hq, Hkv = x.shape[0], cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        q = self.linear(x, p + "q_proj").view(L, Hq, D)
        k = self.linear(x, p + "k_proj").view(L, Hkv, D)
        v = self.linear(x, p + "v_proj").view(L, Hkv, D)
        q = rms_norm(q, self.norm_w(p + "q_norm"), cfg.rms_norm_eps).transpose(0, 1)
        k = rms_norm(k, self.norm_w(p + "k_norm"), cfg.rms_norm_eps).transpose(0, 1)
        v = v.transpose(0, 1).contiguous()
        q = apply_rope(q, cache.offset, self.inv_freq, self.mscale)
        k = apply_rope(k, cache.offset, self.inv_freq, self.mscale)
        keys, values = cache.update_and_fetch(k.contiguous(), v)
        mask = "causal" if L > 1 else None
        scale = D ** -0.5
        if isinstance(cache, QuantizedKVCache):
            kq, vq = tuple(a[None] for a in keys), tuple(a[None] for a in values)
            gs, bits = cache.group_size, cache.bits
        else:
            kq, vq, gs, bits = keys[None], values[None], 64, 8
        if self.attn_block:
            o = blocked_quantized_sdpa(q[None], kq, vq, scale, mask, gs, bits, score_budget_bytes=1,
                                       min_block=self.attn_block, force_blocks=True)
        elif isinstance(cache, QuantizedKVCache):
            o = blocked_quantized_sdpa(q[None], kq, vq, scale, mask, gs, bits)
        else:
            o = dense_quantized_sdpa(q[None], kq, vq, scale, mask)
        o = o[0].transpose(0, 1).reshape(L, Hq * D)
        return self.linear(o, p + "o_proj")

    def mlp(self, i: int, x: torch.Tensor) -> torch.Tensor:
        p = f"model.layers.{i}.mlp."
        if not self.cfg.moe:
            return self.linear(silu_mul(self.linear(x, p + "gate_proj"), self.linear(x, p + "up_proj")),
                               p + "down_proj")
        return self.moe(i, x)[0]

    def route(self, i: int, x: torch.Tensor):
        """Router: (top-k expert ids [L, k] sorted by score desc, renormalised scores [L, k])."""
        cfg = self.cfg
        p = f"model.layers.{i}.mlp."
        gates = self.linear(x, p + "gate")
        probs = rb(torch.softmax(gates, dim=-1))
        k = cfg.num_experts_per_tok
        # Highest probability first; equal probabilities -> lower expert id first.
        order = torch.sort(probs, dim=-1, descending=True, stable=True).indices[:, :k]
        if self.route_log is not None:  # (rows, smallest k-th minus (k+1)-th probability) per call
            sp = torch.sort(probs, dim=-1, descending=True).values
            margin = (sp[:, k - 1] - sp[:, k]).min().item() if k < probs.shape[-1] else float("inf")
            self.route_log.append((x.shape[0], margin))
        scores = torch.gather(probs, 1, order)
        if cfg.norm_topk_prob:
            scores = rb(scores / rb(scores.sum(dim=-1, keepdim=True)))
        return order, scores, gates

    def moe(self, i: int, x: torch.Tensor):
        p = f"model.layers.{i}.mlp.switch_mlp."
        inds, scores, gates = self.route(i, x)
        L, k = inds.shape
        y = torch.zeros(L, k, x.shape[-1])
        # each routed (token, slot) pair through its expert's SwiGLU; an expert's
        # weights are dequantized once per call for all pairs routed to it
        for e in sorted(set(inds.reshape(-1).tolist())):
            wg, wu, wd = (self.deq_expert(p + n, e) for n in ("gate_proj", "up_proj", "down_proj"))
            for t, j in (inds == e).nonzero().tolist():
                g = rb(x[t] @ wg.T)
                u = rb(x[t] @ wu.T)
                y[t, j] = rb(silu_mul(g, u) @ wd.T)
        out = rb((rb(y * scores[..., None])).sum(dim=1))
        return out, inds, scores, gates

    def final_hidden(self, h: torch.Tensor) -> torch.Tensor:
        return rms_norm(h, self.norm_w("model.norm"), self.cfg.rms_norm_eps)

    def lm_head(self, h: torch.Tensor) -> torch.Tensor:
        name = "model.embed_tokens" if self.cfg.tie_word_embeddings else "lm_head"
        return self.linear(h, name)

    def __call__(self, tokens: List[int], cache: list, last_only: bool = False) -> torch.Tensor:
        cfg = self.cfg
        h = self.embed(tokens)
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}."
            r = self.attention(i, rms_norm(h, self.norm_w(p + "input_layernorm"), cfg.rms_norm_eps),
                               cache[i])
            h = rb(h + r)
            r = self.mlp(i, rms_norm(h, self.norm_w(p + "post_attention_layernorm"), cfg.rms_norm_eps))
            h = rb(h + r)
        if last_only:
            h = h[-1:]
        return self.lm_head(self.final_hidden(h))


def greedy(logits_row: torch.Tensor) -> int:
    """argmax over bf16 logits; the first index wins a tie."""
    return int(torch.argmax(logits_row))


def generate(model: Model, prompt: List[int], max_tokens: int, prefill_step: int = 2048,
             kv_bits: Optional[int] = 8, kv_group_size: int = 64, quantized_kv_start: int = 0,
             cache: Optional[list] = None, return_logits: bool = False, feed: Optional[List[int]] = None):
    """Greedy token loop of mlx-lm ``generate_step`` as the reference drives it.

    Returns (tokens, cache[, per-step last-position logits]).  ``feed``
    (teacher forcing, for comparing two runs step by step) replaces the token
    fed at decode step i with feed[i]; the returned tokens stay the greedy ones.
    """
    cache = cache if cache is not None else [KVCache() for _ in range(model.cfg.num_hidden_layers)]
    prompt = list(prompt)
    while len(prompt) > 1:
        n = min(prefill_step, len(prompt) - 1)
        model(prompt[:n], cache, last_only=True)
        maybe_quantize(cache, quantized_kv_start, kv_group_size, kv_bits)
        prompt = prompt[n:]
    logits = model(prompt, cache, last_only=True)[-1]
    maybe_quantize(cache, quantized_kv_start, kv_group_size, kv_bits)
    out, all_logits = [], []
    y = greedy(logits)
    for i in range(max_tokens):
        # generate_step evaluates the next step before yielding y, so the cache
        # ends holding prompt + max_tokens positions.
        nxt = model([y if feed is None else int(feed[i])], cache, last_only=True)[-1]
        maybe_quantize(cache, quantized_kv_start, kv_group_size, kv_bits)
        out.append(y)
        all_logits.append(logits)
        logits, y = nxt, greedy(nxt)
    if return_logits:
        return out, cache, torch.stack(all_logits)
    return out, cache
