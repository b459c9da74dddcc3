"""Qwen3 / Qwen3-MoE model handle over libm5cuda.

``Model`` satisfies what the reference asks of an mlx-lm model
(m5engine/engine.py:124-125, 395; context.py:53, 94-121): it is callable as
``model(tokens[1, L], cache=list) -> logits[1, L, V]``, has ``layers``,
``parameters()`` and a RoPE that ``apply_yarn`` can swap.  The weights are
device tensors in the MLX safetensors layout (``*.weight`` packed uint32 as
int32, ``*.scales`` / ``*.biases`` bf16, norm ``*.weight`` bf16), bound by name
into the C++ model handle; the forward pass is one ``m5_forward`` call.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from . import _lib
from ._lib import M5ModelCfg, call
from .cache import PromptCache, make_prompt_cache
from .distributed import kv_heads_local
from .ops import _stream


@dataclass
class ModelArgs:
    model_type: str = "qwen3"
    hidden_size: int = 1024
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 3072
    vocab_size: int = 151936
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
    rope_scaling: Optional[dict] = None

    @classmethod
    def from_dict(cls, d: dict) -> "ModelArgs":
        q = d.get("quantization") or {}
        kw = {k: d[k] for k in cls.__dataclass_fields__ if k in d and k not in ("group_size", "bits")}
        kw["group_size"] = int(q.get("group_size", 64))
        kw["bits"] = int(q.get("bits", 4))
        if "num_experts" not in d and d.get("model_type") == "qwen3_moe":
            raise ValueError("qwen3_moe config without num_experts")
        return cls(**kw)

    def to_dict(self) -> dict:
        d = {k: getattr(self, k) for k in self.__dataclass_fields__ if k not in ("group_size", "bits")}
        d["quantization"] = {"group_size": self.group_size, "bits": self.bits}
        return d

    @property
    def moe(self) -> bool:
        return self.num_experts > 0


def weight_specs(a: ModelArgs) -> List[tuple]:
    """(name, shape of the unquantized tensor, kind) in the MLX checkpoint layout."""
    H, D = a.hidden_size, a.head_dim
    specs = [("model.embed_tokens", (a.vocab_size, H), "q")]
    for i in range(a.num_hidden_layers):
        p = f"model.layers.{i}."
        specs += [(p + "input_layernorm", (H,), "norm"), (p + "post_attention_layernorm", (H,), "norm"),
                  (p + "self_attn.q_norm", (D,), "norm"), (p + "self_attn.k_norm", (D,), "norm"),
                  (p + "self_attn.q_proj", (a.num_attention_heads * D, H), "q"),
                  (p + "self_attn.k_proj", (a.num_key_value_heads * D, H), "q"),
                  (p + "self_attn.v_proj", (a.num_key_value_heads * D, H), "q"),
                  (p + "self_attn.o_proj", (H, a.num_attention_heads * D), "q")]
        if a.moe:
            E, I = a.num_experts, a.moe_intermediate_size
            specs += [(p + "mlp.gate", (E, H), "q"), (p + "mlp.switch_mlp.gate_proj", (E, I, H), "q"),
                      (p + "mlp.switch_mlp.up_proj", (E, I, H), "q"),
                      (p + "mlp.switch_mlp.down_proj", (E, H, I), "q")]
        else:
            I = a.intermediate_size
            specs += [(p + "mlp.gate_proj", (I, H), "q"), (p + "mlp.up_proj", (I, H), "q"),
                      (p + "mlp.down_proj", (H, I), "q")]
    specs.append(("model.norm", (H,), "norm"))
    if not a.tie_word_embeddings:
        specs.append(("lm_head", (a.vocab_size, H), "q"))
    return specs


EXPERT_BLOCK = 8  # experts of a stacked MoE projection drawn from one generator seed


def random_weights(a: ModelArgs, seed: int, device, std: float = 0.02,
                   experts: Optional[tuple] = None) -> Dict[str, torch.Tensor]:
    """Random-init MLX-layout weights generated and quantized on the device.

    Linear/embedding weights N(0, std) in bf16 -> 4-bit g64 (libm5cuda quantizer);
    norm weights 1 + N(0, std) in bf16.  Tensor i draws from seed*1000003 + i;
    a stacked expert projection ([E, rows, K]) draws each block of
    EXPERT_BLOCK experts from its own seed, so ``experts=(first, count)``
    generates only that range of every stack (an expert-parallel rank's
    shard) with the values the full stack holds there.
    """
    from .ops import quantize
    out: Dict[str, torch.Tensor] = {}
    g = torch.Generator(device=device)
    for idx, (name, shape, kind) in enumerate(weight_specs(a)):
        g.manual_seed(seed * 1000003 + idx)
        if kind == "norm":
            out[name + ".weight"] = (1.0 + std * torch.randn(shape, generator=g, device=device)).to(torch.bfloat16)
            continue
        if ".switch_mlp." in name:
            E = shape[0]
            e0, n = experts if experts is not None else (0, E)
            if e0 < 0 or n <= 0 or e0 + n > E:
                raise ValueError(f"expert range {experts} outside 0..{E}")
            parts = []
            for blk in range(e0 // EXPERT_BLOCK, (e0 + n + EXPERT_BLOCK - 1) // EXPERT_BLOCK):
                g.manual_seed((seed * 1000003 + idx) * 1009 + blk)
                lo, hi = blk * EXPERT_BLOCK, min(E, (blk + 1) * EXPERT_BLOCK)
                w = (std * torch.randn((hi - lo,) + tuple(shape[1:]), generator=g, device=device))
                w = w[max(lo, e0) - lo:min(hi, e0 + n) - lo].to(torch.bfloat16)
                parts.append(quantize(w, a.group_size, a.bits))
                del w
            for j, suf in enumerate((".weight", ".scales", ".biases")):
                out[name + suf] = torch.cat([p[j] for p in parts]) if len(parts) > 1 else parts[0][j]
            continue
        # Quantize in slices to bound the bf16 temporary of large stacks.
        rows = shape[0]
        w_parts, s_parts, b_parts = [], [], []
        per = max(1, (1 << 28) // int(np.prod(shape[1:])))
        for r0 in range(0, rows, per):
            sub = (min(per, rows - r0),) + tuple(shape[1:])
            w = (std * torch.randn(sub, generator=g, device=device)).to(torch.bfloat16)
            wq, s, b = quantize(w, a.group_size, a.bits)
            w_parts.append(wq); s_parts.append(s); b_parts.append(b)
            del w
        out[name + ".weight"] = torch.cat(w_parts) if len(w_parts) > 1 else w_parts[0]
        out[name + ".scales"] = torch.cat(s_parts) if len(s_parts) > 1 else s_parts[0]
        out[name + ".biases"] = torch.cat(b_parts) if len(b_parts) > 1 else b_parts[0]
    return out


def upload_weights(host: Dict[str, np.ndarray], device) -> Dict[str, torch.Tensor]:
    """Host MLX-layout arrays (uint32 words / uint16 bf16 bits) -> device tensors."""
    out = {}
    for k, v in host.items():
        if v.dtype == np.uint32:
            out[k] = torch.from_numpy(v.view(np.int32)).to(device)
        elif v.dtype == np.uint16:
            out[k] = torch.from_numpy(v.view(np.int16)).view(torch.bfloat16).to(device)
        else:
            out[k] = torch.from_numpy(v).to(device)
    return out


class _RoPE:
    """Stand-in for the rope module context.apply_yarn swaps (factor, native)."""

    def __init__(self, dims: int, base: float):
        self.dims, self.base, self.traditional = dims, base, False
        self.factor, self.native = 1.0, 32768


def rope_inv_freq(dims: int, base: float, factor: float = 1.0, native: int = 32768):
    """(inv_freq fp32 [dims/2], mscale): plain RoPE, or YaRN (beta_fast 32, beta_slow 1)."""
    idx = np.arange(0, dims, 2, dtype=np.float64)
    period = base ** (idx / dims)
    if factor <= 1:
        return (1.0 / period).astype(np.float32), 1.0

    def corr_dim(n_rot):
        return (dims * math.log(native / (n_rot * 2 * math.pi))) / (2 * math.log(base))

    low = max(math.floor(corr_dim(32.0)), 0)
    high = min(math.ceil(corr_dim(1.0)), dims - 1)
    if low == high:
        high += 0.001
    ramp = np.clip((np.arange(dims // 2, dtype=np.float64) - low) / (high - low), 0.0, 1.0)
    keep = 1.0 - ramp
    inv = keep / period + (1.0 - keep) / (factor * period)
    return inv.astype(np.float32), 0.1 * math.log(factor) + 1.0


class Model:
    def __init__(self, args: ModelArgs, weights: Dict[str, torch.Tensor], device="cuda", max_tokens: int = 2048,
                 tp_size: int = 1, tp_rank: int = 0, ep_size: int = 1, ep_rank: int = 0, comm=None):
        """``weights``: this rank's shard (``distributed.shard_weights``) when
        tp_size or ep_size > 1, with ``comm`` the rank's ``Communicator``."""
        if args.head_dim != 128:
            raise ValueError("head_dim must be 128")
        self.args = args
        self.device = torch.device(device)
        self.weights = weights
        self.tp_size, self.tp_rank, self.ep_size, self.ep_rank = tp_size, tp_rank, ep_size, ep_rank
        self.n_kv_heads_local = kv_heads_local(args.num_key_value_heads, tp_size)
        self.layers = [None] * args.num_hidden_layers
        cfg = M5ModelCfg(
            hidden_size=args.hidden_size, num_layers=args.num_hidden_layers, num_heads=args.num_attention_heads,
            num_kv_heads=args.num_key_value_heads, head_dim=args.head_dim,
            intermediate_size=args.intermediate_size, vocab_size=args.vocab_size, num_experts=args.num_experts,
            experts_per_tok=args.num_experts_per_tok, moe_intermediate_size=args.moe_intermediate_size,
            norm_topk_prob=int(args.norm_topk_prob), tie_word_embeddings=int(args.tie_word_embeddings),
            rms_norm_eps=args.rms_norm_eps, group_size=args.group_size, bits=args.bits, tp_size=tp_size,
            tp_rank=tp_rank, ep_size=ep_size, ep_rank=ep_rank)
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            call("m5_model_create", ctypes.byref(cfg), ctypes.byref(h))
        self._h = h
        for name, t in weights.items():
            if not t.is_cuda:
                raise ValueError(f"weight {name} is not on the device")
            call("m5_model_bind", self._h, name.encode(), t.data_ptr())
        self.rope = _RoPE(args.head_dim, args.rope_theta)
        self.set_rope(1.0)
        self.comm = comm
        if tp_size > 1 or ep_size > 1:
            if comm is None:
                raise ValueError("a multi-rank model needs a Communicator")
            call("m5_model_set_comm", self._h, comm.handle)
        self.max_tokens = 0
        self.reserve(max_tokens)
        call("m5_model_check", self._h)

    # ------------------------------------------------------------ properties
    def parameters(self) -> Dict[str, torch.Tensor]:
        return self.weights

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.weights.values())

    def set_rope(self, factor: float, native: int = 32768) -> None:
        inv, ms = rope_inv_freq(self.args.head_dim, self.args.rope_theta, factor, native)
        arr = (ctypes.c_float * len(inv))(*inv.tolist())
        call("m5_model_set_rope", self._h, arr, float(ms))
        self.rope.factor, self.rope.native = factor, native

    def reserve(self, max_tokens: int) -> None:
        if max_tokens > self.max_tokens:
            with torch.cuda.device(self.device):
                call("m5_model_reserve", self._h, int(max_tokens))
            self.max_tokens = max_tokens

    def make_cache(self, capacity: int = 0) -> PromptCache:
        return make_prompt_cache(self, capacity)

    # --------------------------------------------------------------- forward
    def forward(self, tokens: torch.Tensor, cache: PromptCache, logits_mode: int = _lib.M5_LOGITS_NONE,
                logits: Optional[torch.Tensor] = None, argmax_out: Optional[torch.Tensor] = None,
                sync_len: bool = True) -> None:
        """Run L tokens (int32 CUDA tensor [L]) and advance every cache layer by L."""
        L = int(tokens.numel())
        if L > self.max_tokens:
            self.reserve(L)
        need = cache.offset + L
        for c in cache:
            if c.capacity < need:
                c.reserve(need)
        if sync_len:
            cache.d_len.fill_(cache.offset)
        structs = cache.structs()
        call("m5_forward", self._h, structs, cache.d_len.data_ptr(), tokens.data_ptr(), L,
             None if logits is None else logits.data_ptr(), logits_mode,
             None if argmax_out is None else argmax_out.data_ptr(), _stream())
        for c in cache:
            c.offset += L

    def prefill_sequence(self, tokens: torch.Tensor, cache: PromptCache, seq: int, chunk: int = 2048) -> None:
        """Prefill sequence `seq` of a batched cache with `tokens` (int32 CUDA
        [L]) from position 0, in chunks; the cache's shared offset is left to
        the caller (every sequence of a batch is prefilled to the same length)."""
        L = int(tokens.numel())
        for c in cache:
            if c.capacity < L:
                c.reserve(L)
        structs = cache.structs(seq)
        d_len = torch.zeros(1, dtype=torch.int32, device=self.device)
        for p0 in range(0, L, chunk):
            n = min(chunk, L - p0)
            if n > self.max_tokens:
                self.reserve(n)
            call("m5_forward", self._h, structs, d_len.data_ptr(), tokens[p0:p0 + n].data_ptr(), n, None,
                 _lib.M5_LOGITS_NONE, None, _stream())

    def forward_batch(self, tokens: torch.Tensor, cache: PromptCache, logits: Optional[torch.Tensor] = None,
                      argmax_out: Optional[torch.Tensor] = None, sync_len: bool = True) -> None:
        """One decode token for each of the cache's B sequences (int32 CUDA
        tokens [B], all at position cache.offset): logits [B, V] and / or the
        greedy tokens [B]; advances the shared offset by one."""
        B = int(tokens.numel())
        if B != cache.batch:
            raise ValueError(f"forward_batch: {B} tokens for a cache of {cache.batch} sequences")
        if B > self.max_tokens:
            self.reserve(B)
        need = cache.offset + 1
        for c in cache:
            if c.capacity < need:
                c.reserve(need)
        if argmax_out is not None and logits is None:
            logits = torch.empty(B, self.args.vocab_size, dtype=torch.bfloat16, device=self.device)
        if sync_len:
            cache.d_len.fill_(cache.offset)
        call("m5_forward_batch", self._h, cache.structs(), cache.d_len.data_ptr(), tokens.data_ptr(), B,
             None if logits is None else logits.data_ptr(),
             _lib.M5_LOGITS_NONE if logits is None else _lib.M5_LOGITS_ALL,
             None if argmax_out is None else argmax_out.data_ptr(), _stream())
        for c in cache:
            c.offset += 1

    def __call__(self, tokens, cache: Optional[PromptCache] = None) -> torch.Tensor:
        """``model(tokens[1, L], cache) -> logits[1, L, V]`` (bf16)."""
        if cache is None:
            cache = self.make_cache()
        t = torch.as_tensor(tokens, dtype=torch.int32, device=self.device).reshape(-1)
        L = t.numel()
        out = torch.empty(L, self.args.vocab_size, dtype=torch.bfloat16, device=self.device)
        self.forward(t, cache, _lib.M5_LOGITS_ALL, out)
        return out.reshape(1, L, -1)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().m5_model_destroy(h)
            except Exception:
                pass
            self._h = None
