"""KV-cache sizing, maximum-context planning and YaRN switching.

Same behaviour and names as m5engine/context.py (KVFootprint :22-29,
measure_kv_footprint :50-73, native_context :76-87, yarn_capable :90-91,
apply_yarn :94-121, yarn_factor_for :124-129, combine :132-135, ContextPlan
:138-159, kv_estimate_per_token :162-170, reserve_bytes :173-175, plan_context
:178-229), written against the device model and caches of this package.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any, List, Optional, Tuple

GB = 1024**3

YARN_FAMILIES = ("qwen2", "qwen2_moe", "qwen3", "qwen3_moe")
MAX_YARN_FACTOR = 4


@dataclass
class KVFootprint:
    bytes_per_token: float
    fixed_bytes: int
    kv_bits: int

    def bytes_for(self, tokens: int) -> int:
        return int(self.fixed_bytes + self.bytes_per_token * tokens)


def _allocated_len(c) -> int:
    keys = getattr(c, "keys", None)
    if keys is None:
        return 0
    first = keys[0] if isinstance(keys, (tuple, list)) else keys
    return first.shape[-2]


def measure_kv_footprint(model, kv_bits: int, group_size: int = 64) -> KVFootprint:
    """Run one token through the model; per-token bytes of every attention cache."""
    from .attention import safe_maybe_quantize_kv_cache
    from .cache import make_prompt_cache
    cache = make_prompt_cache(model)
    model([[0]], cache)
    if kv_bits:
        safe_maybe_quantize_kv_cache(cache, 0, group_size, kv_bits)
    per_tok, fixed = 0.0, 0
    for c in cache:
        alloc = _allocated_len(c)
        if alloc:
            per_tok += c.nbytes / alloc
        else:
            fixed += c.nbytes
    return KVFootprint(per_tok, fixed, kv_bits)


def native_context(config: dict) -> Tuple[int, int]:
    """(native positional limit, current limit under the config's rope scaling)."""
    mpe = int(config.get("max_position_embeddings") or config.get("seq_length") or 4096)
    rs = config.get("rope_scaling") or {}
    kind = rs.get("type") or rs.get("rope_type")
    if kind in ("yarn", "linear", "dynamic") and rs.get("original_max_position_embeddings"):
        orig = int(rs["original_max_position_embeddings"])
        return orig, max(mpe, int(orig * float(rs.get("factor", 1))))
    native = int(config.get("original_max_position_embeddings") or mpe)
    if str(config.get("model_type", "")).startswith("qwen3") and mpe == 40960:
        native = 32768  # Qwen3: 32K positions plus 8K of generation headroom
    return native, mpe


def yarn_capable(config: dict) -> bool:
    return config.get("model_type") in YARN_FAMILIES and not config.get("rope_scaling")


def apply_yarn(model, factor: float, native: int) -> int:
    """Switch the model's RoPE to YaRN(factor) over `native` positions (1 = plain)."""
    model.set_rope(float(factor) if factor > 1 else 1.0, native)
    return len(model.layers)


def yarn_factor_for(tokens: int, native: int, max_factor: float) -> float:
    """Smallest power-of-two YaRN factor covering `tokens` (1.0 = plain RoPE)."""
    f = 1.0
    while native * f < tokens and f < max_factor:
        f *= 2
    return min(f, max_factor)


def combine(a: KVFootprint, b: Optional[KVFootprint]) -> KVFootprint:
    if b is None:
        return a
    return KVFootprint(a.bytes_per_token + b.bytes_per_token, a.fixed_bytes + b.fixed_bytes, a.kv_bits)


@dataclass
class ContextPlan:
    budget_bytes: int
    resident_weight_bytes: int
    expert_cache_bytes: int
    reserve_bytes: int
    kv_budget_bytes: int
    kv_bits: int
    kv_bytes_per_token: float
    native_context: int
    model_context_limit: int
    memory_context_limit: int
    yarn_factor: float
    max_context: int
    limited_by: str

    def to_dict(self) -> dict:
        d = asdict(self)
        for k in [k for k in d if k.endswith("_bytes")]:
            d[k[: -len("_bytes")] + "_gb"] = round(d[k] / GB, 2)
        return d


def kv_estimate_per_token(config: dict, kv_bits: int) -> float:
    """Upper bound of KV bytes per token from the config (before weights load)."""
    tc = config.get("text_config", config)
    layers = int(tc.get("num_hidden_layers") or 32)
    heads = int(tc.get("num_attention_heads") or 32)
    kv_heads = int(tc.get("num_key_value_heads") or heads)
    head_dim = int(tc.get("head_dim") or (int(tc.get("hidden_size") or 4096) // heads))
    per_elem = 2.0 if not kv_bits else kv_bits / 8 + 4 / 64   # bf16 scale + bias per 64 elements
    return 2 * layers * kv_heads * head_dim * per_elem


def reserve_bytes(budget: int, hidden_size: int, prefill_step: int) -> int:
    activations = prefill_step * max(hidden_size, 1) * 2 * 24
    return int(max(1.5 * GB, 0.04 * budget) + activations)


def plan_context(*, config: dict, footprint: KVFootprint, budget_bytes: int, resident_weight_bytes: int,
                 expert_cache_bytes: int = 0, prefill_step: int = 2048, rope_scaling: str = "auto",
                 requested_context: Optional[int] = None) -> ContextPlan:
    native, current = native_context(config)
    reserve = reserve_bytes(budget_bytes, int(config.get("hidden_size") or 0), prefill_step)
    kv_budget = budget_bytes - resident_weight_bytes - expert_cache_bytes - reserve
    if footprint.bytes_per_token > 0:
        mem_limit = int(max(0, kv_budget - footprint.fixed_bytes) // footprint.bytes_per_token)
    else:
        mem_limit = 1 << 30
    mem_limit -= mem_limit % 256

    yarn = 1.0
    model_limit = current
    target = requested_context or mem_limit
    if rope_scaling != "off" and yarn_capable(config) and target > current:
        f = yarn_factor_for(target, native, MAX_YARN_FACTOR) if rope_scaling == "auto" \
            else min(float(rope_scaling), MAX_YARN_FACTOR)
        yarn = float(f)
        model_limit = int(native * yarn)

    max_ctx = min(model_limit, mem_limit)
    if requested_context:
        max_ctx = min(max_ctx, requested_context)
    limited_by = "memory" if mem_limit <= model_limit else "model"
    if requested_context and requested_context <= min(model_limit, mem_limit):
        limited_by = "setting"
    return ContextPlan(budget_bytes=budget_bytes, resident_weight_bytes=resident_weight_bytes,
                       expert_cache_bytes=expert_cache_bytes, reserve_bytes=reserve, kv_budget_bytes=max(0, kv_budget),
                       kv_bits=footprint.kv_bits, kv_bytes_per_token=footprint.bytes_per_token,
                       native_context=native, model_context_limit=model_limit, memory_context_limit=mem_limit,
                       yarn_factor=yarn, max_context=max(0, max_ctx), limited_by=limited_by)
