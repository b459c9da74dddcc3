"""Quantized-KV attention with the reference's operator signature.

``blocked_quantized_sdpa`` keeps the signature and argument meaning of
m5engine/attention.py:29-37; ``safe_maybe_quantize_kv_cache`` keeps
m5engine/attention.py:106-112.  The body is one libm5cuda split-KV flash
attention launch (fp32 online softmax with the reference's bf16 rounding of
scores and of p), so ``score_budget_bytes`` / ``MIN_BLOCK`` only matter to the
reference's block loop and are kept as module attributes for API parity.
"""

from __future__ import annotations

from typing import Optional, Union

import torch

from . import _lib
from ._lib import call
from .ops import _need_cuda, _stream, kv_view, mask_strides

score_budget_bytes = 512 * 1024**2  # m5engine/attention.py:21 (bounds the reference's score blocks)
MIN_BLOCK = 256                      # m5engine/attention.py:22


def _rows_stride(t: torch.Tensor, axis: int) -> int:
    row = t.stride(-2)
    if t.stride(-1) != 1 or t.stride(axis) % row:
        raise ValueError("K/V rows must be contiguous along the last axis")
    return t.stride(axis) // row


def blocked_quantized_sdpa(queries: torch.Tensor, q_keys, q_values, scale: float,
                           mask: Union[None, str, torch.Tensor], group_size: int = 64,
                           bits: int = 8) -> torch.Tensor:
    """softmax(queries * scale @ K^T + mask) @ V over a quantized (or bf16) cache.

    queries: bf16 [B, Hq, L, D].  q_keys / q_values: MLX tuples
    ``(wq int32 [B, Hkv, S, D*bits/32], scales bf16 [B, Hkv, S, D/64], biases)``
    or plain bf16 [B, Hkv, S, D] tensors (then ``bits`` is ignored).  mask:
    None, "causal" (query i at position S - L + i), a bool tensor or an
    additive float tensor broadcastable to [B, Hq, L, S].
    """
    _need_cuda(queries)
    if queries.dtype != torch.bfloat16:
        raise ValueError("queries must be bf16")
    B, Hq, L, D = queries.shape
    packed = isinstance(q_keys, (tuple, list))
    k0 = q_keys[0] if packed else q_keys
    v0 = q_values[0] if packed else q_values
    Hkv, S = k0.shape[-3], k0.shape[-2]
    if Hq % Hkv:
        raise ValueError("number of query heads must be a multiple of kv heads")
    kb = 0 if k0.dim() < 4 else _rows_stride(k0, 0)
    vb = 0 if v0.dim() < 4 else _rows_stride(v0, 0)
    kv_k = kv_view(q_keys, _rows_stride(k0, -3), kb)
    kv_v = kv_view(q_values, _rows_stride(v0, -3), vb)
    eff_bits = bits if packed else 0
    mask_kind, mptr, mstr, keep = _lib.M5_MASK_NONE, None, None, None
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError(f"unknown mask {mask!r}")
        mask_kind = _lib.M5_MASK_CAUSAL
    elif mask is not None:
        m = mask
        while m.dim() < 4:
            m = m.unsqueeze(0)
        if m.dtype == torch.bool:
            keep = m.to(torch.uint8).contiguous()
            mask_kind = _lib.M5_MASK_BOOL
        else:
            keep = m.to(torch.float32).contiguous()
            mask_kind = _lib.M5_MASK_ADDITIVE
        keep = keep.to(queries.device)
        mptr = keep.data_ptr()
        mstr = mask_strides(keep, B, Hq)
    q = queries.contiguous()
    out = torch.empty_like(q)
    call("m5_quantized_sdpa", q.data_ptr(), B, Hq, L, D, kv_k, kv_v, Hkv, S, float(scale), mask_kind, mptr, mstr,
         group_size, eff_bits, out.data_ptr(), _stream())
    return out


def safe_maybe_quantize_kv_cache(prompt_cache, quantized_kv_start: int, kv_group_size: int,
                                 kv_bits: Optional[int]) -> None:
    """Quantize only plain (bf16) KV caches whose offset reached the threshold."""
    if kv_bits is None:
        return
    from .cache import KVCache
    for i, c in enumerate(prompt_cache):
        if type(c) is KVCache and c.offset >= quantized_kv_start:
            prompt_cache[i] = c.to_quantized(group_size=kv_group_size, bits=kv_bits)

