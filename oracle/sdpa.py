"""Attention over a (quantized) KV cache, restated (test infrastructure only).

Two functions follow the reference op for op, including where it rounds to bf16:

* ``dense_quantized_sdpa`` - mlx-lm's own quantized SDPA, which the reference
  saves at m5engine/attention.py:19 and calls for ``S <= block`` or ``L == 1``
  (attention.py:42-45): q*scale (bf16), scores = quantized_matmul (bf16 out),
  mask, precise softmax (fp32 math, bf16 out), P @ V (bf16 out).
* ``blocked_quantized_sdpa`` - attention.py:29-103: key blocks of
  ``max(MIN_BLOCK, budget // (B*Hq*L*12))``; scores rounded to bf16 then fp32
  (attention.py:66-69); masked scores = -1e30 (attention.py:60, 81); p rounded
  to bf16 only for the PV product (attention.py:87-90); fp32 running max /
  denominator; output ``acc / max(denom, 1e-30)`` cast to the query dtype
  (attention.py:100).

Tensors are torch CPU fp32 holding bf16 values; K/V come either as fp32
(unquantized cache) or as the MLX tuple (packed uint32, scales, biases).
"""

from __future__ import annotations

from typing import Optional, Union

import numpy as np
import torch

from .quant import affine_dequantize_torch

SCORE_BUDGET_BYTES = 512 * 1024**2      # attention.py:21
MIN_BLOCK = 256                         # attention.py:22
BF16_MIN = -3.3895313892515355e38       # finfo(bfloat16).min (mlx-lm bool mask fill)


def rb(x: torch.Tensor) -> torch.Tensor:
    """Round an fp32 tensor to bf16 values (round-to-nearest-even)."""
    return x.to(torch.bfloat16).to(torch.float32)


def dequant_kv(kv, group_size: int = 64, bits: int = 8) -> torch.Tensor:
    """MLX (packed, scales, biases) tuple -> fp32 tensor; fp32 input is returned as is."""
    if isinstance(kv, torch.Tensor):
        return kv.float()
    wq, s, b = kv
    return affine_dequantize_torch(np.asarray(wq), np.asarray(s), np.asarray(b), group_size, bits)


def _causal(L: int, S: int) -> torch.Tensor:
    return torch.arange(S - L, S)[:, None] >= torch.arange(S)[None]


def _rounder(dtype: str):
    if dtype == "bf16":
        return rb
    if dtype == "f32":
        return lambda x: x
    raise ValueError(dtype)


def dense_quantized_sdpa(queries: torch.Tensor, keys, values, scale: float,
                         mask: Union[None, str, torch.Tensor], group_size: int = 64,
                         bits: int = 8, dtype: str = "bf16") -> torch.Tensor:
    """queries fp32 [B, Hq, L, D]; keys/values [B, Hkv, S, D] or tuples.

    ``dtype`` is the query dtype the reference would see: "bf16" rounds at every
    point MLX produces a bf16 array, "f32" (the reference's own unit test,
    tests/test_core.py:28) rounds nowhere.
    """
    rb = _rounder(dtype)
    B, Hq, L, D = queries.shape
    K = dequant_kv(keys, group_size, bits)
    V = dequant_kv(values, group_size, bits)
    Hkv, S = K.shape[-3], K.shape[-2]
    rep = Hq // Hkv
    q = rb(queries * scale)
    # The `rep` query heads of a GQA group share kv head h // rep (mlx-lm
    # repeats K/V per group); the group's rows are stacked against one K/V
    # instead of materialising the repeated tensors (same products).
    qg = q.reshape(B, Hkv, rep * L, D)
    scores = rb(qg @ K.transpose(-1, -2)).reshape(B, Hq, L, S)
    if mask is not None:
        if isinstance(mask, str):
            mask = _causal(L, S)
        if mask.dtype == torch.bool:
            scores = torch.where(mask, scores, torch.tensor(BF16_MIN))
        else:
            scores = rb(scores + mask.float())
    p = rb(torch.softmax(scores, dim=-1))
    return rb(p.reshape(B, Hkv, rep * L, S) @ V).reshape(B, Hq, L, D)


def blocked_quantized_sdpa(queries: torch.Tensor, keys, values, scale: float,
                           mask: Union[None, str, torch.Tensor], group_size: int = 64,
                           bits: int = 8, score_budget_bytes: int = SCORE_BUDGET_BYTES,
                           min_block: int = MIN_BLOCK, dtype: str = "bf16",
                           force_blocks: bool = False) -> torch.Tensor:
    """``force_blocks`` runs the block loop even where attention.py:42-45 falls
    back to the dense op (short caches, single queries): the same algorithm
    at any length, for measuring how far its rounding points move a result."""
    rb = _rounder(dtype)
    B, Hq, L, D = queries.shape
    K = dequant_kv(keys, group_size, bits)
    V = dequant_kv(values, group_size, bits)
    S = K.shape[-2]
    per_key = B * Hq * L * 4 * 3
    block = max(min_block, score_budget_bytes // max(per_key, 1))
    if not force_blocks and (S <= block or L == 1):
        return dense_quantized_sdpa(queries, keys, values, scale, mask, group_size, bits, dtype)
    Hkv = K.shape[-3]
    rep = Hq // Hkv
    q = rb(queries * scale)
    if rep > 1:
        K = K.repeat_interleave(rep, dim=-3)
        V = V.repeat_interleave(rep, dim=-3)
    causal = isinstance(mask, str)
    q_pos = torch.arange(S - L, S)[:, None] if causal else None
    neg = torch.tensor(-1e30, dtype=torch.float32)
    m = denom = acc = None
    for start in range(0, S, block):
        end = min(S, start + block)
        scores = rb(q @ K[..., start:end, :].transpose(-1, -2))
        valid: Optional[torch.Tensor] = None
        if causal:
            if end > S - L:
                valid = q_pos >= torch.arange(start, end)[None]
        elif mask is not None:
            blk = mask[..., start:end]
            if blk.dtype == torch.bool:
                valid = blk
            else:
                scores = scores + blk.float()
        if valid is not None:
            scores = torch.where(valid, scores, neg)
        blk_max = scores.amax(dim=-1, keepdim=True)
        m_new = blk_max if m is None else torch.maximum(m, blk_max)
        p = torch.exp(scores - m_new)
        if valid is not None:
            p = torch.where(valid, p, torch.zeros(()))
        pv = rb(rb(p) @ V[..., start:end, :])
        if m is None:
            denom = p.sum(dim=-1, keepdim=True)
            acc = pv
        else:
            corr = torch.exp(m - m_new)
            denom = denom * corr + p.sum(dim=-1, keepdim=True)
            acc = acc * corr + pv
        m = m_new
    return rb(acc / torch.clamp(denom, min=1e-30))


def reference_attention(q: torch.Tensor, kd: torch.Tensor, vd: torch.Tensor, scale: float,
                        mask: Optional[torch.Tensor]) -> torch.Tensor:
    """Dense fp32 attention on dequantized K/V (tests/test_core.py:16-20)."""
    s = (q * scale) @ kd.transpose(-1, -2)
    if mask is not None:
        s = torch.where(mask, s, torch.tensor(-1e30))
    return torch.softmax(s, dim=-1) @ vd
