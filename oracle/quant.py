"""MLX affine group quantization, restated in numpy (bit-exact integer work).

Test infrastructure only (see ``oracle/__init__``).

The rule restated here is MLX's published affine quantizer (``mx.quantize``):
per group of ``group_size`` consecutive elements along the last axis,

    n_bins = 2**bits - 1
    scale  = max((w_max - w_min) / n_bins, 1e-7)            (fp32)
    if |w_min| > |w_max|:  edge = w_min, scale = +scale
    else:                  edge = w_max, scale = -scale
    q0 = rint(edge / scale)
    if q0 != 0:  scale = edge / q0, bias = edge             (zero is exact)
    else:        bias = 0
    q  = clip(rint((w - bias) / scale), 0, n_bins)           (fp32, IEEE div)

``scale`` and ``bias`` are stored in the input dtype (bf16 here) while ``q`` is
computed from their fp32 values.  ``rint`` is round-half-to-even (the CPU
backend's rounding).  q is packed low-bits-first: element ``j`` of a uint32
word sits at bit ``j * bits`` (the same order as
native/src/memory_arena.mm:229-238 and native/include/tensor.hpp:76-86).

Assumption (cannot be checked without MLX): the pinned MLX version uses exactly
this edge rule, eps floor and fp32 intermediate; re-confirm on a box with MLX.
Callers of this rule in the reference: m5engine/attention.py:111-112 (KV cache
``to_quantized``) and mlx-lm ``QuantizedKVCache.update_and_fetch``.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------- bf16
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (round-to-nearest-even); returns uint16 bit patterns."""
    x = np.ascontiguousarray(x, dtype=F32)
    b = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    lsb = (b >> 16) & 1
    r = ((b + 0x7FFF + lsb) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(F32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 value, returned as fp32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ------------------------------------------------------------ quantization
def affine_quantize(w: np.ndarray, group_size: int = 64, bits: int = 4):
    """Quantize ``w`` (fp32 values; bf16 inputs already exact in fp32).

    Returns ``(wq uint32 [..., K*bits/32], scales_bits uint16 [..., K/gs],
    biases_bits uint16 [..., K/gs])`` with scales/biases as bf16 bit patterns.
    """
    if bits not in (4, 8):
        raise ValueError("bits must be 4 or 8")
    w = np.asarray(w, dtype=F32)
    K = w.shape[-1]
    if K % group_size:
        raise ValueError("last dim must be a multiple of group_size")
    lead = w.shape[:-1]
    g = w.reshape(-1, K // group_size, group_size)
    n_bins = F32((1 << bits) - 1)
    w_max = g.max(axis=-1, keepdims=True)
    w_min = g.min(axis=-1, keepdims=True)
    side = np.abs(w_min) > np.abs(w_max)
    scale = np.maximum((w_max - w_min) / n_bins, F32(1e-7)).astype(F32)
    scale = np.where(side, scale, -scale).astype(F32)
    edge = np.where(side, w_min, w_max).astype(F32)
    with np.errstate(divide="ignore", invalid="ignore"):
        q0 = np.rint(edge / scale).astype(F32)
        nz = q0 != 0
        scale = np.where(nz, edge / np.where(nz, q0, F32(1)), scale).astype(F32)
    bias = np.where(nz, edge, F32(0)).astype(F32)
    q = np.clip(np.rint((g - bias) / scale), F32(0), n_bins).astype(np.uint32)
    per = 32 // bits
    q = q.reshape(-1, K // per, per)
    shifts = (np.arange(per, dtype=np.uint32) * bits).astype(np.uint32)
    wq = np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)
    return (
        wq.reshape(*lead, K * bits // 32),
        f32_to_bf16_bits(scale).reshape(*lead, K // group_size),
        f32_to_bf16_bits(bias).reshape(*lead, K // group_size),
    )


def unpack(wq: np.ndarray, bits: int) -> np.ndarray:
    """uint32 words -> integer codes, low bits first."""
    per = 32 // bits
    mask = np.uint32((1 << bits) - 1)
    shifts = (np.arange(per, dtype=np.uint32) * bits).astype(np.uint32)
    q = (wq[..., None] >> shifts) & mask
    return q.reshape(*wq.shape[:-1], wq.shape[-1] * per)


def affine_dequantize(wq, scales_bits, biases_bits, group_size: int = 64, bits: int = 4) -> np.ndarray:
    """``scale * q + bias`` in fp32 (the value a dequantizing matmul multiplies by)."""
    q = unpack(np.asarray(wq, dtype=np.uint32), bits).astype(F32)
    K = q.shape[-1]
    s = bf16_bits_to_f32(scales_bits)
    b = bf16_bits_to_f32(biases_bits)
    qg = q.reshape(*q.shape[:-1], K // group_size, group_size)
    w = qg * s[..., None] + b[..., None]
    return w.reshape(q.shape).astype(F32)


def affine_dequantize_torch(wq: np.ndarray, scales_bits: np.ndarray, biases_bits: np.ndarray,
                            group_size: int = 64, bits: int = 4):
    """``affine_dequantize`` with torch CPU kernels (multithreaded), same values:
    the code times the fp32 scale, rounded, plus the fp32 bias, rounded (two
    IEEE steps, no fused multiply-add), as the numpy version computes them."""
    import torch
    per = 32 // bits
    w = torch.from_numpy(np.ascontiguousarray(wq, dtype=np.uint32).view(np.int32)).long() & 0xFFFFFFFF
    shifts = torch.arange(per, dtype=torch.long) * bits
    q = ((w[..., None] >> shifts) & ((1 << bits) - 1)).to(torch.float32)
    q = q.reshape(*w.shape[:-1], w.shape[-1] * per)
    K = q.shape[-1]
    s = torch.from_numpy(bf16_bits_to_f32(scales_bits))
    b = torch.from_numpy(bf16_bits_to_f32(biases_bits))
    qg = q.reshape(*q.shape[:-1], K // group_size, group_size)
    out = torch.mul(qg, s[..., None])
    out = torch.add(out, b[..., None])
    return out.reshape(q.shape)
