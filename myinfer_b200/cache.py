"""Device KV caches with the mlx-lm cache contract the reference relies on.

What the reference reads from a cache: ``offset`` (m5engine/prefix_cache.py:27-38,
104), ``nbytes`` (prefix_cache.py:17-24, context.py:60-61), ``keys`` as an
array or an MLX tuple whose sequence axis is -2 (context.py:41-47), ``state``
(context.py:56), and trimming through ``can_trim_prompt_cache`` /
``trim_prompt_cache`` (prefix_cache.py:14, 90, 97-99).  Quantization switches a
``KVCache`` to a ``QuantizedKVCache`` (attention.py:106-112).

Layout in HBM: bf16 K/V ``[B, Hkv, capacity, D]``; packed K/V
``[B, Hkv, capacity, D*bits/32]`` int32 words + bf16 scales/biases
``[B, Hkv, capacity, D/64]`` (B = 1 except for batched decode, where the B
sequences share one length).  Capacity grows in steps of 256 positions like
mlx-lm, and may be reserved ahead of time so a captured decode graph never
sees a reallocation.  Trimming only moves ``offset`` back (move-not-copy).
"""

from __future__ import annotations

from typing import List, Optional

import torch

from ._lib import M5LayerKv, call
from .ops import _stream

STEP = 256


def _round_up(n: int, step: int = STEP) -> int:
    return max(step, (n + step - 1) // step * step)


class _Base:
    bits = 0
    group_size = 64

    def __init__(self, n_kv_heads: int, head_dim: int, device, capacity: int = 0, batch: int = 1):
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.batch = batch
        self.device = torch.device(device)
        self.offset = 0
        self.capacity = 0
        self.generation = 0  # bumps whenever buffers move (invalidates captured graphs)
        if capacity:
            self.reserve(capacity)

    # ---- mlx-lm cache API
    def is_trimmable(self) -> bool:
        return True

    def trim(self, n: int) -> int:
        n = min(self.offset, n)
        self.offset -= n
        return n

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self._tensors())

    @property
    def state(self):
        return self.keys, self.values

    # ---- device plumbing
    def reserve(self, capacity: int) -> None:
        capacity = _round_up(capacity)
        if capacity <= self.capacity:
            return
        old = self._tensors() if self.capacity else None
        new = self._alloc(capacity)
        if old is not None:
            for o, n in zip(old, new):
                n[..., : self.capacity, :].copy_(o[..., : self.capacity, :])
        self._set(new)
        self.capacity = capacity
        self.generation += 1

    def layer_struct(self, seq: Optional[int] = None) -> M5LayerKv:
        """The C-ABI view of this layer: all sequences, or (seq given) sequence
        `seq` alone as a batch-1 layer (per-sequence prefill)."""
        t = self._tensors()
        if seq is not None:
            t = [x[seq] for x in t]
        if len(t) == 2:
            return M5LayerKv(t[0].data_ptr(), None, None, t[1].data_ptr(), None, None, self.capacity, 0,
                             self.group_size)
        return M5LayerKv(t[0].data_ptr(), t[1].data_ptr(), t[2].data_ptr(), t[3].data_ptr(), t[4].data_ptr(),
                         t[5].data_ptr(), self.capacity, self.bits, self.group_size)

    def bytes_per_token(self) -> float:
        return self.nbytes / max(self.capacity, 1)


class KVCache(_Base):
    """Unquantized bf16 cache (mlx-lm ``KVCache``)."""

    def _alloc(self, cap):
        shape = (self.batch, self.n_kv_heads, cap, self.head_dim)
        return [torch.zeros(shape, dtype=torch.bfloat16, device=self.device) for _ in range(2)]

    def _set(self, t):
        self._k, self._v = t

    def _tensors(self):
        return [self._k, self._v] if self.capacity else []

    @property
    def keys(self):
        return self._k if self.capacity else None

    @property
    def values(self):
        return self._v if self.capacity else None

    def update_and_fetch(self, k: torch.Tensor, v: torch.Tensor):
        """Host-driven append of bf16 k/v [1, Hkv, L, D] (tests and tools)."""
        L = k.shape[-2]
        self.reserve(self.offset + L)
        self._k[..., self.offset:self.offset + L, :].copy_(k)
        self._v[..., self.offset:self.offset + L, :].copy_(v)
        self.offset += L
        return self._k[..., : self.offset, :], self._v[..., : self.offset, :]

    def to_quantized(self, group_size: int = 64, bits: int = 4, capacity: Optional[int] = None) -> "QuantizedKVCache":
        qc = QuantizedKVCache(self.n_kv_heads, self.head_dim, self.device, group_size=group_size, bits=bits,
                              capacity=max(capacity or 0, self.capacity, self.offset))
        if self.offset:
            src, dst = self.layer_struct(), qc.layer_struct()
            call("m5_kv_quantize_layer", src, dst, self.n_kv_heads, self.head_dim, self.offset, _stream())
        qc.offset = self.offset
        return qc


class QuantizedKVCache(_Base):
    """Packed 8/4-bit cache (mlx-lm ``QuantizedKVCache``)."""

    def __init__(self, n_kv_heads: int, head_dim: int, device, group_size: int = 64, bits: int = 8,
                 capacity: int = 0, batch: int = 1):
        if bits not in (4, 8) or group_size != 64:
            raise ValueError("quantized KV cache supports bits 4/8 with group_size 64")
        self.bits = bits
        self.group_size = group_size
        super().__init__(n_kv_heads, head_dim, device, capacity, batch)

    def _alloc(self, cap):
        B, H, D = self.batch, self.n_kv_heads, self.head_dim
        out = []
        for _ in range(2):
            out.append(torch.zeros((B, H, cap, D * self.bits // 32), dtype=torch.int32, device=self.device))
            out.append(torch.zeros((B, H, cap, D // self.group_size), dtype=torch.bfloat16, device=self.device))
            out.append(torch.zeros((B, H, cap, D // self.group_size), dtype=torch.bfloat16, device=self.device))
        return out

    def _set(self, t):
        self._kq, self._ks, self._kb, self._vq, self._vs, self._vb = t

    def _tensors(self):
        return [self._kq, self._ks, self._kb, self._vq, self._vs, self._vb] if self.capacity else []

    @property
    def keys(self):
        return (self._kq, self._ks, self._kb) if self.capacity else None

    @property
    def values(self):
        return (self._vq, self._vs, self._vb) if self.capacity else None

    def fetch(self):
        """Trimmed (keys, values) tuples covering positions [0, offset)."""
        o = self.offset
        return (tuple(t[..., :o, :] for t in self.keys), tuple(t[..., :o, :] for t in self.values))


class PromptCache(list):
    """The per-layer cache list (mlx-lm ``make_prompt_cache`` result) plus the
    device-side length counter the forward pass reads and advances."""

    def __init__(self, layers: List[_Base], device):
        super().__init__(layers)
        self.d_len = torch.zeros(1, dtype=torch.int32, device=device)

    @property
    def offset(self) -> int:
        return self[0].offset if len(self) else 0

    def reserve(self, capacity: int) -> None:
        for c in self:
            c.reserve(capacity)

    @property
    def batch(self) -> int:
        return self[0].batch if len(self) else 1

    def structs(self, seq: Optional[int] = None):
        """C-ABI layer views: the whole batch, or one sequence of it."""
        arr = (M5LayerKv * len(self))(*[c.layer_struct(seq) for c in self])
        return arr

    def signature(self):
        """Changes whenever any layer's buffers or format change."""
        return tuple((type(c).__name__, c.generation, c.capacity, c.bits) for c in self)


def make_prompt_cache(model, capacity: int = 0) -> PromptCache:
    a = model.args
    dev = model.device
    return PromptCache([KVCache(model.n_kv_heads_local, a.head_dim, dev, capacity) for _ in range(a.num_hidden_layers)],
                       dev)


def can_trim_prompt_cache(cache) -> bool:
    return all(c.is_trimmable() for c in cache)


def trim_prompt_cache(cache, num_tokens: int) -> int:
    if not can_trim_prompt_cache(cache) or not cache:
        return 0
    return [c.trim(num_tokens) for c in cache][0]
