"""Token sampling on the device: the mlx-lm ``make_sampler`` /
``make_logits_processors`` surface the reference builds per request
(m5engine/engine.py:384-392), served by one libm5cuda kernel
(``m5_sample_bf16``) per call.

The processors are not separate callables here: ``make_logits_processors``
returns the penalty settings, and ``DeviceSampler`` applies them inside the
sampling kernel on the bf16 logits (in place, as mlx-lm's processors return
the processed logits) before top-p / min-p / top-k and the draw at the
temperature.  The penalty window holds the tokens that passed through the
sampling step, as mlx-lm's generate_step feeds its processors: the last
prompt token, then every generated token.

Random numbers: each sampler owns a 64-bit seed (``seed=`` or drawn from a
module stream that ``seed()`` resets, like ``mx.random.seed``) and a draw
counter in device memory that every call advances by its row count, so a
sampling step captured in a CUDA graph draws new numbers on every replay.
"""

from __future__ import annotations

import os
import random
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional

import torch

from . import _lib
from ._lib import M5SampleParams, call

_MASK64 = (1 << 64) - 1
_seed_source = random.Random(int.from_bytes(os.urandom(8), "little"))


def seed(s: int) -> None:
    """``mx.random.seed``: samplers built afterwards without an explicit seed
    draw their seeds from a stream fixed by ``s``."""
    _seed_source.seed(int(s))


@dataclass(frozen=True)
class LogitsPenalty:
    """One entry of ``make_logits_processors``' list."""
    kind: str            # "repetition" | "presence" | "frequency"
    value: float
    context_size: int = 20


def make_logits_processors(repetition_penalty: Optional[float] = None, repetition_context_size: int = 20,
                           presence_penalty: Optional[float] = None, presence_context_size: int = 20,
                           frequency_penalty: Optional[float] = None,
                           frequency_context_size: int = 20) -> List[LogitsPenalty]:
    """mlx-lm ``make_logits_processors``: an entry per penalty that is set and nonzero."""
    out: List[LogitsPenalty] = []
    for kind, value, ctx in (("repetition", repetition_penalty, repetition_context_size),
                             ("presence", presence_penalty, presence_context_size),
                             ("frequency", frequency_penalty, frequency_context_size)):
        if value and value != 0.0:
            if not isinstance(value, (int, float)) or (kind == "repetition" and value < 0):
                raise ValueError(f"{kind} penalty must be a non-negative float, got {value!r}")
            if int(ctx) < 1 or int(ctx) > 1024:
                raise ValueError(f"{kind}_context_size must be in [1, 1024]")
            out.append(LogitsPenalty(kind, float(value), int(ctx)))
    return out


class DeviceSampler:
    """``make_sampler(temp, top_p, min_p, top_k)`` plus the penalties of
    ``make_logits_processors``, as one kernel over bf16 logits rows."""

    def __init__(self, temp: float = 0.0, top_p: float = 0.0, min_p: float = 0.0, top_k: int = 0,
                 processors: Iterable[LogitsPenalty] = (), seed: Optional[int] = None):
        if not isinstance(top_k, int) or top_k < 0:
            raise ValueError(f"top_k must be a non-negative int, got {top_k!r}")
        if min_p and not (0.0 <= min_p <= 1.0):
            raise ValueError(f"min_p must be a float between 0 and 1, got {min_p}")
        self.temp, self.top_p, self.min_p, self.top_k = float(temp), float(top_p), float(min_p), top_k
        procs = list(processors)
        sizes = {p.context_size for p in procs}
        if len(sizes) > 1:
            raise ValueError("penalties with different context sizes are not supported by the device sampler")
        self.window = sizes.pop() if sizes else 0
        vals = {p.kind: p.value for p in procs}
        self.repetition = vals.get("repetition", 1.0)
        self.presence = vals.get("presence", 0.0)
        self.frequency = vals.get("frequency", 0.0)
        self.seed = (int(seed) if seed is not None else _seed_source.getrandbits(64)) & _MASK64
        self._state: Dict[torch.device, torch.Tensor] = {}

    @property
    def greedy(self) -> bool:
        return self.temp <= 0

    def state(self, device) -> torch.Tensor:
        """The device draw counter {count, CTAs done} (create it before a graph capture)."""
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if dev not in self._state:
            self._state[dev] = torch.zeros(2, dtype=torch.int64, device=dev)
        return self._state[dev]

    def history(self, tokens: List[int], device, rows: int = 1) -> Optional[torch.Tensor]:
        """A [rows, window] int32 penalty window holding the last ``window`` of
        ``tokens`` (oldest first, -1 where empty); None without penalties."""
        if self.window == 0:
            return None
        tail = [int(t) for t in tokens[-self.window:]]
        row = [-1] * (self.window - len(tail)) + tail
        return torch.tensor([row] * rows, dtype=torch.int32).to(device)

    def __call__(self, logits: torch.Tensor, history: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None, append: bool = False) -> torch.Tensor:
        """One token per row of bf16 CUDA ``logits`` ([V] or [R, V]; penalised in
        place).  ``history`` [R, window] int32 (None: no penalties); ``append``
        rolls each window left and ends it with the drawn token.  Returns int32 [R]."""
        if not logits.is_cuda or logits.dtype != torch.bfloat16:
            raise ValueError("DeviceSampler takes bf16 CUDA logits")
        lg = logits if logits.dim() == 2 else logits.reshape(1, -1)
        if lg.stride(-1) != 1:
            raise ValueError("logits rows must be contiguous")
        R, V = lg.shape
        if self.top_k >= V and self.temp > 0:
            raise ValueError(f"top_k must be in (0, {V}), got {self.top_k}")
        if out is None:
            out = torch.empty(R, dtype=torch.int32, device=lg.device)
        hist_ptr, hist_len, hist_ld = None, 0, 0
        if history is not None and self.window > 0:
            h = history if history.dim() == 2 else history.reshape(1, -1)
            if h.dtype != torch.int32 or not h.is_cuda or h.shape[0] != R or h.stride(-1) != 1:
                raise ValueError("history must be int32 CUDA [rows, window] with contiguous rows")
            # a single row's stride is meaningless (torch keeps any stride on a size-1 dimension)
            hist_ptr, hist_len, hist_ld = h.data_ptr(), h.shape[1], h.stride(0) if R > 1 else h.shape[1]
        elif append:
            raise ValueError("append needs a history window")
        p = M5SampleParams(temperature=self.temp, top_p=self.top_p, min_p=self.min_p, top_k=self.top_k,
                           repetition_penalty=self.repetition, presence_penalty=self.presence,
                           frequency_penalty=self.frequency,
                           flags=_lib.M5_SAMPLE_APPEND_HISTORY if append else 0, seed=self.seed, offset=0)
        call("m5_sample_bf16", lg.data_ptr(), R, V, lg.stride(0) if R > 1 else V, hist_ptr, hist_len, hist_ld, p,
             self.state(lg.device).data_ptr(), out.data_ptr(), torch.cuda.current_stream(lg.device).cuda_stream)
        return out


def make_sampler(temp: float = 0.0, top_p: float = 0.0, min_p: float = 0.0, top_k: int = 0,
                 seed: Optional[int] = None) -> Optional[DeviceSampler]:
    """mlx-lm ``make_sampler``: None for temperature 0 (the token loop's greedy
    argmax, captured with the decode step), else a ``DeviceSampler``."""
    if temp <= 0:
        return None
    return DeviceSampler(temp, top_p, min_p, top_k, seed=seed)


def with_processors(sampler, processors: Optional[Iterable[LogitsPenalty]]):
    """The sampler a token loop runs: ``sampler`` with the penalties folded in
    (a greedy ``DeviceSampler`` when only penalties are given).  Other
    callables are returned unchanged and must not be combined with penalties."""
    procs = list(processors or [])
    if not procs:
        return sampler
    if sampler is None:
        return DeviceSampler(0.0, processors=procs)
    if isinstance(sampler, DeviceSampler):
        return DeviceSampler(sampler.temp, sampler.top_p, sampler.min_p, sampler.top_k, procs, sampler.seed)
    raise ValueError("logits processors need a DeviceSampler (make_sampler) or the greedy default")
