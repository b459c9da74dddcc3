"""Token sampling: mlx-lm ``make_sampler`` + ``make_logits_processors``, restated.

Test infrastructure only (see ``oracle/__init__``).

Reference call site: m5engine/engine.py:384-392 builds, per request,
``make_sampler(temp, top_p, min_p, top_k)`` and ``make_logits_processors(
repetition_penalty, presence_penalty, frequency_penalty)`` from mlx-lm 0.31.3
(requirements.txt:4; third-party, not vendored under the reference and not
installable here, so this restatement is parity-unpinned against mlx-lm
itself).  mlx-lm's generate_step applies the processors to the bf16 logits
of the last position with the tokens that passed through its sampling step
(the last prompt token, then every generated one), takes
``logprobs = logits - logsumexp(logits)`` and hands them to the sampler, which
applies, in order, top-p (ascending sort, keep where the cumulative
probability exceeds 1 - top_p), min-p (keep logprob >= max + log(min_p)),
top-k (argpartition, keep k) and draws ``categorical(logprobs / temp)``.

Two forms live here:

* ``mlx_kept``: those steps literally (sorts and cumulative sums), for rows
  without ties;
* ``kept_mask``: the threshold form the device kernel implements.  Every
  filter keeps the values at or above a threshold computed on the full row,
  so the three compose to one threshold; ties at a threshold are all kept
  (mlx-lm breaks them by sort order, which a threshold cannot).

The uniform number of a draw is SplitMix64 (Steele, Lea and Flood, OOPSLA
2014) of counter ``offset + row`` under ``seed``, its top 24 bits over 2^24,
and the draw is the inverse CDF over the kept set in index order (mlx-lm
draws with Gumbel noise from MLX's own generator; no two generators agree
token for token, so only the distribution is comparable with mlx-lm).
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np

MASK64 = (1 << 64) - 1


def splitmix64(seed: int, ctr: int) -> int:
    z = (seed + (ctr + 1) * 0x9E3779B97F4A7C15) & MASK64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
    return z ^ (z >> 31)


def uniform(seed: int, ctr: int) -> float:
    return (splitmix64(seed, ctr) >> 40) / float(1 << 24)


def bf16_round(x) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even), returned as fp32."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return (u & 0xFFFFFFFF).astype(np.uint32).view(np.float32)


def apply_penalties(row: np.ndarray, window: Sequence[int], repetition: Optional[float] = None,
                    presence: Optional[float] = None, frequency: Optional[float] = None) -> np.ndarray:
    """mlx-lm's repetition, presence and frequency processors on one bf16-valued
    fp32 row, each rounding its result to bf16.  repetition: x<0 ? x*r : x/r on
    the distinct window tokens; presence: x - p once per distinct token;
    frequency: x - f * (occurrences in the window)."""
    v = np.array(row, dtype=np.float32)
    toks = [int(t) for t in window if 0 <= int(t) < v.size]
    if not toks:
        return v
    uniq, counts = np.unique(np.asarray(toks, dtype=np.int64), return_counts=True)
    if repetition:
        x = v[uniq]
        v[uniq] = bf16_round(np.where(x < 0, x * np.float32(repetition), x / np.float32(repetition)))
    if presence:
        v[uniq] = bf16_round(v[uniq] - np.float32(presence))
    if frequency:
        v[uniq] = bf16_round(v[uniq] - np.float32(frequency) * counts.astype(np.float32))
    return v


# ---------------------------------------------------------------- mlx-lm steps, literally
def _logprobs(v: np.ndarray) -> np.ndarray:
    x = v.astype(np.float64)
    m = x.max()
    return x - (m + np.log(np.exp(x - m).sum()))


def mlx_kept(v: np.ndarray, top_p: float = 0.0, min_p: float = 0.0, top_k: int = 0) -> np.ndarray:
    """Boolean mask of the tokens mlx-lm's filters leave finite (rows without ties)."""
    lp = _logprobs(v)
    if 0 < top_p < 1:
        order = np.argsort(lp, kind="stable")           # ascending
        cum = np.cumsum(np.exp(lp[order]))
        cum_orig = np.empty_like(cum)
        cum_orig[order] = cum
        lp = np.where(cum_orig > 1 - top_p, lp, -np.inf)
    if min_p > 0:
        order = np.argsort(-lp, kind="stable")
        top = lp[order[0]]
        remove = lp < top + np.log(min_p)
        remove[order[0]] = False                         # min_tokens_to_keep = 1
        lp = np.where(remove, -np.inf, lp)
    if 0 < top_k < v.size:
        drop = np.argpartition(-lp, top_k - 1)[top_k:]
        lp = lp.copy()
        lp[drop] = -np.inf
    return np.isfinite(lp)


# ---------------------------------------------------------------- threshold form
def kept_mask(v: np.ndarray, top_p: float = 0.0, min_p: float = 0.0, top_k: int = 0) -> np.ndarray:
    v = np.asarray(v, dtype=np.float32)
    keep = np.ones(v.size, dtype=bool)
    vmax = v.max()
    if 0 < top_p < 1:
        p = np.exp(v.astype(np.float64) - float(vmax))
        uniq, inv = np.unique(v, return_inverse=True)    # ascending values
        mass = np.bincount(inv, weights=p)
        above = np.concatenate([np.cumsum(mass[::-1])[::-1][1:], [0.0]])  # mass strictly above each value
        keep &= (above < top_p * p.sum())[inv]
    if min_p > 0:
        keep &= v >= np.float32(vmax) + np.float32(np.log(np.float32(min_p)))
    if 0 < top_k < v.size:
        kth = np.sort(v)[-top_k]
        keep &= v >= kth
    return keep


def draw(v: np.ndarray, keep: np.ndarray, temp: float, u: float):
    """Inverse-CDF draw: (index, cdf before it, cdf through it, total)."""
    v = np.asarray(v, dtype=np.float64)
    w = np.where(keep, np.exp((v - v[keep].max()) / temp), 0.0)
    cdf = np.cumsum(w)
    total = cdf[-1]
    target = u * total
    i = int(np.searchsorted(cdf, target, side="right"))
    if i >= v.size or w[i] == 0:
        i = int(np.nonzero(w)[0][-1])
    return i, (cdf[i - 1] if i > 0 else 0.0), cdf[i], total


def sample_rows(logits: np.ndarray, temp: float, top_p: float = 0.0, min_p: float = 0.0, top_k: int = 0,
                windows: Optional[List[Sequence[int]]] = None, repetition: Optional[float] = None,
                presence: Optional[float] = None, frequency: Optional[float] = None, seed: int = 0,
                offset: int = 0):
    """Tokens for every row of bf16-valued fp32 ``logits`` [R, V] and the
    penalised rows; temperature <= 0 is greedy (first index of the max)."""
    rows = np.asarray(logits, dtype=np.float32)
    out, pen = [], []
    for r in range(rows.shape[0]):
        v = apply_penalties(rows[r], windows[r] if windows else [], repetition, presence, frequency)
        pen.append(v)
        if temp <= 0:
            out.append(int(np.argmax(v)))
            continue
        keep = kept_mask(v, top_p, min_p, top_k)
        out.append(draw(v, keep, temp, uniform(seed, offset + r))[0])
    return np.asarray(out, dtype=np.int64), np.stack(pen)
