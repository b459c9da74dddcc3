"""RoPE / YaRN tables, restated (test infrastructure only).

m5engine/context.py:94-121 (``apply_yarn``) replaces each default RoPE with
mlx-lm ``initialize_rope(dims, base, traditional, scaling_config={"rope_type":
"yarn", "factor": f, "original_max_position_embeddings": native})``.  The YaRN
rule restated here is the published one (Peng et al., "YaRN", 2023) with the
defaults that call leaves in place: beta_fast = 32, beta_slow = 1,
mscale = 1, mscale_all_dim = 0.  Qwen3 uses the split-half (non-traditional)
rotation with theta = 1e6.

Both the oracle and the device path consume the same fp32 ``inv_freq`` table
(built here in fp64, rounded once), so only sin/cos evaluation can differ.
"""

from __future__ import annotations

import math

import numpy as np


def plain_inv_freq(dims: int, base: float) -> np.ndarray:
    i = np.arange(0, dims, 2, dtype=np.float64)
    return (1.0 / (base ** (i / dims))).astype(np.float32)


def yarn_mscale(factor: float) -> float:
    """Magnitude correction multiplied into q and k (0.1 ln f + 1; 1 for f <= 1)."""
    if factor <= 1:
        return 1.0
    return 0.1 * math.log(factor) + 1.0


def yarn_inv_freq(dims: int, base: float, factor: float, original_max_pos: int,
                  beta_fast: float = 32.0, beta_slow: float = 1.0) -> np.ndarray:
    if factor <= 1:
        return plain_inv_freq(dims, base)

    def corr_dim(n_rot: float) -> float:
        return (dims * math.log(original_max_pos / (n_rot * 2 * math.pi))) / (2 * math.log(base))

    low = max(math.floor(corr_dim(beta_fast)), 0)
    high = min(math.ceil(corr_dim(beta_slow)), dims - 1)
    if low == high:
        high += 0.001
    half = dims // 2
    ramp = np.clip((np.arange(half, dtype=np.float64) - low) / (high - low), 0.0, 1.0)
    keep = 1.0 - ramp                      # 1: keep the original frequency
    period = base ** (np.arange(0, dims, 2, dtype=np.float64) / dims)
    inv = keep / period + (1.0 - keep) / (factor * period)
    return inv.astype(np.float32)


def rope_table(dims: int, base: float, factor: float = 1.0, native: int = 32768):
    """(inv_freq fp32 [dims/2], mscale) for plain RoPE (factor<=1) or YaRN."""
    if factor <= 1:
        return plain_inv_freq(dims, base), 1.0
    return yarn_inv_freq(dims, base, factor, native), yarn_mscale(factor)
