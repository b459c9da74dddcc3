"""Quantized-KV attention (m5_quantized_sdpa through blocked_quantized_sdpa)
against the CPU restatement of m5engine/attention.py.

Bar: the device rounds scores and p to bf16 at the reference's points
(attention.py:66-69, 87-90) but normalises p only at the end of its split-KV
merge, sums in another order and over other key blocks, and rounds the output
to bf16.  Each of those moves an output by a fraction of a bf16 step, so the
test asks |d| <= 2^-7 |ref| + 1e-2 std(ref) (two bf16 steps of the value
itself, plus a floor of 1 % of the output's spread for values near zero) of
99.9 % of the elements, cosine >= 0.9999 over the whole output, and
|d| <= 2^-7 |ref| + 5e-2 std(ref) of every element.  The last bound is wider
because a score whose fp32 value sits on a bf16 rounding boundary rounds one
way here and the other way in the oracle (their fp32 dot products differ in
the last bits): one bf16 step of a score of magnitude s changes its weight
exp(s) by s * 2^-8, about 1-2 % for the scores of these inputs, which moves a
row dominated by few keys by that much.  The grid covers the
reference's own test (tests/test_core.py:23-40), every GQA shape of the
configs, and the attention microbenchmark's shapes (64 q / 8 kv heads,
8- and 4-bit keys and values, decode at 4K / 32K / 128K keys, a 2048-token
causal prefill chunk over 4K keys)."""

import numpy as np
import pytest
import torch

from oracle.quant import affine_dequantize, affine_quantize, bf16_bits_to_f32, f32_to_bf16_bits
from oracle.sdpa import blocked_quantized_sdpa as ref_blocked
from oracle.sdpa import dense_quantized_sdpa as ref_dense
from oracle.sdpa import reference_attention

pytestmark = pytest.mark.gpu


def _bf16(a):
    return bf16_bits_to_f32(f32_to_bf16_bits(a.astype(np.float32)))


def _kv(rng, B, Hkv, S, D, bits):
    k = _bf16(rng.standard_normal((B, Hkv, S, D)))
    v = _bf16(rng.standard_normal((B, Hkv, S, D)))
    if bits == 0:
        return k, v, torch.from_numpy(k), torch.from_numpy(v)
    qk = affine_quantize(k, 64, bits)
    qv = affine_quantize(v, 64, bits)
    return qk, qv, None, None


def _check(out, ref):
    """99.9 % of |d| <= 2^-7 |ref| + 1e-2 std(ref), all |d| <= 2^-7 |ref| +
    5e-2 std(ref), cosine >= 0.9999."""
    out, ref = out.float().cpu().reshape(-1), ref.float().cpu().reshape(-1)
    err = (out - ref).abs()
    std = ref.std()
    tight = err <= ref.abs() * 2 ** -7 + 1e-2 * std
    assert tight.float().mean().item() >= 0.999, (tight.float().mean().item(), float(err.max()), float(std))
    wide = ref.abs() * 2 ** -7 + 5e-2 * std
    worst = int((err - wide).argmax())
    assert bool((err <= wide).all()), (float(err[worst]), float(ref[worst]), float(std))
    cos = torch.nn.functional.cosine_similarity(out, ref, dim=0).item()
    assert cos >= 0.9999, cos


def _dev(t):
    wq, s, b = t
    return (torch.from_numpy(wq.view(np.int32)).cuda(), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).cuda(),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).cuda())


@pytest.mark.parametrize("hq,hk", [(4, 4), (8, 2)])
@pytest.mark.parametrize("mask_kind", ["causal", "bool", None])
def test_reference_grid(hq, hk, mask_kind):
    """The grid of tests/test_core.py:23-40 (L=6, S=700, D=64, 8-bit g64)."""
    from myinfer_b200.attention import blocked_quantized_sdpa
    rng = np.random.default_rng(0)
    L, S, D = 6, 700, 64
    q = _bf16(rng.standard_normal((1, hq, L, D)))
    qk, qv, _, _ = _kv(rng, 1, hk, S, D, 8)
    causal = torch.arange(S - L, S)[:, None] >= torch.arange(S)[None]
    mask = {"causal": "causal", "bool": causal, None: None}[mask_kind]
    dmask = mask.cuda() if isinstance(mask, torch.Tensor) else mask
    out = blocked_quantized_sdpa(torch.from_numpy(q).to(torch.bfloat16).cuda(), _dev(qk), _dev(qv), 0.125, dmask,
                                 64, 8).float().cpu()
    oracle = ref_blocked(torch.from_numpy(q), qk, qv, 0.125, mask, 64, 8, score_budget_bytes=1, min_block=128)
    kd = torch.from_numpy(affine_dequantize(*qk, 64, 8)).repeat_interleave(hq // hk, dim=1)
    vd = torch.from_numpy(affine_dequantize(*qv, 64, 8)).repeat_interleave(hq // hk, dim=1)
    dense = reference_attention(torch.from_numpy(q), kd, vd, 0.125, None if mask_kind is None else causal)
    _check(out, oracle)
    # the reference's own test compares blocked with dense fp32 attention (no
    # bf16 rounding at all) at 1e-4; with the bf16 rounding points of the
    # real op the distance to fp32 is a bf16-sized one
    assert (out - dense).abs().max().item() < 2e-2


@pytest.mark.parametrize("bits", [8, 4, 0])
@pytest.mark.parametrize("hq,hk,S", [(64, 8, 4096), (16, 8, 700), (32, 4, 2500), (64, 4, 1500)])
def test_decode(bits, hq, hk, S):
    """L == 1 (mlx-lm's dense quantized SDPA path), GQA groups of the BASELINE configs."""
    from myinfer_b200.attention import blocked_quantized_sdpa
    rng = np.random.default_rng(S + hq)
    D = 128
    q = _bf16(rng.standard_normal((1, hq, 1, D)))
    k, v, kt, vt = _kv(rng, 1, hk, S, D, bits)
    qd = torch.from_numpy(q).to(torch.bfloat16).cuda()
    if bits:
        out = blocked_quantized_sdpa(qd, _dev(k), _dev(v), D ** -0.5, None, 64, bits)
        oracle = ref_dense(torch.from_numpy(q), k, v, D ** -0.5, None, 64, bits)
    else:
        out = blocked_quantized_sdpa(qd, kt.to(torch.bfloat16).cuda(), vt.to(torch.bfloat16).cuda(), D ** -0.5, None)
        oracle = ref_dense(torch.from_numpy(q), kt, vt, D ** -0.5, None)
    _check(out, oracle)


@pytest.mark.parametrize("bits", [8, 4])
def test_prefill_chunk_causal(bits):
    """L > 1 causal chunk at the end of a longer cache (blocked path)."""
    from myinfer_b200.attention import blocked_quantized_sdpa
    rng = np.random.default_rng(11)
    hq, hk, L, S, D = 16, 8, 200, 1200, 128
    q = _bf16(rng.standard_normal((1, hq, L, D)))
    k, v, _, _ = _kv(rng, 1, hk, S, D, bits)
    out = blocked_quantized_sdpa(torch.from_numpy(q).to(torch.bfloat16).cuda(), _dev(k), _dev(v), D ** -0.5,
                                 "causal", 64, bits)
    oracle = ref_blocked(torch.from_numpy(q), k, v, D ** -0.5, "causal", 64, bits, score_budget_bytes=1,
                         min_block=256)
    _check(out, oracle)


def test_additive_mask():
    from myinfer_b200.attention import blocked_quantized_sdpa
    rng = np.random.default_rng(3)
    hq, hk, L, S, D = 8, 2, 4, 300, 128
    q = _bf16(rng.standard_normal((1, hq, L, D)))
    k, v, _, _ = _kv(rng, 1, hk, S, D, 8)
    add = torch.from_numpy(rng.standard_normal((1, 1, L, S)).astype(np.float32))
    out = blocked_quantized_sdpa(torch.from_numpy(q).to(torch.bfloat16).cuda(), _dev(k), _dev(v), D ** -0.5,
                                 add.cuda(), 64, 8)
    oracle = ref_blocked(torch.from_numpy(q), k, v, D ** -0.5, add, 64, 8, score_budget_bytes=1, min_block=128)
    _check(out, oracle)


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("hq,hk,L,S,mask", [(64, 8, 64, 1500, "causal"), (64, 8, 33, 700, "causal"),
                                            (32, 4, 300, 2100, "causal"), (64, 4, 17, 900, "causal"),
                                            (16, 8, 130, 130, "causal"), (64, 8, 40, 500, None)])
def test_prefill_tensor_core(bits, hq, hk, L, S, mask):
    """Prefill kernel (128 rows per CTA, every GQA group size of the BASELINE
    configs, ragged tails, split-KV on small grids) against the blocked oracle."""
    from myinfer_b200.attention import blocked_quantized_sdpa
    rng = np.random.default_rng(L * 7 + S + bits)
    D = 128
    q = _bf16(rng.standard_normal((1, hq, L, D)))
    k, v, _, _ = _kv(rng, 1, hk, S, D, bits)
    out = blocked_quantized_sdpa(torch.from_numpy(q).to(torch.bfloat16).cuda(), _dev(k), _dev(v), D ** -0.5,
                                 mask, 64, bits)
    oracle = ref_blocked(torch.from_numpy(q), k, v, D ** -0.5, mask, 64, bits, score_budget_bytes=1,
                         min_block=256)
    _check(out, oracle)


_LONG = {}


def _long_kv(S, bits):
    """Seeded N(0,1) bf16 keys / values [1, 8, S, 128] quantized to `bits`
    (generated once per length and shared by the 8- and 4-bit cases)."""
    if S not in _LONG:
        _LONG.clear()
        rng = np.random.default_rng(S)
        _LONG[S] = {"k": _bf16(rng.standard_normal((1, 8, S, 128), dtype=np.float32)),
                    "v": _bf16(rng.standard_normal((1, 8, S, 128), dtype=np.float32))}
    d = _LONG[S]
    if bits not in d:
        d[bits] = (affine_quantize(d["k"], 64, bits), affine_quantize(d["v"], 64, bits))
    return d[bits]


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("S", [32768, 131072])
def test_decode_long_context(S, bits):
    """The attention microbenchmark's decode shapes: 64 q / 8 kv heads at 32K
    and 128K keys, 8- and 4-bit cache (one query row, split-KV + merge)."""
    from myinfer_b200.attention import blocked_quantized_sdpa
    k, v = _long_kv(S, bits)
    q = _bf16(np.random.default_rng(S + bits).standard_normal((1, 64, 1, 128), dtype=np.float32))
    out = blocked_quantized_sdpa(torch.from_numpy(q).to(torch.bfloat16).cuda(), _dev(k), _dev(v), 128 ** -0.5,
                                 None, 64, bits)
    _check(out, ref_dense(torch.from_numpy(q), k, v, 128 ** -0.5, None, 64, bits))


@pytest.mark.parametrize("bits", [8, 4])
def test_prefill_chunk_2048(bits):
    """The microbenchmark's prefill shape: a causal 2048-token chunk at the end
    of 4096 keys, 64 q / 8 kv heads (the reference's blocked loop, 341-key
    blocks at this size)."""
    from myinfer_b200.attention import blocked_quantized_sdpa
    S, L = 4096, 2048
    k, v = _long_kv(S, bits)
    q = _bf16(np.random.default_rng(L + bits).standard_normal((1, 64, L, 128), dtype=np.float32))
    out = blocked_quantized_sdpa(torch.from_numpy(q).to(torch.bfloat16).cuda(), _dev(k), _dev(v), 128 ** -0.5,
                                 "causal", 64, bits)
    _check(out, ref_blocked(torch.from_numpy(q), k, v, 128 ** -0.5, "causal", 64, bits))
