"""Pins of the CPU oracle itself (no GPU).

* blocked attention against dense fp32 attention on dequantized K/V at the
  reference's own tolerance and block forcing (tests/test_core.py:23-40);
* the affine quantizer's invariants and the low-bits-first packing order
  (native/include/tensor.hpp:76-86, native/src/memory_arena.mm:229-238);
* the Qwen3 / Qwen3-MoE restatement against HF transformers run on the same
  dequantized weights: architecture (QK-norm, RoPE convention, GQA, router
  renormalisation, tied head) and the YaRN table, independent of MLX's bf16
  rounding points.
"""

import math

import numpy as np
import pytest
import torch

from oracle import model as OM
from oracle.quant import (affine_dequantize, affine_quantize, bf16_bits_to_f32, bf16_round,
                          f32_to_bf16_bits, unpack)
from oracle.rope import rope_table
from oracle.sdpa import blocked_quantized_sdpa, reference_attention


# ---------------------------------------------------------------- attention
@pytest.mark.parametrize("hq,hk", [(4, 4), (8, 2)])
@pytest.mark.parametrize("mask_kind", ["causal", "bool", None])
def test_blocked_attention_matches_dense(hq, hk, mask_kind):
    g = torch.Generator().manual_seed(0)
    L, S, D = 6, 700, 64
    q = torch.randn(1, hq, L, D, generator=g)
    k = torch.randn(1, hk, S, D, generator=g).numpy()
    v = torch.randn(1, hk, S, D, generator=g).numpy()
    qk, qv = affine_quantize(k, 64, 8), affine_quantize(v, 64, 8)
    kd = torch.from_numpy(affine_dequantize(*qk, 64, 8)).repeat_interleave(hq // hk, dim=1)
    vd = torch.from_numpy(affine_dequantize(*qv, 64, 8)).repeat_interleave(hq // hk, dim=1)
    causal = torch.arange(S - L, S)[:, None] >= torch.arange(S)[None]
    mask = {"causal": "causal", "bool": causal, None: None}[mask_kind]
    # score budget 1 byte -> blocks of MIN_BLOCK=128 keys: 6 blocks, last one ragged
    out = blocked_quantized_sdpa(q, qk, qv, 0.125, mask, 64, 8, score_budget_bytes=1, min_block=128,
                                 dtype="f32")
    ref = reference_attention(q, kd, vd, 0.125, None if mask_kind is None else causal)
    assert (out - ref).abs().max().item() < 1e-4


# ---------------------------------------------------------------- quantizer
@pytest.mark.parametrize("bits", [4, 8])
def test_quantize_invariants(bits):
    rng = np.random.default_rng(1)
    w = bf16_round(rng.standard_normal((33, 256)).astype(np.float32) * 0.05)
    w[0] = 0.0                                   # all-zero groups
    w[1, :64] = 0.25                             # constant group
    w[2, :64] = np.linspace(-1, 1, 64, dtype=np.float32)
    w[3, 64:128] = -w[3, 64:128] ** 2            # one-signed group
    wq, s, b = affine_quantize(w, 64, bits)
    assert wq.dtype == np.uint32 and wq.shape == (33, 256 * bits // 32)
    assert s.dtype == np.uint16 and s.shape == (33, 4) and b.shape == (33, 4)
    q = unpack(wq, bits)
    assert q.max() <= (1 << bits) - 1
    deq = affine_dequantize(wq, s, b, 64, bits)
    sc = np.abs(np.repeat(bf16_bits_to_f32(s), 64, axis=1))
    bb = np.abs(np.repeat(bf16_bits_to_f32(b), 64, axis=1))
    err = np.abs(deq - w)
    slack = (1 << bits) * sc * 2 ** -8 + bb * 2 ** -8 + 1e-7      # bf16 storage of scale and bias
    inner = (q > 0) & (q < (1 << bits) - 1)
    # codes strictly inside the range sit within half a step; making the edge exact
    # (scale = edge / rint(edge / scale)) can shrink the step so the far end clips,
    # by less than one step since |rint(edge / scale)| >= 2**(bits-1)
    assert np.all(err[inner] <= (0.5 * sc + slack)[inner])
    assert np.all(err <= 1.0 * sc + slack)
    # the chosen edge (the larger-magnitude endpoint) is representable: zero stays exact
    assert np.all(deq[0] == 0)
    # packing is low-bits-first: element j of a word at bit j*bits
    per = 32 // bits
    manual = np.zeros_like(wq)
    for j in range(per):
        manual |= q.reshape(33, -1, per)[:, :, j].astype(np.uint32) << np.uint32(j * bits)
    assert np.array_equal(manual, wq)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, np.inf, 65504.0], dtype=np.float32)
    got = bf16_bits_to_f32(f32_to_bf16_bits(x))
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(got, want)


# ---------------------------------------------------------- HF cross-check
def _hf_state(cfg: OM.Config, weights) -> dict:
    m = OM.Model(cfg, weights)
    sd = {}
    for name, shape, kind in OM.weight_specs(cfg):
        if kind == "norm":
            sd[name + ".weight"] = m.norm_w(name)
        elif ".switch_mlp." in name:
            continue
        else:
            sd[name + ".weight"] = m.deq(name)
    if cfg.tie_word_embeddings:
        sd["lm_head.weight"] = m.deq("model.embed_tokens")
    if cfg.moe:
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}.mlp."
            g, u, d = (m.deq(p + "switch_mlp." + n) for n in ("gate_proj", "up_proj", "down_proj"))
            sd[p + "experts.gate_up_proj"] = torch.cat([g, u], dim=1)
            sd[p + "experts.down_proj"] = d
    return sd, m


def _hf_model(cfg: OM.Config, sd: dict, yarn: float = 1.0):
    tr = pytest.importorskip("transformers")
    rope = {"rope_type": "default", "rope_theta": cfg.rope_theta}
    if yarn > 1:
        rope = {"rope_type": "yarn", "rope_theta": cfg.rope_theta, "factor": yarn,
                "original_max_position_embeddings": 32768}
    common = dict(vocab_size=cfg.vocab_size, hidden_size=cfg.hidden_size,
                  num_hidden_layers=cfg.num_hidden_layers, num_attention_heads=cfg.num_attention_heads,
                  num_key_value_heads=cfg.num_key_value_heads, head_dim=cfg.head_dim,
                  rms_norm_eps=cfg.rms_norm_eps, tie_word_embeddings=cfg.tie_word_embeddings,
                  max_position_embeddings=32768 * max(1, int(yarn)), rope_parameters=rope,
                  attn_implementation="eager", torch_dtype=torch.float32)
    if cfg.moe:
        hc = tr.Qwen3MoeConfig(intermediate_size=cfg.moe_intermediate_size,
                               moe_intermediate_size=cfg.moe_intermediate_size, num_experts=cfg.num_experts,
                               num_experts_per_tok=cfg.num_experts_per_tok, norm_topk_prob=cfg.norm_topk_prob,
                               decoder_sparse_step=1, mlp_only_layers=[], **common)
        model = tr.Qwen3MoeForCausalLM(hc)
    else:
        hc = tr.Qwen3Config(intermediate_size=cfg.intermediate_size, **common)
        model = tr.Qwen3ForCausalLM(hc)
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in k for k in missing), (missing, unexpected)
    return model.float().eval()


DENSE = OM.Config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                  head_dim=128, intermediate_size=512, vocab_size=512, tie_word_embeddings=True)
MOE = OM.Config(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                head_dim=128, intermediate_size=0, vocab_size=512, num_experts=8, num_experts_per_tok=2,
                moe_intermediate_size=128)


@pytest.mark.parametrize("cfg,yarn", [(DENSE, 1.0), (DENSE, 4.0), (MOE, 1.0)], ids=["dense", "yarn4", "moe"])
def test_oracle_matches_transformers(cfg, yarn):
    """Same weights, same tokens: logits of the oracle (bf16 rounding at every
    MLX array boundary) and of HF transformers (fp32 throughout) agree to bf16
    noise; the argmax token agrees wherever the top-2 gap exceeds that noise."""
    weights = OM.generate_weights(cfg, seed=7, std=0.05)
    sd, om = _hf_state(cfg, weights)
    if yarn > 1:
        om.set_rope(yarn, 32768)
    hf = _hf_model(cfg, sd, yarn)
    tokens = list(np.random.default_rng(3).integers(0, cfg.vocab_size, 24))
    cache = [OM.KVCache() for _ in range(cfg.num_hidden_layers)]
    ours = om(tokens, cache)                                    # [L, V]
    with torch.no_grad():
        ref = hf(torch.tensor([tokens])).logits[0].float()
    cos = torch.nn.functional.cosine_similarity(ours, ref, dim=-1)
    assert cos.min().item() > 0.999, cos
    err = (ours - ref).abs().max().item()
    assert err < 0.05 * ref.abs().max().item(), err
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > 4 * err
    assert torch.equal(ours.argmax(-1)[clear], ref.argmax(-1)[clear])


def test_yarn_table_matches_transformers():
    tr = pytest.importorskip("transformers")
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    for f in (2.0, 4.0):
        hc = tr.Qwen3Config(head_dim=128, hidden_size=256, num_attention_heads=2,
                            max_position_embeddings=int(32768 * f),
                            rope_parameters={"rope_type": "yarn", "rope_theta": 1e6, "factor": f,
                                             "original_max_position_embeddings": 32768})
        inv, att = ROPE_INIT_FUNCTIONS["yarn"](hc, "cpu")
        ours, ms = rope_table(128, 1e6, f, 32768)
        np.testing.assert_allclose(ours, inv.float().numpy(), rtol=2e-7)
        assert math.isclose(ms, att, rel_tol=1e-12)
