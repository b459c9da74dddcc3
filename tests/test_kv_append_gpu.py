"""KV quantize-on-append and bf16 -> packed conversion, bit-exact against the
oracle's MLX affine quantizer (m5engine/attention.py:106-112 switches a cache
to mlx-lm's QuantizedKVCache, whose update_and_fetch / to_quantized apply
mx.quantize per token, per kv head, in groups of 64 along head_dim).

The fused append (rope_append_kernel: QK-norm, RoPE, quantize, store) writes
packed rows the host never sees in bf16.  The same model call is therefore
run twice on the same tokens: once over a bf16 cache, once over an 8-bit (or
4-bit) cache.  Layer 0's K/V depend only on the tokens and layer 0's weights,
so both runs see identical bf16 rows there: the prefill chunk goes through
the deterministic tensor-core GEMM, and the decode tokens through the GEMV,
which with hidden size 1024 gives every CTA whole 16-row tiles (reduced in
shared memory in a fixed order, no atomics).  The oracle's quantization of
the bf16 run's rows must then equal the packed run's codes, scales and
biases byte for byte, at every prefill and decode position.
m5_kv_quantize_layer (KVCache.to_quantized) is held to the same bar on every
layer of the bf16 run."""

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle.quant import affine_quantize

pytestmark = pytest.mark.gpu

CFG = dict(model_type="qwen3", hidden_size=1024, num_hidden_layers=2, num_attention_heads=16, num_key_value_heads=8,
           head_dim=128, intermediate_size=1024, vocab_size=2048, tie_word_embeddings=False,
           max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6)
PREFILL, DECODE = 40, 3


@pytest.fixture(scope="module")
def model():
    from myinfer_b200.model import Model, ModelArgs, upload_weights
    host = om.generate_weights(om.Config.from_dict(CFG), seed=17)
    return Model(ModelArgs.from_dict(CFG), upload_weights(host, "cuda"), "cuda", max_tokens=64)


def _run(model, cache, ids):
    model.forward(ids[:PREFILL], cache)
    for i in range(PREFILL, PREFILL + DECODE):
        model.forward(ids[i:i + 1], cache)
    torch.cuda.synchronize()


def _bf16_run(model, ids):
    from myinfer_b200.cache import make_prompt_cache
    cache = make_prompt_cache(model, PREFILL + DECODE)
    _run(model, cache, ids)
    return cache


def _packed(t, n):
    """[1, Hkv, cap, w] device tensor -> host uint32 / uint16 array of the first n positions."""
    a = t[0, :, :n].contiguous().cpu()
    return a.numpy().view(np.uint32) if a.dtype == torch.int32 else a.view(torch.int16).numpy().view(np.uint16)


def _expect_equal(bf16_kv, packed, n, bits, what):
    ref = affine_quantize(bf16_kv[0, :, :n].float().cpu().numpy(), 64, bits)
    for r, got, name in zip(ref, packed, ("codes", "scales", "biases")):
        g = _packed(got, n)
        bad = np.argwhere(g != r)
        assert bad.size == 0, f"{what} {name}: {len(bad)} mismatches, first at (head, pos, word) {bad[0].tolist()}"


@pytest.mark.parametrize("bits", [8, 4])
def test_fused_append_bit_exact(model, bits):
    from myinfer_b200.cache import PromptCache, QuantizedKVCache
    ids = torch.from_numpy(np.random.default_rng(bits).integers(0, CFG["vocab_size"], PREFILL + DECODE)
                           .astype(np.int32)).cuda()
    plain = _bf16_run(model, ids)
    a = model.args
    packed = PromptCache([QuantizedKVCache(model.n_kv_heads_local, a.head_dim, "cuda", 64, bits,
                                           capacity=PREFILL + DECODE) for _ in range(a.num_hidden_layers)], "cuda")
    _run(model, packed, ids)
    n = PREFILL + DECODE
    _expect_equal(plain[0].keys, packed[0].keys, n, bits, "layer 0 keys")
    _expect_equal(plain[0].values, packed[0].values, n, bits, "layer 0 values")


@pytest.mark.parametrize("bits", [8, 4])
def test_kv_quantize_layer_bit_exact(model, bits):
    ids = torch.from_numpy(np.random.default_rng(10 + bits).integers(0, CFG["vocab_size"], PREFILL + DECODE)
                           .astype(np.int32)).cuda()
    plain = _bf16_run(model, ids)
    n = PREFILL + DECODE
    for li, c in enumerate(plain):
        q = c.to_quantized(64, bits)
        torch.cuda.synchronize()
        assert q.offset == n
        _expect_equal(c.keys, q.keys, n, bits, f"layer {li} keys")
        _expect_equal(c.values, q.values, n, bits, f"layer {li} values")
