"""Speculative decoding with a draft model (speculative_generate_step, the
engine's draft_model option) against the main model's plain greedy decode and
the oracle's greedy tokens for the main model.

With greedy sampling the accepted tokens are the main model's own choices, so
the streams are equal.  The verify call scores 1 + k tokens at once (an
MT = k + 1 GEMV) where the plain decode scores one per call, so logits differ
by fp32 summation order: the streams may part only at a step whose top-2 logit
gap in the plain run is below 0.02, and are compared up to there."""

import json

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAIN = dict(model_type="qwen3", hidden_size=512, num_hidden_layers=3, num_attention_heads=8, num_key_value_heads=2,
            head_dim=128, intermediate_size=1024, vocab_size=4096, tie_word_embeddings=False,
            max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6)
DRAFT = dict(MAIN, hidden_size=256, num_hidden_layers=2, num_attention_heads=4, intermediate_size=512)


def _model(cfg, seed, with_oracle=False):
    from myinfer_b200.model import Model, ModelArgs, upload_weights
    from oracle import model as om
    host = om.generate_weights(om.Config.from_dict(cfg), seed)
    m = Model(ModelArgs.from_dict(cfg), upload_weights(host, "cuda"), "cuda", max_tokens=64)
    return (m, om.Model(om.Config.from_dict(cfg), host)) if with_oracle else m


def _plain(model, prompt, n):
    from myinfer_b200.generate import generate_step
    out = list(generate_step(prompt, model, n, prefill_step_size=16, kv_bits=8, quantized_kv_start=0,
                             return_logits=True))
    return [t for t, _ in out], [l.float().cpu() for _, l in out]


def _agree(spec, plain, logits):
    """Equal up to the first step whose plain top-2 gap is a near-tie."""
    for i, (a, b) in enumerate(zip(spec, plain)):
        if a != b:
            top2 = logits[i].topk(2).values
            assert (top2[0] - top2[1]).item() < 0.02, (i, a, b)
            return i
    return len(plain)


@pytest.mark.parametrize("k", [1, 3, 5])
def test_speculative_equals_greedy(k):
    from myinfer_b200.generate import speculative_generate_step
    from myinfer_b200.cache import make_prompt_cache
    from oracle import model as om
    (main, ora), draft = _model(MAIN, 31, with_oracle=True), _model(DRAFT, 32)
    prompt = np.random.default_rng(k).integers(0, MAIN["vocab_size"], 30).tolist()
    n = 24
    plain, logits = _plain(main, prompt, n)
    got = list(speculative_generate_step(prompt, main, draft, num_draft_tokens=k, max_tokens=n,
                                         prompt_cache=make_prompt_cache(main), draft_cache=make_prompt_cache(draft),
                                         prefill_step_size=16, kv_bits=8, quantized_kv_start=0))
    assert len(got) == n
    _agree([t for t, _ in got], plain, logits)
    # and the oracle's greedy tokens for the main model, up to its first near-tie
    toks_o, _, logits_o = om.generate(ora, prompt, n, prefill_step=16, kv_bits=8, quantized_kv_start=0,
                                      return_logits=True)
    _agree([t for t, _ in got], toks_o, list(logits_o))


def test_self_draft_accepts_everything():
    """The main model as its own draft: every proposal is the main model's
    choice, so all but the round-closing tokens come from the draft."""
    from myinfer_b200.generate import speculative_generate_step
    from myinfer_b200.cache import make_prompt_cache
    main = _model(MAIN, 33)
    prompt = list(range(5, 40))
    n, k = 20, 4
    plain, logits = _plain(main, prompt, n)
    got = list(speculative_generate_step(prompt, main, main, num_draft_tokens=k, max_tokens=n,
                                         prompt_cache=make_prompt_cache(main), draft_cache=make_prompt_cache(main),
                                         prefill_step_size=16, kv_bits=8, quantized_kv_start=0))
    _agree([t for t, _ in got], plain, logits)
    # k proposals accepted per round plus the round's own token: n - n / (k + 1)
    # from the draft, less any proposal rejected at a near-tie of the two calls
    assert sum(d for _, d in got) >= n - n // (k + 1) - 3


def test_engine_draft_model(tmp_path):
    from myinfer_b200.engine import Engine, GenerationParams, LoadOptions
    pm, pd = tmp_path / "main.json", tmp_path / "draft.json"
    pm.write_text(json.dumps(MAIN))
    pd.write_text(json.dumps(DRAFT))
    eng = Engine()
    eng.load(LoadOptions(model=f"random:{pm}", draft_model=f"random:{pd}", num_draft_tokens=3, kv_bits=8,
                         quantized_kv_start=0, memory_budget_gb=4.0, prefill_step=64, seed=5))
    try:
        prompt = eng.encode_text("speculative decoding keeps the main model's greedy tokens")
        chunks = list(eng.generate(prompt, GenerationParams(max_tokens=16, temperature=0.0, use_prefix_cache=False)))
        plain = list(eng.generate(prompt, GenerationParams(max_tokens=16, temperature=0.0, use_draft=False,
                                                           use_prefix_cache=False)))
        m = chunks[-1].metrics
        assert m.completion_tokens == 16 and 0 <= m.draft_accepted <= 16
        assert plain[-1].metrics.completion_tokens == 16 and plain[-1].metrics.draft_accepted == 0
        # prefix reuse keeps both models' layers
        list(eng.generate(prompt, GenerationParams(max_tokens=4, temperature=0.0)))
        follow = prompt + eng.encode_text(" more")
        chunks2 = list(eng.generate(follow, GenerationParams(max_tokens=4, temperature=0.0)))
        assert chunks2[-1].metrics.cached_tokens == len(prompt)
        assert eng.benchmark(prompt_tokens=64, gen_tokens=8)["draft_model"] is not None
    finally:
        eng.unload()
