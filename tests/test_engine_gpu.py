"""Engine surface on the device: load a seeded random model, generate, reuse a
prefix, plan the context, benchmark (m5engine/engine.py:192-553 contract)."""

import json

import pytest
import torch

pytestmark = pytest.mark.gpu

# Hidden and intermediate sizes of 1024: every decode GEMV tile (16 rows x K)
# stays inside one CTA and reduces in shared memory in a fixed order, so two
# runs of the same request are bitwise equal and a seed reproduces its
# sampled text.  (Where a tile is split over CTAs the partial sums meet in
# fp32 atomics in no fixed order, and logits may differ in the last bit.)
TINY = dict(model_type="qwen3", hidden_size=1024, num_hidden_layers=3, num_attention_heads=8, num_key_value_heads=2,
            head_dim=128, intermediate_size=1024, vocab_size=4096, tie_word_embeddings=False,
            max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6)


@pytest.fixture(scope="module")
def engine(tmp_path_factory):
    from myinfer_b200.engine import Engine, LoadOptions
    p = tmp_path_factory.mktemp("cfg") / "config.json"
    p.write_text(json.dumps(TINY))
    eng = Engine()
    info = eng.load(LoadOptions(model=f"random:{p}", kv_bits=8, quantized_kv_start=0, memory_budget_gb=4.0,
                                prefill_step=64, seed=5))
    assert info["state"] == "ready" and info["context"]["max_context"] >= 512
    yield eng
    eng.unload()


def _run(eng, tokens, n, **kw):
    from myinfer_b200.engine import GenerationParams
    chunks = list(eng.generate(tokens, GenerationParams(max_tokens=n, temperature=0.0, **kw)))
    assert chunks[-1].finish_reason in ("length", "stop")
    return "".join(c.text for c in chunks), chunks[-1].metrics


def test_generate_matches_token_loop(engine):
    from myinfer_b200.cache import make_prompt_cache
    from myinfer_b200.generate import generate_step
    prompt = engine.encode_text("The quick brown fox jumps over the lazy dog. " * 3)
    text, m = _run(engine, prompt, 12, use_prefix_cache=False)
    assert m.prompt_tokens == len(prompt) and m.completion_tokens == 12 and m.cached_tokens == 0
    assert m.decode_tps > 0 and m.prompt_tps > 0
    toks = [t for t, _ in generate_step(prompt, engine.model, 12, prompt_cache=make_prompt_cache(engine.model),
                                        prefill_step_size=64, kv_bits=8, quantized_kv_start=0)]
    assert text == engine.tokenizer.decode(toks)


def test_prefix_cache_reuse(engine):
    engine.prefix.clear()
    base = engine.encode_text("A long shared system prompt that both requests start with. " * 2)
    _, m1 = _run(engine, base, 8)
    assert m1.cached_tokens == 0 and len(engine.prefix) == 1
    follow = base + engine.encode_text(" And a follow-up question?")
    _, m2 = _run(engine, follow, 8)
    # the first request's prompt is a prefix of the second: reused without re-prefill
    assert m2.cached_tokens == len(base)
    assert engine.prefix.total_hit_tokens >= len(base)
    # the reused cache was trimmed back, not copied: one entry per key
    assert len(engine.prefix) == 1


def test_stop_strings_and_errors(engine):
    from myinfer_b200.engine import ContextOverflow, GenerationParams
    prompt = engine.encode_text("stop test")
    full, _ = _run(engine, prompt, 10, use_prefix_cache=False)
    if len(full) > 3:
        cut = full[2:4]
        chunks = list(engine.generate(prompt, GenerationParams(max_tokens=10, temperature=0.0, stop=[cut],
                                                               use_prefix_cache=False)))
        text = "".join(c.text for c in chunks)
        assert cut not in text and chunks[-1].finish_reason == "stop"
    with pytest.raises(ContextOverflow):
        next(iter(engine.generate([5] * (engine.plan.max_context + 1), GenerationParams(max_tokens=1))))


def test_sampling_and_benchmark(engine):
    from myinfer_b200.engine import GenerationParams
    prompt = engine.encode_text("sampling")
    outs = set()
    for seed in (1, 1, 2):
        chunks = list(engine.generate(prompt, GenerationParams(max_tokens=6, temperature=1.0, top_p=0.9,
                                                               seed=seed, use_prefix_cache=False)))
        outs.add((seed, "".join(c.text for c in chunks)))
    assert len({t for s, t in outs if s == 1}) == 1          # seeded sampling is reproducible
    b = engine.benchmark(prompt_tokens=256, gen_tokens=16)
    assert b["prompt_tokens"] == 256 and b["completion_tokens"] == 16 and b["decode_tps"] > 0
    info = engine.info()
    assert info["totals"]["requests"] >= 1 and info["model"]["type"] == "qwen3"


def _oracle_greedy(model, prompt, n, prefill_step=64):
    """The oracle's greedy tokens and per-step logits for the engine's own
    (device-generated) weights, copied to the host."""
    import numpy as np
    from oracle import model as om
    host = {}
    for k, t in model.weights.items():
        c = t.cpu()
        host[k] = c.numpy().view(np.uint32) if c.dtype == torch.int32 else c.view(torch.int16).numpy().view(np.uint16)
    ora = om.Model(om.Config.from_dict(model.args.to_dict()), host)
    toks, _, logits = om.generate(ora, prompt, n, prefill_step=prefill_step, kv_bits=8, quantized_kv_start=0,
                                  return_logits=True)
    return toks, logits


def _agree_with_oracle(got, toks_o, logits_o):
    """Equal to the oracle's greedy tokens up to the first step where the
    oracle's own top-2 logits are within 0.02 (a numerical near-tie)."""
    for i, (a, b) in enumerate(zip(got, toks_o)):
        if a != b:
            top2 = logits_o[i].topk(2).values
            assert (top2[0] - top2[1]).item() < 0.02, (i, got, toks_o)
            return i
    assert len(got) == len(toks_o)
    return len(got)


def test_prefix_reuse_matches_oracle(engine):
    """A follow-up request that reuses a trimmed cached prefix (move-not-copy)
    generates the oracle's greedy tokens for the whole prompt, as does the
    same request with a fresh prefill."""
    engine.prefix.clear()
    base = engine.encode_text("Shared context for a two-turn conversation about caches. " * 2)
    follow = base + engine.encode_text(" Second turn: what is reused?")
    _run(engine, base, 8)
    _, m = _run(engine, follow, 10)
    assert m.cached_tokens == len(base)
    reused = list(engine.last_tokens)
    _, m_fresh = _run(engine, follow, 10, use_prefix_cache=False)
    assert m_fresh.cached_tokens == 0
    fresh = list(engine.last_tokens)
    toks_o, logits_o = _oracle_greedy(engine.model, follow, 10)
    _agree_with_oracle(reused, toks_o, logits_o)
    _agree_with_oracle(fresh, toks_o, logits_o)


def test_engine_loads_mlx_checkpoint_directory(tmp_path):
    """Engine.load on an MLX-style checkpoint directory (weights written by
    loader.save_mlx_checkpoint in two files with an index, no tokenizer files)
    generates the oracle's greedy tokens for those weights."""
    import numpy as np
    import warnings
    from myinfer_b200.engine import Engine, LoadOptions
    from myinfer_b200.loader import save_mlx_checkpoint
    from oracle import model as om
    cfg = dict(TINY, quantization={"group_size": 64, "bits": 4})
    host = om.generate_weights(om.Config.from_dict(cfg), seed=9)
    w = {k: torch.from_numpy(v.view(np.int32)) if v.dtype == np.uint32 else
         torch.from_numpy(v.view(np.int16)).view(torch.bfloat16) for k, v in host.items()}
    save_mlx_checkpoint(tmp_path, cfg, w, files=2)
    eng = Engine()
    with warnings.catch_warnings(record=True):
        eng.load(LoadOptions(model=str(tmp_path), kv_bits=8, quantized_kv_start=0, memory_budget_gb=4.0,
                             prefill_step=64, seed=5))
    try:
        prompt = list(np.random.default_rng(4).integers(3, 250, 40))
        _run(eng, prompt, 8, use_prefix_cache=False)
        toks_o, _, logits_o = om.generate(om.Model(om.Config.from_dict(cfg), host), prompt, 8, prefill_step=64,
                                          kv_bits=8, quantized_kv_start=0, return_logits=True)
        _agree_with_oracle(list(eng.last_tokens), toks_o, logits_o)
    finally:
        eng.unload()
