"""Measure the bf16 noise floor of the logits parity bar on the Qwen3-0.6B config.

Every implementation of the path rounds activations to bf16 at the same points
but accumulates its fp32 dot products in its own order, so two correct
implementations drift apart by a few bf16 ulps per layer.  This script puts a
number on that drift: it runs the CPU oracle twice, once with fp32 matmuls
(the oracle as the tests use it) and once with fp64 accumulation rounded to
bf16 at the same points (order-independent, the closest thing to exact), and
the device token loop teacher-forced on the oracle's greedy tokens.  It prints
the per-step logits cosine and max-abs error of every pair.

    python tests/parity_floor.py [--steps 8] [--prompt 512] [--no-device]

Test infrastructure: imports the oracle; the device leg needs libm5cuda and a GPU.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle import model as om  # noqa: E402

QWEN3_06B = dict(model_type="qwen3", hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                 num_key_value_heads=8, head_dim=128, intermediate_size=3072, vocab_size=151936,
                 tie_word_embeddings=True, max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6)


class Fp64Model(om.Model):
    """The oracle with fp64 accumulation in every linear layer (same bf16 rounding points)."""

    def linear(self, x, name):
        return om.rb((x.double() @ self.deq(name).double().T).float())


def stats(a: torch.Tensor, b: torch.Tensor) -> dict:
    cos = torch.nn.functional.cosine_similarity(a.float(), b.float(), dim=-1)
    return {"cos_min": round(cos.min().item(), 6), "cos_median": round(cos.median().item(), 6),
            "max_abs": round((a.float() - b.float()).abs().max().item(), 5)}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-device", action="store_true")
    a = ap.parse_args()
    cfg = om.Config.from_dict(QWEN3_06B)
    t = time.time()
    host = om.generate_weights(cfg, a.seed)
    prompt = np.random.default_rng(a.seed).integers(0, cfg.vocab_size, a.prompt).tolist()
    kw = dict(prefill_step=2048, kv_bits=8, quantized_kv_start=0, return_logits=True)
    m32 = om.Model(cfg, host)
    tok32, _, l32 = om.generate(m32, prompt, a.steps, **kw)
    m64 = Fp64Model(cfg, host)
    m64._deq = m32._deq
    tok64, _, l64 = om.generate(m64, prompt, a.steps, **kw)
    out = {"config": "qwen3-0.6b", "prompt": a.prompt, "steps": a.steps, "seed": a.seed,
           "oracle32_vs_oracle64": stats(l32, l64), "tokens_equal_32_64": tok32 == tok64,
           "oracle_seconds": round(time.time() - t, 1)}
    if not a.no_device and torch.cuda.is_available():
        from myinfer_b200.cache import make_prompt_cache
        from myinfer_b200.generate import generate_step
        from myinfer_b200.model import Model, ModelArgs, upload_weights
        dev = Model(ModelArgs.from_dict(QWEN3_06B), upload_weights(host, "cuda"), "cuda", max_tokens=a.prompt)
        for name, toks, ref in (("oracle32", tok32, l32), ("oracle64", tok64, l64)):
            forced = list(generate_step(prompt, dev, a.steps, prompt_cache=make_prompt_cache(dev), feed=toks,
                                        prefill_step_size=2048, kv_bits=8, quantized_kv_start=0,
                                        return_logits=True))
            ld = torch.stack([l.float().cpu() for _, l in forced])
            out[f"device_vs_{name}"] = stats(ld, ref)
            out[f"device_tokens_equal_{name}"] = [t for t, _ in forced] == toks
    print(json.dumps(out))


if __name__ == "__main__":
    main()
