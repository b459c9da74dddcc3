"""QK-norm + RoPE + KV append fused into the q|k|v GEMV's epilogue against the
separate rope_append kernel: the same model, tokens and caches, byte for byte.

Decode-sized calls (up to 8 tokens) run the fused epilogue by default;
M5_FUSE_ROPE=0 keeps the separate kernel.  The switch is read once per
process, so each setting runs in a child process that writes the layers'
bf16 K/V, the 8-bit and 4-bit caches' codes / scales / biases, and every
step's logits.  Hidden size 1024 gives the GEMVs whole 16-row tiles (fixed
reduction order), so any difference is the epilogue's."""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(model_type="qwen3", hidden_size=1024, num_hidden_layers=2, num_attention_heads=16, num_key_value_heads=8,
           head_dim=128, intermediate_size=1024, vocab_size=2048, tie_word_embeddings=False,
           max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6)
PREFILL, DECODE = 12, 6


def _dump(out: str) -> None:
    import torch
    from myinfer_b200.cache import PromptCache, QuantizedKVCache, make_prompt_cache
    from myinfer_b200.model import Model, ModelArgs, random_weights
    a = ModelArgs.from_dict(CFG)
    m = Model(a, random_weights(a, 5, "cuda"), "cuda", max_tokens=64)
    ids = torch.from_numpy(np.random.default_rng(5).integers(0, CFG["vocab_size"], PREFILL + DECODE + 8)
                           .astype(np.int32)).cuda()
    n = PREFILL + DECODE + 8
    res = {}
    caches = {"bf16": make_prompt_cache(m, n)}
    for bits in (8, 4):
        caches[f"q{bits}"] = PromptCache([QuantizedKVCache(m.n_kv_heads_local, a.head_dim, "cuda", 64, bits,
                                                           capacity=n) for _ in range(a.num_hidden_layers)], "cuda")
    from myinfer_b200 import _lib

    def step(cache, toks):
        out = torch.empty(int(toks.numel()), CFG["vocab_size"], dtype=torch.bfloat16, device="cuda")
        m.forward(toks, cache, _lib.M5_LOGITS_ALL, out)
        return out.float().cpu()

    for name, cache in caches.items():
        logits = [step(cache, ids[:PREFILL])]
        for i in range(PREFILL, PREFILL + DECODE):
            logits.append(step(cache, ids[i:i + 1]))
        # an 8-token call: the fused epilogue at MT = 8
        logits.append(step(cache, ids[PREFILL + DECODE:n]))
        torch.cuda.synchronize()
        res[f"{name}_logits"] = torch.cat(logits).numpy()
        for li, c in enumerate(cache):
            for kind, t in (("k", c.keys), ("v", c.values)):
                parts = t if isinstance(t, (tuple, list)) else (t,)
                for j, p in enumerate(parts):
                    x = p[..., :n, :].contiguous().cpu()
                    res[f"{name}_{li}_{kind}{j}"] = x.view(torch.int16).numpy() if x.dtype == torch.bfloat16 \
                        else x.numpy()
    np.savez(out, **res)


def _child(tmp: Path, fuse: str) -> dict:
    out = tmp / f"fuse{fuse}.npz"
    env = dict(os.environ, M5_FUSE_ROPE=fuse)
    r = subprocess.run([sys.executable, __file__, str(out)], env=env, capture_output=True, text=True, timeout=600,
                       cwd=str(Path(__file__).resolve().parents[1]))
    assert r.returncode == 0, r.stderr[-3000:]
    return dict(np.load(out))


def test_fused_rope_matches_separate_kernel(tmp_path):
    fused = _child(tmp_path, "1")
    plain = _child(tmp_path, "0")
    assert fused.keys() == plain.keys()
    for k in sorted(fused):
        a, b = fused[k], plain[k]
        assert a.shape == b.shape, k
        bad = np.argwhere(a != b)
        assert bad.size == 0, f"{k}: {len(bad)} differences, first at {bad[0].tolist()}"


if __name__ == "__main__":
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    _dump(sys.argv[1])
