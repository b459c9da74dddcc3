"""Generate tests/golden/policy_fixtures.json from the reference's own host logic.

Runs m5engine/context.py and m5engine/prefix_cache.py of the reference
(tdcb/myinfer, mounted read-only) unchanged, with minimal stand-ins for the
`mlx` / `mlx_lm` modules they import at top level (they are not installable
here; the functions exercised never call into them except the cache trimming
helpers, which the stand-in implements as mlx-lm documents: a cache list is
trimmable when every entry is, and trimming moves each entry's offset back).

Usage (in the development container only; the fixture is committed):
    python tests/golden/make_policy_fixtures.py /path/to/reference
"""

from __future__ import annotations

import json
import sys
import types
from pathlib import Path


def install_stubs() -> None:
    def mod(name):
        m = types.ModuleType(name)
        sys.modules[name] = m
        return m

    mlx = mod("mlx")
    core = mod("mlx.core")
    mlx.core = core
    core.array = lambda *a, **k: None
    nn = mod("mlx.nn")
    mlx.nn = nn

    class Module:
        pass

    class RoPE(Module):
        pass

    nn.Module, nn.RoPE = Module, RoPE
    utils = mod("mlx.utils")
    mlx.utils = utils
    utils.tree_map = lambda f, x: x
    utils.tree_flatten = lambda x: []
    mod("mlx_lm")
    mod("mlx_lm.models")
    cache = mod("mlx_lm.models.cache")

    class KVCache:
        pass

    class QuantizedKVCache:
        pass

    class RotatingKVCache:
        pass

    cache.KVCache, cache.QuantizedKVCache, cache.RotatingKVCache = KVCache, QuantizedKVCache, RotatingKVCache
    cache.make_prompt_cache = lambda model: []
    cache.can_trim_prompt_cache = lambda c: all(x.is_trimmable() for x in c)

    def trim(c, n):
        return [x.trim(n) for x in c][0] if c else 0

    cache.trim_prompt_cache = trim
    rope = mod("mlx_lm.models.rope_utils")
    rope.initialize_rope = lambda *a, **k: None
    base = mod("mlx_lm.models.base")
    base.quantized_scaled_dot_product_attention = lambda *a, **k: None


class FakeCache:
    """One attention-cache layer: offset, nbytes and offset-moving trim."""

    def __init__(self, n, per_tok=100, trimmable=True):
        self.offset = n
        self.per_tok = per_tok
        self.trimmable = trimmable

    @property
    def nbytes(self):
        return self.offset * self.per_tok

    def is_trimmable(self):
        return self.trimmable

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n


def prefix_scenarios(PrefixCache, common_prefix_len):
    out = []
    # 1: reference unit test sequence (tests/test_core.py:79-88)
    pc = PrefixCache(max_entries=2)
    rec = {"common": common_prefix_len([1, 2, 3], [1, 2, 4])}
    pc.put("k", [1, 2, 3, 4, 5], [FakeCache(5)])
    c, hit = pc.take("k", [1, 2, 3, 9])
    rec["take1"] = [hit, c[0].offset, len(pc)]
    pc.put("k", [1, 2, 3, 4, 5], [FakeCache(5)])
    c, hit = pc.take("k", [1, 2, 3, 4, 5])
    rec["take2"] = [hit, c[0].offset]
    rec["other_none"] = pc.take("other", [1, 2, 3])[0] is None
    out.append(rec)
    # 2: LRU count and bytes (tests/test_core.py:91-97) plus offsets / bytes
    pc = PrefixCache(max_entries=2)
    for i in range(3):
        pc.put("k", [i, 1, 2], [FakeCache(3)])
    rec = {"len_after_3": len(pc), "nbytes": pc.nbytes}
    rec["freed"] = pc.evict_to(0)
    rec["len_after_evict"] = len(pc)
    out.append(rec)
    # 3: prefix replacement, disagreeing offsets, untrimmable entries, put truncation
    pc = PrefixCache(max_entries=4)
    pc.put("a", [1, 2, 3], [FakeCache(3)])
    pc.put("a", [1, 2, 3, 4, 5, 6], [FakeCache(6)])           # replaces [1,2,3]
    pc.put("a", [7, 8], [FakeCache(2), FakeCache(1)])         # layers disagree: refused
    pc.put("a", [9, 9, 9, 9], [FakeCache(2)])                 # tokens truncated to offset 2
    pc.put("b", [1, 2, 3, 4], [FakeCache(4, trimmable=False)])
    rec = {"len": len(pc), "nbytes": pc.nbytes}
    c, hit = pc.take("b", [1, 2, 3, 4, 5])                    # exact prefix of untrimmable entry: ok
    rec["take_b"] = [hit, None if c is None else c[0].offset]
    pc.put("b", [1, 2, 3, 4], [FakeCache(4, trimmable=False)])
    c, hit = pc.take("b", [1, 2, 9])                          # needs a trim: entry skipped
    rec["take_b_trim"] = [hit, c is None]
    c, hit = pc.take("a", [1, 2, 3, 4, 5, 6, 7])
    rec["take_a"] = [hit, None if c is None else c[0].offset]
    c, hit = pc.take("a", [9, 9, 5])
    rec["take_a2"] = [hit, None if c is None else c[0].offset]
    rec["stats"] = [pc.total_hit_tokens, pc.total_prompt_tokens, len(pc)]
    out.append(rec)
    return out


def main(ref: str) -> None:
    install_stubs()
    sys.path.insert(0, ref)
    from m5engine import context as C
    from m5engine.prefix_cache import PrefixCache, common_prefix_len

    GB = C.GB
    configs = [
        {"model_type": "qwen3", "max_position_embeddings": 40960},
        {"model_type": "qwen3_moe", "max_position_embeddings": 40960, "hidden_size": 2048},
        {"model_type": "qwen3", "max_position_embeddings": 131072,
         "rope_scaling": {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768}},
        {"model_type": "llama", "max_position_embeddings": 8192},
        {"model_type": "qwen2", "seq_length": 32768},
        {"model_type": "qwen3", "max_position_embeddings": 32768, "original_max_position_embeddings": 16384},
        {},
    ]
    fx = {"native_context": [[cfg, list(C.native_context(cfg))] for cfg in configs],
          "yarn_capable": [[cfg, C.yarn_capable(cfg)] for cfg in configs]}
    fx["yarn_factor_for"] = [[t, n, m, C.yarn_factor_for(t, n, m)]
                             for t in (1, 1000, 32768, 32769, 40000, 65536, 65537, 100000, 10 ** 6)
                             for n in (4096, 32768) for m in (1, 2, 4)]
    kvcfg = [{"num_hidden_layers": 28, "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128},
             {"num_hidden_layers": 64, "num_attention_heads": 64, "num_key_value_heads": 8, "hidden_size": 5120},
             {"text_config": {"num_hidden_layers": 48, "num_attention_heads": 32, "num_key_value_heads": 4,
                              "head_dim": 128}},
             {}]
    fx["kv_estimate_per_token"] = [[cfg, b, C.kv_estimate_per_token(cfg, b)] for cfg in kvcfg for b in (0, 4, 8)]
    fx["reserve_bytes"] = [[b, h, p, C.reserve_bytes(b, h, p)] for b in (8 * GB, 48 * GB, 180 * GB)
                           for h in (0, 2048, 5120) for p in (512, 2048)]
    plans = []
    for cfg in configs[:4]:
        for bpt in (52 * 1024, 139264, 0):
            for budget, resident in ((48 * GB, 17 * GB), (20 * GB, 17 * GB), (180 * GB, 18 * GB)):
                for rs in ("auto", "off", "4"):
                    for req in (None, 8192, 200000):
                        fp = C.KVFootprint(bytes_per_token=bpt, fixed_bytes=1 << 20, kv_bits=8)
                        p = C.plan_context(config=cfg, footprint=fp, budget_bytes=budget,
                                           resident_weight_bytes=resident, expert_cache_bytes=GB // 2,
                                           prefill_step=2048, rope_scaling=rs, requested_context=req)
                        plans.append([cfg, bpt, budget, resident, rs, req, p.to_dict()])
    fx["plan_context"] = plans
    fx["prefix_cache"] = prefix_scenarios(PrefixCache, common_prefix_len)
    out = Path(__file__).with_name("policy_fixtures.json")
    out.write_text(json.dumps(fx, sort_keys=True, separators=(",", ":")))
    print(f"wrote {out} ({out.stat().st_size} bytes, {len(plans)} plans)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
