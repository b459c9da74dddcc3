"""Host policy (KV planner, YaRN choice, prefix cache) vs the reference.

tests/golden/policy_fixtures.json was produced by running the reference's own
m5engine/context.py and m5engine/prefix_cache.py (make_policy_fixtures.py);
the known answers of tests/test_core.py:43-97 are asserted directly too."""

import json
from pathlib import Path

import pytest

from myinfer_b200 import context as C
from myinfer_b200.prefix_cache import PrefixCache, common_prefix_len

FX = json.loads((Path(__file__).parent / "golden" / "policy_fixtures.json").read_text())
GB = C.GB


def test_reference_known_answers():
    # tests/test_core.py:43-54
    assert C.native_context({"model_type": "qwen3", "max_position_embeddings": 40960}) == (32768, 40960)
    cfg = {"max_position_embeddings": 131072,
           "rope_scaling": {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 32768}}
    assert C.native_context(cfg) == (32768, 131072)
    assert C.yarn_factor_for(1000, 32768, 4) == 1
    assert C.yarn_factor_for(40000, 32768, 4) == 2
    assert C.yarn_factor_for(100000, 32768, 4) == 4
    assert C.yarn_factor_for(10 ** 6, 32768, 4) == 4
    # tests/test_core.py:57-70
    cfg = {"model_type": "qwen3_moe", "max_position_embeddings": 40960, "hidden_size": 2048}
    fp = C.KVFootprint(bytes_per_token=52 * 1024, fixed_bytes=0, kv_bits=8)
    plan = C.plan_context(config=cfg, footprint=fp, budget_bytes=48 * GB, resident_weight_bytes=17 * GB)
    assert plan.yarn_factor == 4 and plan.max_context == 131072 and plan.limited_by == "model"
    tight = C.plan_context(config=cfg, footprint=fp, budget_bytes=20 * GB, resident_weight_bytes=17 * GB)
    assert tight.limited_by == "memory" and tight.max_context == tight.memory_context_limit
    assert tight.max_context % 256 == 0 and tight.max_context < 40960
    off = C.plan_context(config=cfg, footprint=fp, budget_bytes=48 * GB, resident_weight_bytes=17 * GB,
                         rope_scaling="off")
    assert off.max_context == 40960 and off.yarn_factor == 1
    capped = C.plan_context(config=cfg, footprint=fp, budget_bytes=48 * GB, resident_weight_bytes=17 * GB,
                            requested_context=8192)
    assert capped.max_context == 8192 and capped.limited_by == "setting"


def test_native_context_and_yarn_capable():
    for cfg, want in FX["native_context"]:
        assert list(C.native_context(cfg)) == want, cfg
    for cfg, want in FX["yarn_capable"]:
        assert C.yarn_capable(cfg) == want, cfg


def test_yarn_factor_for():
    for t, n, m, want in FX["yarn_factor_for"]:
        assert C.yarn_factor_for(t, n, m) == want, (t, n, m)


def test_kv_estimate_and_reserve():
    for cfg, b, want in FX["kv_estimate_per_token"]:
        assert C.kv_estimate_per_token(cfg, b) == want, (cfg, b)
    for b, h, p, want in FX["reserve_bytes"]:
        assert C.reserve_bytes(b, h, p) == want


def test_plan_context_grid():
    for cfg, bpt, budget, resident, rs, req, want in FX["plan_context"]:
        fp = C.KVFootprint(bytes_per_token=bpt, fixed_bytes=1 << 20, kv_bits=8)
        got = C.plan_context(config=cfg, footprint=fp, budget_bytes=budget, resident_weight_bytes=resident,
                             expert_cache_bytes=GB // 2, prefill_step=2048, rope_scaling=rs,
                             requested_context=req).to_dict()
        assert got == want, (cfg, bpt, budget, resident, rs, req)


class FakeCache:
    def __init__(self, n, per_tok=100, trimmable=True):
        self.offset, self.per_tok, self.trimmable = n, per_tok, trimmable

    @property
    def nbytes(self):
        return self.offset * self.per_tok

    def is_trimmable(self):
        return self.trimmable

    def trim(self, n):
        n = min(self.offset, n)
        self.offset -= n
        return n


def test_prefix_cache_scenarios():
    want = FX["prefix_cache"]
    pc = PrefixCache(max_entries=2)
    rec = {"common": common_prefix_len([1, 2, 3], [1, 2, 4])}
    pc.put("k", [1, 2, 3, 4, 5], [FakeCache(5)])
    c, hit = pc.take("k", [1, 2, 3, 9])
    rec["take1"] = [hit, c[0].offset, len(pc)]
    pc.put("k", [1, 2, 3, 4, 5], [FakeCache(5)])
    c, hit = pc.take("k", [1, 2, 3, 4, 5])
    rec["take2"] = [hit, c[0].offset]
    rec["other_none"] = pc.take("other", [1, 2, 3])[0] is None
    assert rec == want[0]

    pc = PrefixCache(max_entries=2)
    for i in range(3):
        pc.put("k", [i, 1, 2], [FakeCache(3)])
    rec = {"len_after_3": len(pc), "nbytes": pc.nbytes}
    rec["freed"] = pc.evict_to(0)
    rec["len_after_evict"] = len(pc)
    assert rec == want[1]

    pc = PrefixCache(max_entries=4)
    pc.put("a", [1, 2, 3], [FakeCache(3)])
    pc.put("a", [1, 2, 3, 4, 5, 6], [FakeCache(6)])
    pc.put("a", [7, 8], [FakeCache(2), FakeCache(1)])
    pc.put("a", [9, 9, 9, 9], [FakeCache(2)])
    pc.put("b", [1, 2, 3, 4], [FakeCache(4, trimmable=False)])
    rec = {"len": len(pc), "nbytes": pc.nbytes}
    c, hit = pc.take("b", [1, 2, 3, 4, 5])
    rec["take_b"] = [hit, None if c is None else c[0].offset]
    pc.put("b", [1, 2, 3, 4], [FakeCache(4, trimmable=False)])
    c, hit = pc.take("b", [1, 2, 9])
    rec["take_b_trim"] = [hit, c is None]
    c, hit = pc.take("a", [1, 2, 3, 4, 5, 6, 7])
    rec["take_a"] = [hit, None if c is None else c[0].offset]
    c, hit = pc.take("a", [9, 9, 5])
    rec["take_a2"] = [hit, None if c is None else c[0].offset]
    rec["stats"] = [pc.total_hit_tokens, pc.total_prompt_tokens, len(pc)]
    assert rec == want[2]


def test_device_cache_trim_contract():
    """The device caches keep the mlx-lm contract the prefix cache relies on
    (offset, nbytes, trimmable, sequence axis -2) without touching a GPU."""
    from myinfer_b200.cache import KVCache, QuantizedKVCache, can_trim_prompt_cache, trim_prompt_cache
    k = KVCache(2, 128, "cpu", capacity=300)
    k.offset = 40
    q = QuantizedKVCache(2, 128, "cpu", bits=8, capacity=300)
    q.offset = 40
    assert k.capacity == 512 and q.capacity == 512           # steps of 256 like mlx-lm
    assert k.keys.shape[-2] == 512 and q.keys[0].shape[-2] == 512
    assert k.nbytes == 2 * 2 * 512 * 128 * 2
    assert q.nbytes == 2 * (2 * 512 * 32 * 4 + 2 * 2 * 512 * 2 * 2)  # 1.0625 bytes per element
    cache = [k, q]
    assert can_trim_prompt_cache(cache)
    assert trim_prompt_cache(cache, 15) == 15 and k.offset == 25 and q.offset == 25
    assert trim_prompt_cache(cache, 100) == 25 and k.offset == 0
