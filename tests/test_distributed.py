"""Multi-GPU host logic on CPU: weight shards (tensor / expert parallel) and the
communicator id exchange over a world-size-2 gloo group."""

import os

import numpy as np
import pytest
import torch

from myinfer_b200.distributed import Communicator, shard_weights
from myinfer_b200.model import ModelArgs
from oracle import model as om
from oracle.quant import affine_dequantize

TINY = dict(model_type="qwen3", hidden_size=512, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
            head_dim=128, intermediate_size=1024, vocab_size=4096, tie_word_embeddings=True,
            max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6)
TINY_MOE = dict(TINY, model_type="qwen3_moe", num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256,
                norm_topk_prob=True, intermediate_size=0, tie_word_embeddings=False)


def _host(cfg):
    w = om.generate_weights(om.Config.from_dict(cfg), seed=1)
    out = {}
    for k, v in w.items():
        out[k] = torch.from_numpy(v.view(np.int32) if v.dtype == np.uint32 else v.view(np.int16))
    return out


def _deq(w, name):
    return affine_dequantize(w[name + ".weight"].numpy().view(np.uint32), w[name + ".scales"].numpy().view(np.uint16),
                             w[name + ".biases"].numpy().view(np.uint16), 64, 4).astype(np.float64)


@pytest.mark.parametrize("tp", [2, 4])
def test_tensor_parallel_shards_recompose(tp):
    args = ModelArgs.from_dict(TINY)
    full = _host(TINY)
    shards = [shard_weights(full, args, tp_size=tp, tp_rank=r) for r in range(tp)]
    p = "model.layers.1."
    for name in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.gate_proj", "mlp.up_proj"):
        kv = name in ("self_attn.k_proj", "self_attn.v_proj")
        for suf in (".weight", ".scales", ".biases"):
            if kv and args.num_key_value_heads < tp:  # each kv head replicated on tp / Hkv ranks
                per = tp // args.num_key_value_heads
                for r, s in enumerate(shards):
                    h = r // per
                    assert torch.equal(s[p + name + suf], full[p + name + suf][h * 128:(h + 1) * 128]), name
                continue
            cat = torch.cat([s[p + name + suf] for s in shards], dim=0)
            assert torch.equal(cat, full[p + name + suf]), name
    for name in ("self_attn.o_proj", "mlp.down_proj"):
        for suf in (".weight", ".scales", ".biases"):
            cat = torch.cat([s[p + name + suf] for s in shards], dim=-1)
            assert torch.equal(cat, full[p + name + suf]), name
    # tied embeddings: every rank binds its vocabulary rows of the embedding as lm_head
    head = torch.cat([s["lm_head.weight"] for s in shards], dim=0)
    assert torch.equal(head, full["model.embed_tokens.weight"])
    assert all(torch.equal(s["model.embed_tokens.weight"], full["model.embed_tokens.weight"]) for s in shards)
    assert all(torch.equal(s[p + "self_attn.q_norm.weight"], full[p + "self_attn.q_norm.weight"]) for s in shards)


def test_column_shards_sum_to_the_full_product():
    """o_proj / down split along K: the per-rank partial products add up to x @ W^T."""
    args = ModelArgs.from_dict(TINY)
    full = _host(TINY)
    tp = 2
    name = "model.layers.0.mlp.down_proj"
    rng = np.random.default_rng(0)
    x = rng.standard_normal((3, args.intermediate_size))
    ref = x @ _deq(full, name).T
    parts = 0
    k = args.intermediate_size // tp
    for r in range(tp):
        s = shard_weights(full, args, tp_size=tp, tp_rank=r)
        parts = parts + x[:, r * k:(r + 1) * k] @ _deq(s, name).T
    np.testing.assert_allclose(parts, ref, rtol=1e-12, atol=1e-12)


def test_expert_parallel_shards():
    args = ModelArgs.from_dict(TINY_MOE)
    full = _host(TINY_MOE)
    ep = 4
    shards = [shard_weights(full, args, ep_size=ep, ep_rank=r) for r in range(ep)]
    p = "model.layers.0.mlp."
    for name in ("switch_mlp.gate_proj", "switch_mlp.up_proj", "switch_mlp.down_proj"):
        cat = torch.cat([s[p + name + ".weight"] for s in shards], dim=0)
        assert torch.equal(cat, full[p + name + ".weight"])
        assert shards[1][p + name + ".scales"].shape[0] == args.num_experts // ep
    # router and attention replicated
    for s in shards:
        assert torch.equal(s[p + "gate.weight"], full[p + "gate.weight"])
        assert torch.equal(s["model.layers.0.self_attn.q_proj.weight"], full["model.layers.0.self_attn.q_proj.weight"])


def test_shard_errors():
    args = ModelArgs.from_dict(TINY)
    full = _host(TINY)
    with pytest.raises(ValueError):
        shard_weights(full, args, tp_size=3, tp_rank=0)  # 8 heads over 3 ranks
    with pytest.raises(ValueError):
        shard_weights(full, args, ep_size=2, ep_rank=0)  # dense model
    moe = ModelArgs.from_dict(TINY_MOE)
    with pytest.raises(ValueError):
        shard_weights(_host(TINY_MOE), moe, tp_size=2, tp_rank=0)  # heads without the experts
    with pytest.raises(ValueError):
        shard_weights(_host(TINY_MOE), moe, tp_size=2, tp_rank=0, ep_size=2, ep_rank=1)  # different ranks
    with pytest.raises(ValueError):
        shard_weights(_host(TINY_MOE), moe, tp_size=2, tp_rank=0, ep_size=4, ep_rank=0)  # different groups
    with pytest.raises(ValueError):  # 3 kv heads neither split over nor replicate onto 2 ranks
        shard_weights(full, ModelArgs.from_dict(dict(TINY, num_attention_heads=12, num_key_value_heads=3)),
                      tp_size=2, tp_rank=0)


def _exchange_worker(rank, world, port, q):
    import torch.distributed as dist

    from myinfer_b200 import _lib
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    seen = {}

    def fake_call(name, *a):
        if name == "m5_comm_unique_id":
            a[0].raw = bytes(range(128))
        elif name == "m5_comm_init":
            seen["id"] = bytes(a[0].raw[:128])
            seen["world"], seen["rank"] = a[2], a[3]
            a[4]._obj.value = 1234 + rank
        return 0

    _lib.call = fake_call
    c = Communicator(world, rank)
    q.put((rank, seen["id"] == bytes(range(128)), seen["world"], seen["rank"], c.handle.value))
    c.handle = None
    dist.destroy_process_group()


def test_communicator_id_exchange_gloo():
    """Rank 0's id reaches every rank through torch.distributed (gloo, 2 ranks)."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == [(0, True, 2, 0, 1234), (1, True, 2, 1, 1235)]


def test_device_check_maps_error_word(monkeypatch):
    """_lib.device_check raises M5_ERR_TIMEOUT when the device error word is
    set (faked status call; no GPU involved) and passes when it is clear."""
    from myinfer_b200 import _lib

    class FakeLib:
        def __init__(self, word):
            self.word = word

        def m5_device_status(self, code_ptr, reset):
            code_ptr._obj.value = self.word
            return _lib.M5_OK

        def m5_last_error(self, buf, n):
            return 0

    monkeypatch.setattr(_lib, "lib", lambda: FakeLib(0))
    _lib.device_check()
    monkeypatch.setattr(_lib, "lib", lambda: FakeLib(1))
    with pytest.raises(_lib.M5CudaError) as e:
        _lib.device_check()
    assert e.value.code == _lib.M5_ERR_TIMEOUT


def test_kv_head_placement():
    from myinfer_b200.distributed import kv_head_first, kv_heads_local
    assert [kv_heads_local(8, t) for t in (1, 2, 4, 8)] == [8, 4, 2, 1]
    assert [kv_heads_local(4, t) for t in (2, 4, 8)] == [2, 1, 1]  # 8 ranks: each kv head on 2 ranks
    assert [kv_head_first(4, 8, r) for r in range(8)] == [0, 0, 1, 1, 2, 2, 3, 3]
    assert [kv_head_first(8, 4, r) for r in range(4)] == [0, 2, 4, 6]
    with pytest.raises(ValueError):
        kv_heads_local(4, 3)
    with pytest.raises(ValueError):
        kv_heads_local(3, 2)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_moe_head_sharded_with_experts(world):
    """MoE with attention heads sharded over the expert-parallel ranks: q rows
    and o_proj columns split by heads, k/v rows of the rank's kv head (each of
    the 4 kv heads replicated on world / 4 ranks at 8), lm_head rows split,
    experts split, router replicated; every rank's q heads belong to the kv
    head it holds (GQA group = heads // kv_heads)."""
    cfg = dict(TINY_MOE, num_attention_heads=16, num_key_value_heads=4, num_experts=16)
    args = ModelArgs.from_dict(cfg)
    full = _host(cfg)
    D, Hq, Hkv = 128, 16, 4
    shards = [shard_weights(full, args, tp_size=world, tp_rank=r, ep_size=world, ep_rank=r) for r in range(world)]
    p = "model.layers.1."
    for suf in (".weight", ".scales", ".biases"):
        assert torch.equal(torch.cat([s[p + "self_attn.q_proj" + suf] for s in shards]), full[p + "self_attn.q_proj" + suf])
        assert torch.equal(torch.cat([s[p + "self_attn.o_proj" + suf] for s in shards], dim=-1),
                           full[p + "self_attn.o_proj" + suf])
        assert torch.equal(torch.cat([s["lm_head" + suf] for s in shards]), full["lm_head" + suf])
        ex = p + "mlp.switch_mlp.up_proj" + suf
        assert torch.equal(torch.cat([s[ex] for s in shards]), full[ex])
    for r, s in enumerate(shards):
        hq0 = r * Hq // world                       # first q head of the rank
        kv = hq0 // (Hq // Hkv)                      # its group's kv head
        n_kv = max(1, Hkv // world)
        assert (hq0 + Hq // world - 1) // (Hq // Hkv) < kv + n_kv  # all the rank's q heads map into its kv heads
        for name in ("self_attn.k_proj", "self_attn.v_proj"):
            assert torch.equal(s[p + name + ".weight"], full[p + name + ".weight"][kv * D:(kv + n_kv) * D])
        assert torch.equal(s[p + "mlp.gate.weight"], full[p + "mlp.gate.weight"])
    # experts generated per rank are taken as they are
    local = {k: (v[:16 // world] if ".switch_mlp." in k else v) for k, v in full.items()}
    s0 = shard_weights(local, args, tp_size=world, tp_rank=0, ep_size=world, ep_rank=0, experts_local=True)
    assert torch.equal(s0[p + "mlp.switch_mlp.down_proj.weight"], shards[0][p + "mlp.switch_mlp.down_proj.weight"])
