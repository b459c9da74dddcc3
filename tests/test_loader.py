"""MLX checkpoint loader (myinfer_b200/loader.py) on the CPU: a seeded tiny
model written as an MLX-style checkpoint (uint32 packed words, bf16 scales,
biases and norms; one file, or several with model.safetensors.index.json)
loads back bit for bit, and a tensor- or expert-parallel rank reads exactly
the shard distributed.shard_weights would cut from the whole model."""

import numpy as np
import pytest
import torch

from myinfer_b200.distributed import shard_weights
from myinfer_b200.loader import checkpoint_files, load_mlx_checkpoint, save_mlx_checkpoint
from myinfer_b200.model import ModelArgs
from oracle import model as om

DENSE = dict(model_type="qwen3", hidden_size=512, num_hidden_layers=2, num_attention_heads=8, num_key_value_heads=2,
             head_dim=128, intermediate_size=1024, vocab_size=4096, tie_word_embeddings=True,
             max_position_embeddings=40960, rms_norm_eps=1e-6, rope_theta=1e6,
             quantization={"group_size": 64, "bits": 4})
MOE = dict(DENSE, model_type="qwen3_moe", num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256,
           norm_topk_prob=True, intermediate_size=0, tie_word_embeddings=False)


def _weights(cfg):
    host = om.generate_weights(om.Config.from_dict(cfg), seed=3)
    return {k: torch.from_numpy(v.view(np.int32) if v.dtype == np.uint32 else v.view(np.int16)).view(
        torch.int32 if v.dtype == np.uint32 else torch.bfloat16) for k, v in host.items()}


def _same(a, b):
    assert sorted(a) == sorted(b)
    for k in a:
        assert a[k].dtype == b[k].dtype and a[k].shape == b[k].shape, k
        assert torch.equal(a[k].view(torch.int16) if a[k].dtype == torch.bfloat16 else a[k],
                           b[k].view(torch.int16) if b[k].dtype == torch.bfloat16 else b[k]), k


@pytest.mark.parametrize("files", [1, 3])
def test_roundtrip(tmp_path, files):
    w = _weights(DENSE)
    save_mlx_checkpoint(tmp_path, DENSE, w, files=files)
    assert (tmp_path / "model.safetensors.index.json").exists() == (files > 1)
    assert set(checkpoint_files(tmp_path)) == set(w)
    _same(load_mlx_checkpoint(tmp_path, "cpu"), w)


@pytest.mark.parametrize("tp", [2, 4])
def test_tensor_parallel_rank_reads_its_shard(tmp_path, tp):
    w = _weights(DENSE)
    save_mlx_checkpoint(tmp_path, DENSE, w, files=2)
    args = ModelArgs.from_dict(DENSE)
    for r in range(tp):
        _same(load_mlx_checkpoint(tmp_path, "cpu", tp_size=tp, tp_rank=r),
              shard_weights(w, args, tp_size=tp, tp_rank=r))


@pytest.mark.parametrize("ep", [2, 4])
def test_expert_parallel_rank_reads_its_experts(tmp_path, ep):
    w = _weights(MOE)
    save_mlx_checkpoint(tmp_path, MOE, w, files=2)
    args = ModelArgs.from_dict(MOE)
    for r in range(ep):
        _same(load_mlx_checkpoint(tmp_path, "cpu", ep_size=ep, ep_rank=r),
              shard_weights(w, args, ep_size=ep, ep_rank=r))


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_moe_rank_reads_its_shard(tmp_path, world):
    """Attention heads and experts over the same ranks (kv heads replicated at
    4 ranks: 2 kv heads)."""
    w = _weights(MOE)
    save_mlx_checkpoint(tmp_path, MOE, w, files=3)
    args = ModelArgs.from_dict(MOE)
    for r in range(world):
        _same(load_mlx_checkpoint(tmp_path, "cpu", tp_size=world, tp_rank=r, ep_size=world, ep_rank=r),
              shard_weights(w, args, tp_size=world, tp_rank=r, ep_size=world, ep_rank=r))


def test_uneven_split_is_rejected(tmp_path):
    w = _weights(MOE)
    save_mlx_checkpoint(tmp_path, MOE, w)
    with pytest.raises(ValueError):
        load_mlx_checkpoint(tmp_path, "cpu", ep_size=3, ep_rank=0)
