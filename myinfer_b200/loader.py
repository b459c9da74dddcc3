"""MLX checkpoint loader into HBM, shard-aware.

An mlx-community checkpoint directory holds ``config.json`` and one or more
``model*.safetensors`` files (with ``model.safetensors.index.json`` mapping
tensor names to files when there are several).  Quantized layers are stored as
MLX writes them: ``*.weight`` packed uint32 ``[..., rows, K/8]``, ``*.scales``
/ ``*.biases`` bf16 ``[..., rows, K/64]``; norms bf16.  The reference reads the
same files, tensor by tensor, from the safetensors headers
(m5engine/expert_stream.py:122-134, ``read_safetensors_index``) to stream
experts from SSD.

Here every tensor goes to the device once, and a rank of a tensor- or
expert-parallel group reads only its own part from the file (through the
safetensors slice API, which maps the file and copies just the requested
rows): q/k/v and gate/up rows, o_proj/down columns in whole scale groups,
lm_head rows (tensor parallel; k/v rows of the rank's kv head when kv heads
are replicated over the ranks); its experts of every ``switch_mlp`` stack
(expert parallel; both at once for head-sharded MoE attention).  The result equals ``distributed.shard_weights`` applied
to the whole checkpoint, without the whole checkpoint ever being in host or
device memory.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import torch

TP_ROWS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "mlp.gate_proj", "mlp.up_proj")
TP_COLS = ("self_attn.o_proj", "mlp.down_proj")


def checkpoint_files(path: Path) -> Dict[str, Path]:
    """Tensor name -> file, from the index when present, else from the headers
    of every ``model*.safetensors`` (as the reference's reader does)."""
    path = Path(path)
    idx = path / "model.safetensors.index.json"
    if idx.exists():
        wm = json.loads(idx.read_text())["weight_map"]
        return {k: path / v for k, v in wm.items()}
    from safetensors import safe_open
    out: Dict[str, Path] = {}
    files = sorted(path.glob("model*.safetensors")) or sorted(path.glob("*.safetensors"))
    for f in files:
        with safe_open(str(f), framework="pt") as h:
            for k in h.keys():
                out[k] = f
    if not out:
        raise FileNotFoundError(f"no safetensors files in {path}")
    return out


def _part(name: str, shape: List[int], tp_size: int, tp_rank: int, ep_size: int,
          ep_rank: int, n_kv_heads: int = 0) -> Tuple[Optional[Tuple[int, int]], Optional[Tuple[int, int]]]:
    """(row range on the leading axis, column range on the last axis) of this
    rank's part of tensor `name` (None = whole axis).  `n_kv_heads` (the
    model's) decides the k/v rows under tensor parallelism."""
    from .distributed import kv_head_first, kv_heads_local
    base, suffix = name.rsplit(".", 1)
    if ep_size > 1 and ".switch_mlp." in name:
        E = shape[0]
        if E % ep_size:
            raise ValueError(f"{name}: {E} experts do not split over {ep_size} ranks")
        k = E // ep_size
        return (ep_rank * k, (ep_rank + 1) * k), None
    if tp_size > 1 and n_kv_heads and base.endswith(("self_attn.k_proj", "self_attn.v_proj")) \
            and suffix in ("weight", "scales", "biases"):
        D = shape[0] // n_kv_heads
        r0 = kv_head_first(n_kv_heads, tp_size, tp_rank) * D
        return (r0, r0 + kv_heads_local(n_kv_heads, tp_size) * D), None
    if tp_size > 1 and suffix in ("weight", "scales", "biases"):
        if base.endswith(TP_ROWS) or base == "lm_head":
            R = shape[0]
            if R % tp_size:
                raise ValueError(f"cannot split {R} rows of {name} over {tp_size} ranks")
            k = R // tp_size
            return (tp_rank * k, (tp_rank + 1) * k), None
        if base.endswith(TP_COLS):
            C = shape[-1]
            per_group = 8 if suffix == "weight" else 1  # packed words of a 64-column 4-bit group
            if C % (tp_size * per_group):
                raise ValueError(f"{name}: {C} columns do not split over {tp_size} ranks in whole groups")
            k = C // tp_size
            return None, (tp_rank * k, (tp_rank + 1) * k)
    return None, None


def load_mlx_checkpoint(path, device, tp_size: int = 1, tp_rank: int = 0, ep_size: int = 1, ep_rank: int = 0,
                        tie_word_embeddings: Optional[bool] = None) -> Dict[str, torch.Tensor]:
    """This rank's weights of the checkpoint at `path`, on `device`.

    Packed uint32 tensors come back as int32 tensors holding the same bits (the
    layout libm5cuda binds).  Under tensor parallelism a model with tied
    embeddings also gets ``lm_head.*``: its vocabulary rows of the embedding."""
    from safetensors import safe_open
    if tp_size > 1 and ep_size > 1 and (tp_size != ep_size or tp_rank != ep_rank):
        raise ValueError("head-sharded attention with expert parallelism uses the same ranks for both")
    path = Path(path)
    cfg_path = path / "config.json"
    cfg = json.loads(cfg_path.read_text()) if cfg_path.exists() else {}
    if tie_word_embeddings is None:
        tie_word_embeddings = bool(cfg.get("tie_word_embeddings", False))
    n_kv_heads = int(cfg.get("num_key_value_heads", 0))
    by_file: Dict[Path, List[str]] = {}
    for name, f in checkpoint_files(path).items():
        by_file.setdefault(f, []).append(name)
    out: Dict[str, torch.Tensor] = {}
    dev = torch.device(device)
    for f, names in sorted(by_file.items()):
        with safe_open(str(f), framework="pt") as h:
            for name in sorted(names):
                sl = h.get_slice(name)
                shape = list(sl.get_shape())
                rows, cols = _part(name, shape, tp_size, tp_rank, ep_size, ep_rank, n_kv_heads)
                if rows is not None:
                    t = sl[rows[0]:rows[1]]
                elif cols is not None:
                    t = sl[:, cols[0]:cols[1]]
                else:
                    t = sl[:]
                if t.dtype == torch.uint32:
                    t = t.view(torch.int32)
                out[name] = t.contiguous().to(dev)
                if tp_size > 1 and tie_word_embeddings and name.startswith("model.embed_tokens."):
                    V = shape[0]
                    k = V // tp_size
                    lt = sl[tp_rank * k:(tp_rank + 1) * k]
                    if lt.dtype == torch.uint32:
                        lt = lt.view(torch.int32)
                    out["lm_head." + name.rsplit(".", 1)[1]] = lt.contiguous().to(dev)
    return out


def save_mlx_checkpoint(path, config: dict, weights: Dict[str, torch.Tensor], files: int = 1) -> None:
    """Write `weights` (int32 packed words are stored as uint32, as MLX does)
    as an MLX-style checkpoint: config.json, `files` safetensors shards and,
    with more than one, model.safetensors.index.json."""
    from safetensors.torch import save_file
    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    (path / "config.json").write_text(json.dumps(config))
    names = sorted(weights)
    parts = [names[i::files] for i in range(files)]
    wm = {}
    for i, part in enumerate(parts):
        fname = "model.safetensors" if files == 1 else f"model-{i + 1:05d}-of-{files:05d}.safetensors"
        tensors = {}
        for n in part:
            t = weights[n].detach().cpu().contiguous()
            tensors[n] = t.view(torch.uint32) if t.dtype == torch.int32 else t
            wm[n] = fname
        save_file(tensors, str(path / fname), metadata={"format": "mlx"})
    if files > 1:
        (path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
