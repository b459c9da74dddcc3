"""Multi-GPU plumbing: weight shards and the libm5cuda communicator.

One process per GPU.  Dense Qwen3 runs tensor parallel over ``tp`` ranks
(q/k/v heads, gate/up rows, o_proj/down columns and lm_head rows split; the
C++ forward all-reduces the o_proj and down partial sums and all-gathers the
vocabulary shards).  Qwen3-MoE runs expert parallel over ``ep`` ranks (the
stacked ``switch_mlp`` experts split, the router replicated; the MoE partial
sums are all-reduced), with attention either replicated (``tp_size`` 1) or
head-sharded over the same ranks (``tp_size == ep_size``: q/k/v heads,
o_proj columns and lm_head rows split as for a dense model, one more
all-reduce per layer).  Where a model has fewer kv heads than ranks
(Qwen3-235B-A22B: 4 kv heads, 8 ranks) each kv head is replicated on
``tp / Hkv`` consecutive ranks, which hold the q heads of its group.  The
reference (m5engine) is single-device; this is the B200 build's own
partitioning.

``shard_weights`` works on any tensors (CPU or device) in the MLX layout:
packed ``*.weight`` [rows, K/8] int32, ``*.scales`` / ``*.biases`` [rows, K/64].
"""

from __future__ import annotations

import ctypes
from typing import Dict, Optional

import torch

from . import _lib


def _row_slice(t: torch.Tensor, n: int, r: int, axis: int = 0) -> torch.Tensor:
    size = t.shape[axis]
    if size % n:
        raise ValueError(f"cannot split {size} rows over {n} ranks")
    k = size // n
    return t.narrow(axis, r * k, k).contiguous()


def _col_slice(w: Dict[str, torch.Tensor], name: str, n: int, r: int, out: Dict[str, torch.Tensor]) -> None:
    """Split a quantized linear along K (its input columns) in whole scale groups."""
    wq, s, b = w[name + ".weight"], w[name + ".scales"], w[name + ".biases"]
    groups = s.shape[-1]
    if groups % n:
        raise ValueError(f"{name}: {groups} scale groups do not split over {n} ranks")
    g = groups // n
    words = wq.shape[-1] // groups  # packed words per group (8 for 4-bit g64)
    out[name + ".weight"] = wq.narrow(-1, r * g * words, g * words).contiguous()
    out[name + ".scales"] = s.narrow(-1, r * g, g).contiguous()
    out[name + ".biases"] = b.narrow(-1, r * g, g).contiguous()


def _rows(w: Dict[str, torch.Tensor], name: str, n: int, r: int, out: Dict[str, torch.Tensor],
          axis: int = 0, src: Optional[str] = None) -> None:
    src = src or name
    for suf in (".weight", ".scales", ".biases"):
        out[name + suf] = _row_slice(w[src + suf], n, r, axis)


def kv_heads_local(n_kv_heads: int, tp_size: int) -> int:
    """kv heads a rank holds: Hkv / tp, or 1 (replicated) when tp is a multiple of Hkv."""
    if n_kv_heads % tp_size == 0:
        return n_kv_heads // tp_size
    if tp_size % n_kv_heads == 0:
        return 1
    raise ValueError(f"{n_kv_heads} kv heads neither split over nor replicate onto {tp_size} ranks")


def kv_head_first(n_kv_heads: int, tp_size: int, tp_rank: int) -> int:
    """First kv head of rank tp_rank (the group of its q heads)."""
    return tp_rank * kv_heads_local(n_kv_heads, tp_size) if n_kv_heads % tp_size == 0 \
        else tp_rank * n_kv_heads // tp_size


def check_parallel(args, tp_size: int, tp_rank: int, ep_size: int, ep_rank: int) -> None:
    """The partitions the C++ model accepts (m5_model_create)."""
    moe = args.num_experts > 0
    if not moe and ep_size > 1:
        raise ValueError("ep_size > 1 needs a MoE model")
    if tp_size > 1 and ep_size > 1 and (tp_size != ep_size or tp_rank != ep_rank):
        raise ValueError("head-sharded attention with expert parallelism uses the same ranks for both")
    if moe and tp_size > 1 and ep_size != tp_size:
        raise ValueError("a MoE model shards heads only together with its experts (tp_size == ep_size)")
    if args.num_attention_heads % tp_size:
        raise ValueError("num_attention_heads not divisible by tp_size")
    kv_heads_local(args.num_key_value_heads, tp_size)


def shard_weights(w: Dict[str, torch.Tensor], args, tp_size: int = 1, tp_rank: int = 0, ep_size: int = 1,
                  ep_rank: int = 0, experts_local: bool = False) -> Dict[str, torch.Tensor]:
    """This rank's tensors (new contiguous tensors; the full set is not modified).
    ``experts_local``: the expert stacks in ``w`` already hold only this rank's
    experts (``random_weights(experts=...)``) and are taken as they are."""
    if tp_size == 1 and ep_size == 1:
        return dict(w)
    check_parallel(args, tp_size, tp_rank, ep_size, ep_rank)
    out: Dict[str, torch.Tensor] = {}
    D = args.head_dim
    Hkv = args.num_key_value_heads
    for name, t in w.items():
        if name in out:
            continue
        base = name.rsplit(".", 1)[0]
        if ".switch_mlp." in name and ep_size > 1:
            if experts_local:
                out[name] = t
            else:
                _rows(w, base, ep_size, ep_rank, out)  # experts are the leading axis
        elif tp_size > 1 and base.endswith(("self_attn.k_proj", "self_attn.v_proj")):
            n = kv_heads_local(Hkv, tp_size)
            r0 = kv_head_first(Hkv, tp_size, tp_rank) * D
            for suf in (".weight", ".scales", ".biases"):
                out[base + suf] = w[base + suf].narrow(0, r0, n * D).contiguous()
        elif tp_size > 1 and base.endswith(("self_attn.q_proj", "mlp.gate_proj", "mlp.up_proj")):
            _rows(w, base, tp_size, tp_rank, out)  # whole heads / intermediate rows per rank
        elif tp_size > 1 and base.endswith(("self_attn.o_proj", "mlp.down_proj")):
            _col_slice(w, base, tp_size, tp_rank, out)
        elif tp_size > 1 and base == "lm_head":
            _rows(w, base, tp_size, tp_rank, out)
        else:
            out[name] = t
    if tp_size > 1 and args.tie_word_embeddings:
        _rows(w, "lm_head", tp_size, tp_rank, out, src="model.embed_tokens")
    if tp_size > 1:
        h = args.num_attention_heads // tp_size
        assert out[f"model.layers.0.self_attn.q_proj.weight"].shape[0] == h * D
    return out


class Communicator:
    """libm5cuda communicator of this rank, its id exchanged over torch.distributed.

    ``exchange`` overrides how the 128-byte id travels from rank 0 to the others
    (default: ``torch.distributed.broadcast_object_list`` on ``group``)."""

    def __init__(self, world: int, rank: int, group=None, exchange=None):
        self.world, self.rank = world, rank
        buf = ctypes.create_string_buffer(_lib.M5_COMM_ID_BYTES)
        if rank == 0:
            _lib.call("m5_comm_unique_id", buf, _lib.M5_COMM_ID_BYTES)
        payload = bytes(buf.raw) if rank == 0 else None
        if exchange is None:
            import torch.distributed as dist
            obj = [payload]
            dist.broadcast_object_list(obj, src=0, group=group)
            payload = obj[0]
        else:
            payload = exchange(payload)
        if not isinstance(payload, (bytes, bytearray)) or len(payload) != _lib.M5_COMM_ID_BYTES:
            raise RuntimeError("communicator id exchange returned a malformed id")
        self.id = bytes(payload)
        h = ctypes.c_void_p()
        _lib.call("m5_comm_init", ctypes.create_string_buffer(self.id, len(self.id)), len(self.id), world, rank,
                  ctypes.byref(h))
        self.handle = h

    def check(self) -> None:
        """Raise M5CudaError if NCCL reported an asynchronous error (or the
        communicator was aborted)."""
        _lib.call("m5_comm_check", self.handle)

    def abort(self) -> None:
        """Abort the communicator: every later collective fails fast instead of
        waiting on a peer that is gone."""
        if self.handle is not None and self.handle.value:
            _lib.call("m5_comm_abort", self.handle)

    def set_wait_ms(self, ms: int) -> None:
        """Bound on the peer all-reduce's wait for the other ranks."""
        _lib.call("m5_comm_set_wait_ms", self.handle, int(ms))

    def allreduce_(self, t: torch.Tensor) -> torch.Tensor:
        """In-place fp32 sum over the ranks (testing / host utilities)."""
        from .ops import _stream
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("allreduce_ takes a contiguous fp32 CUDA tensor")
        _lib.call("m5_allreduce_f32", self.handle, t.data_ptr(), t.numel(), _stream())
        return t

    def close(self) -> None:
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            _lib.lib().m5_comm_destroy(h)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
