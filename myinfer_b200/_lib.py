"""ctypes binding of libm5cuda.so (the C ABI declared in include/m5cuda.h).

There is no fallback: if the library is missing or a call fails, an
``M5CudaError`` is raised.  Torch tensors are only used to carry device
pointers and streams.
"""

from __future__ import annotations

import ctypes
import re
from ctypes import POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32, c_uint64, c_void_p
from pathlib import Path
from typing import List, Optional

LIB_PATH = Path(__file__).resolve().with_name("libm5cuda.so")
HEADER_PATH = Path(__file__).resolve().parent.parent / "include" / "m5cuda.h"

M5_OK, M5_ERR_INVALID, M5_ERR_CUDA, M5_ERR_UNSUPPORTED, M5_ERR_TIMEOUT, M5_ERR_COMM, M5_ERR_STATE = range(7)
M5_DTYPE_BF16, M5_DTYPE_F32 = 0, 1
M5_MASK_NONE, M5_MASK_CAUSAL, M5_MASK_BOOL, M5_MASK_ADDITIVE = range(4)
M5_LOGITS_NONE, M5_LOGITS_LAST, M5_LOGITS_ALL = range(3)
M5_SAMPLE_APPEND_HISTORY = 1


class M5CudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[m5 error {code}] {msg}")
        self.code = code


class M5KvView(ctypes.Structure):
    _fields_ = [("data", c_void_p), ("scales", c_void_p), ("biases", c_void_p),
                ("batch_stride", c_int64), ("head_stride", c_int64)]


class M5LayerKv(ctypes.Structure):
    _fields_ = [("k", c_void_p), ("k_scales", c_void_p), ("k_biases", c_void_p),
                ("v", c_void_p), ("v_scales", c_void_p), ("v_biases", c_void_p),
                ("capacity", c_int64), ("bits", c_int), ("group_size", c_int)]


class M5SampleParams(ctypes.Structure):
    _fields_ = [("temperature", c_float), ("top_p", c_float), ("min_p", c_float), ("top_k", c_int),
                ("repetition_penalty", c_float), ("presence_penalty", c_float), ("frequency_penalty", c_float),
                ("flags", c_int), ("seed", c_uint64), ("offset", c_uint64)]


class M5ModelCfg(ctypes.Structure):
    _fields_ = [(n, c_int) for n in (
        "hidden_size", "num_layers", "num_heads", "num_kv_heads", "head_dim", "intermediate_size",
        "vocab_size", "num_experts", "experts_per_tok", "moe_intermediate_size", "norm_topk_prob",
        "tie_word_embeddings")] + [("rms_norm_eps", c_float)] + [(n, c_int) for n in (
            "group_size", "bits", "tp_size", "tp_rank", "ep_size", "ep_rank")]


_SIGS = {
    "m5_version": (c_int, []),
    "m5_last_error": (c_size_t, [c_char_p, c_size_t]),
    "m5_device_status": (c_int, [POINTER(c_int), c_int]),
    "m5_affine_quantize": (c_int, [c_void_p, c_int, c_int64, c_int64, c_int64, c_int, c_int, c_void_p,
                                   c_void_p, c_void_p, c_void_p]),
    "m5_affine_dequantize": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int, c_int,
                                     c_void_p, c_void_p]),
    "m5_quantized_matmul": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64,
                                    c_int, c_int, c_void_p, c_void_p]),
    "m5_quantized_matmul_noalloc": (c_int, [c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_int64,
                                            c_int, c_int, c_void_p, c_void_p]),
    "m5_rms_norm": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_float, c_void_p, c_void_p]),
    "m5_quantized_sdpa": (c_int, [c_void_p, c_int, c_int, c_int, c_int, M5KvView, M5KvView, c_int, c_int,
                                  c_float, c_int, c_void_p, POINTER(c_int64), c_int, c_int, c_void_p,
                                  c_void_p]),
    "m5_model_create": (c_int, [POINTER(M5ModelCfg), POINTER(c_void_p)]),
    "m5_model_destroy": (c_int, [c_void_p]),
    "m5_model_bind": (c_int, [c_void_p, c_char_p, c_void_p]),
    "m5_model_check": (c_int, [c_void_p]),
    "m5_model_set_rope": (c_int, [c_void_p, POINTER(c_float), c_float]),
    "m5_model_reserve": (c_int, [c_void_p, c_int]),
    "m5_forward": (c_int, [c_void_p, POINTER(M5LayerKv), c_void_p, c_void_p, c_int, c_void_p, c_int,
                           c_void_p, c_void_p]),
    "m5_forward_batch": (c_int, [c_void_p, POINTER(M5LayerKv), c_void_p, c_void_p, c_int, c_void_p, c_int,
                                 c_void_p, c_void_p]),
    "m5_kv_quantize_layer": (c_int, [POINTER(M5LayerKv), POINTER(M5LayerKv), c_int, c_int, c_int, c_void_p]),
    "m5_argmax_bf16": (c_int, [c_void_p, c_int64, c_void_p, c_void_p]),
    "m5_sample_bf16": (c_int, [c_void_p, c_int, c_int64, c_int64, c_void_p, c_int, c_int64,
                               POINTER(M5SampleParams), c_void_p, c_void_p, c_void_p]),
    "m5_moe_route": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                             c_void_p, c_void_p, c_void_p, c_void_p]),
    "m5_comm_unique_id": (c_int, [c_void_p, c_size_t]),
    "m5_comm_init": (c_int, [c_void_p, c_size_t, c_int, c_int, POINTER(c_void_p)]),
    "m5_comm_destroy": (c_int, [c_void_p]),
    "m5_model_set_comm": (c_int, [c_void_p, c_void_p]),
    "m5_allreduce_f32": (c_int, [c_void_p, c_void_p, c_int64, c_void_p]),
    "m5_comm_check": (c_int, [c_void_p]),
    "m5_comm_abort": (c_int, [c_void_p]),
    "m5_comm_set_wait_ms": (c_int, [c_void_p, c_int]),
    "m5_comm_peer_wait_selftest": (c_int, [c_int, POINTER(c_int), POINTER(ctypes.c_double), POINTER(c_int)]),
}
M5_COMM_ID_BYTES = 128

_lib: Optional[ctypes.CDLL] = None


def header_symbols() -> List[str]:
    """Every function the public header declares."""
    text = HEADER_PATH.read_text()
    return re.findall(r"^M5_API\s+\w+\s+(m5_\w+)\s*\(", text, flags=re.M)


def lib() -> ctypes.CDLL:
    """Load libm5cuda.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise M5CudaError(M5_ERR_STATE, f"{LIB_PATH.name} is not built; run `python -m myinfer_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(2048)
    lib().m5_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != M5_OK:
        raise M5CudaError(rc, last_error())


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def device_check() -> None:
    """Raise if a kernel on the current device recorded an error: a bounded
    wait that ran out (a TMA copy or a peer rank that never arrived).  The
    error words are cleared when read, so each failure is reported once."""
    code = c_int(0)
    call("m5_device_status", ctypes.byref(code), 1)
    if code.value:
        raise M5CudaError(M5_ERR_TIMEOUT, f"device reported error code {code.value}: a bounded wait ran out "
                                          "(a copy that never landed or a peer rank that never arrived)")
