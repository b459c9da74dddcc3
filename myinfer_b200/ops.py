"""Tensor-level wrappers of the libm5cuda kernels (mx.* ops the reference calls).

Each function takes CUDA torch tensors, checks shapes/dtypes, and calls the C
ABI on the current torch stream.  Packed quantized weights are int32 tensors
holding the uint32 words bit for bit (torch has no general uint32 arithmetic).
"""

from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import M5KvView, call


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _need_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libm5cuda ops take CUDA tensors")


def quantize(x: torch.Tensor, group_size: int = 64, bits: int = 4) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``mx.quantize``: x [..., K] (bf16 or fp32) -> (wq int32 [..., K*bits/32], scales, biases bf16)."""
    _need_cuda(x)
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("quantize expects bf16 or fp32 input")
    x = x.contiguous()
    K = x.shape[-1]
    rows = x.numel() // max(K, 1)
    lead = x.shape[:-1]
    wq = torch.empty(*lead, K * bits // 32, dtype=torch.int32, device=x.device)
    s = torch.empty(*lead, K // group_size, dtype=torch.bfloat16, device=x.device)
    b = torch.empty_like(s)
    dt = _lib.M5_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.M5_DTYPE_F32
    call("m5_affine_quantize", x.data_ptr(), dt, rows, K, K, group_size, bits, wq.data_ptr(), s.data_ptr(),
         b.data_ptr(), _stream())
    return wq, s, b


def dequantize(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4) -> torch.Tensor:
    _need_cuda(wq, scales, biases)
    K = wq.shape[-1] * 32 // bits
    rows = wq.numel() // wq.shape[-1]
    out = torch.empty(*wq.shape[:-1], K, dtype=torch.bfloat16, device=wq.device)
    call("m5_affine_dequantize", wq.contiguous().data_ptr(), scales.contiguous().data_ptr(),
         biases.contiguous().data_ptr(), rows, K, group_size, bits, out.data_ptr(), _stream())
    return out


def quantized_matmul(x: torch.Tensor, wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``mx.quantized_matmul(x, w, scales, biases, transpose=True)`` for bf16 x.

    Up to 15 tokens run on the streaming decode GEMV; 16 or more on the
    tensor-core GEMM (K a multiple of 512, N of 128), else the GEMV in chunks."""
    if not transpose:
        raise NotImplementedError("only transpose=True (x @ W.T) is implemented")
    _need_cuda(x, wq, scales, biases)
    if x.dtype != torch.bfloat16:
        raise ValueError("quantized_matmul expects bf16 activations")
    x2 = x.contiguous().reshape(-1, x.shape[-1])
    N = wq.shape[-2]
    y = out if out is not None else torch.empty(x2.shape[0], N, dtype=torch.bfloat16, device=x.device)
    if y.shape != (x2.shape[0], N) or y.dtype != torch.bfloat16 or not y.is_contiguous():
        raise ValueError("out must be a contiguous bf16 tensor of shape [tokens, N]")
    call("m5_quantized_matmul", x2.data_ptr(), x2.shape[0], x2.shape[1], wq.data_ptr(), scales.data_ptr(),
         biases.data_ptr(), N, group_size, bits, y.data_ptr(), _stream())
    return y.reshape(*x.shape[:-1], N)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    _need_cuda(x, w)
    x2 = x.contiguous()
    y = torch.empty_like(x2)
    D = x.shape[-1]
    call("m5_rms_norm", x2.data_ptr(), w.contiguous().data_ptr(), x2.numel() // D, D, eps, y.data_ptr(), _stream())
    return y


def argmax(x: torch.Tensor) -> torch.Tensor:
    """Greedy sampler over bf16 logits (first index wins a tie); int32 tensor [1]."""
    _need_cuda(x)
    out = torch.empty(1, dtype=torch.int32, device=x.device)
    xc = x.contiguous()
    call("m5_argmax_bf16", xc.data_ptr(), xc.numel(), out.data_ptr(), _stream())
    return out


def moe_route(x: torch.Tensor, gate: Tuple[torch.Tensor, torch.Tensor, torch.Tensor], k: int,
              norm_topk_prob: bool = True):
    """Qwen3-MoE router: (ids int32 [T, k], scores bf16 [T, k], logits bf16 [T, E])."""
    wq, s, b = gate
    _need_cuda(x, wq, s, b)
    x2 = x.contiguous().reshape(-1, x.shape[-1])
    T, H = x2.shape
    E = wq.shape[0]
    ids = torch.empty(T, k, dtype=torch.int32, device=x.device)
    scores = torch.empty(T, k, dtype=torch.bfloat16, device=x.device)
    logits = torch.empty(T, E, dtype=torch.bfloat16, device=x.device)
    call("m5_moe_route", x2.data_ptr(), T, H, wq.data_ptr(), s.data_ptr(), b.data_ptr(), E, k,
         int(norm_topk_prob), ids.data_ptr(), scores.data_ptr(), logits.data_ptr(), _stream())
    return ids, scores, logits


def kv_view(t, head_stride: int, batch_stride: int) -> M5KvView:
    """M5KvView of a K or V operand: a bf16 tensor or an MLX (wq, scales, biases) tuple."""
    if isinstance(t, torch.Tensor):
        return M5KvView(t.data_ptr(), None, None, batch_stride, head_stride)
    wq, s, b = t
    return M5KvView(wq.data_ptr(), s.data_ptr(), b.data_ptr(), batch_stride, head_stride)


def mask_strides(mask: torch.Tensor, B: int, H: int) -> "ctypes.Array":
    """(batch, head, row) element strides of a mask broadcast to [B, H, L, S]."""
    m = mask
    while m.dim() < 4:
        m = m.unsqueeze(0)
    st = [m.stride(i) if m.shape[i] != 1 else 0 for i in range(3)]
    if m.stride(3) != 1:
        raise ValueError("mask's last axis must be contiguous")
    return (ctypes.c_int64 * 3)(*st)
