"""m5_quantized_matmul_noalloc: the allocation-free quantized matmul.

Some callers of this library cannot allocate device memory: a serving host
whose own allocator reserved the whole device pool at start-up, or an
embedder that forbids allocation once it is running.  This entry point keeps
its scratch in an array compiled into the library instead of a cudaMalloc'd
buffer.  Its output must match m5_quantized_matmul and the fp32 product on
the oracle's dequantized weights within the GEMV tolerance of
test_gemv_gpu.py (2^-7 |y| + 1e-3), on two consecutive calls: the shared
array keeps the previous call's contents, and every call must still start
from a clean scratch.  M > 8 runs several GEMV launches over the same array
in one call.  After the first call on the device, further calls leave the
device's free memory unchanged.

This file sorts last so a stop-at-first-failure run has already run every
other test when it gets here.
"""

import ctypes

import numpy as np
import pytest
import torch

from myinfer_b200 import _lib
from oracle.quant import affine_dequantize, affine_quantize, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _weights(N, K, seed):
    rng = np.random.default_rng(seed)
    w = bf16_bits_to_f32(f32_to_bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32)))
    q, s, b = affine_quantize(w, 64, 4)
    dev = (torch.from_numpy(q.view(np.int32)).cuda(), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).cuda(),
           torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).cuda())
    return dev, torch.from_numpy(affine_dequantize(q, s, b, 64, 4))


def _call(name, x, w, N, y=None):
    wq, s, b = w
    M, K = x.shape
    if y is None:
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _lib.call(name, x.data_ptr(), M, K, wq.data_ptr(), s.data_ptr(), b.data_ptr(), N, 64, 4, y.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return y


def _close(out, ref):
    err = (out - ref).abs()
    return bool((err <= ref.abs() * 2 ** -7 + 1e-3).all()), float(err.max())


@pytest.mark.parametrize("M,N,K", [(1, 4096, 5120), (3, 2048, 1024), (8, 1000, 2048), (13, 1536, 1024),
                                   (40, 512, 3072)])
def test_noalloc_matches_allocating_entry_point(M, N, K):
    w, wd = _weights(N, K, seed=N + K)
    g = torch.Generator(device="cuda").manual_seed(M)
    for call in range(2):  # the second call runs on the first call's leftover scratch
        x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
        ref = _call("m5_quantized_matmul", x, w, N).float()
        out = _call("m5_quantized_matmul_noalloc", x, w, N).float()
        torch.cuda.synchronize()
        ok, err = _close(out, ref)
        assert ok, ("vs m5_quantized_matmul", call, err)
        fp32 = (x.float().cpu() @ wd.T).to(torch.bfloat16).float()
        ok, err = _close(out.cpu(), fp32)
        assert ok, ("vs the fp32 product on the oracle's weights", call, err)


def test_noalloc_leaves_free_memory_unchanged():
    N, K, M = 2048, 2048, 13
    w, _ = _weights(N, K, seed=3)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ref = _call("m5_quantized_matmul", x, w, N).float()
    _call("m5_quantized_matmul_noalloc", x, w, N, y)  # first call on the device: looks the array up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        _call("m5_quantized_matmul_noalloc", x, w, N, y)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    ok, err = _close(y.float(), ref)
    assert ok, err


def test_noalloc_rejects_oversized_matrix():
    dummy = ctypes.c_void_p(256)
    rc = _lib.lib().m5_quantized_matmul_noalloc(dummy, 1, 64, dummy, dummy, dummy, (1 << 18) + 1, 64, 4, dummy, None)
    assert rc == _lib.M5_ERR_INVALID
    assert "scratch limit" in _lib.last_error()
