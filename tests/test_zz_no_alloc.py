"""m5_quantized_matmul_noalloc: the allocation-free quantized matmul.

Callers that cannot allocate device memory (a CUDA graph being captured, a
serving host that handed the whole device pool to its own allocator) use
this entry point; it keeps its scratch in an array compiled into the library
instead of a cudaMalloc'd buffer.  Its output must match m5_quantized_matmul
(same kernels, so within the GEMV tolerance of test_gemv_gpu.py, 2^-7 |y| +
1e-3), on two consecutive calls: the shared array keeps the previous call's
contents, and every call must still start from a clean scratch.

This file sorts last so a stop-at-first-failure run has already run every
other test when it gets here.
"""

import ctypes

import numpy as np
import pytest
import torch

from myinfer_b200 import _lib
from oracle.quant import affine_quantize, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _weights(N, K, seed):
    rng = np.random.default_rng(seed)
    w = bf16_bits_to_f32(f32_to_bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32)))
    q, s, b = affine_quantize(w, 64, 4)
    return (torch.from_numpy(q.view(np.int32)).cuda(), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).cuda(),
            torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).cuda())


def _call(name, x, w, N):
    wq, s, b = w
    M, K = x.shape
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    _lib.call(name, x.data_ptr(), M, K, wq.data_ptr(), s.data_ptr(), b.data_ptr(), N, 64, 4, y.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return y


@pytest.mark.parametrize("M,N,K", [(1, 4096, 5120), (3, 2048, 1024), (8, 1000, 2048)])
def test_noalloc_matches_allocating_entry_point(M, N, K):
    w = _weights(N, K, seed=N + K)
    g = torch.Generator(device="cuda").manual_seed(M)
    for call in range(2):  # the second call runs on the first call's leftover scratch
        x = torch.randn(M, K, generator=g, device="cuda").to(torch.bfloat16)
        ref = _call("m5_quantized_matmul", x, w, N).float()
        out = _call("m5_quantized_matmul_noalloc", x, w, N).float()
        torch.cuda.synchronize()
        err = (out - ref).abs()
        assert (err <= ref.abs() * 2 ** -7 + 1e-3).all(), (call, float(err.max()))


def test_noalloc_rejects_oversized_matrix():
    dummy = ctypes.c_void_p(256)
    rc = _lib.lib().m5_quantized_matmul_noalloc(dummy, 1, 64, dummy, dummy, dummy, (1 << 18) + 1, 64, 4, dummy, None)
    assert rc == _lib.M5_ERR_INVALID
    assert "scratch limit" in _lib.last_error()
