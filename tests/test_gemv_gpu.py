"""Dequant-GEMV (m5_quantized_matmul) vs an fp32 reference on the dequantized
weights.  Both accumulate in fp32 in different orders, so the bf16 outputs may
differ by one bf16 rounding step: tolerance |d| <= 2^-7 |y| + 1e-3."""

import numpy as np
import pytest
import torch

from oracle.quant import affine_dequantize, affine_quantize, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _weights(N, K, seed):
    rng = np.random.default_rng(seed)
    w = bf16_bits_to_f32(f32_to_bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32)))
    q, s, b = affine_quantize(w, 64, 4)
    dev = (torch.from_numpy(q.view(np.int32)).cuda(), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).cuda(),
           torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).cuda())
    return dev, torch.from_numpy(affine_dequantize(q, s, b, 64, 4))


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8, 13])
# K % 1024 != 0 with K % 512 == 0 (1536, 2560, 12800): the tensor-map kernel's
# partial last unit of a row, e.g. a down_proj sharded over 2 ranks (25600 / 2);
# 1280 and 3328 (K % 512 != 0) take the register-fed GEMV
@pytest.mark.parametrize("N,K", [(256, 1024), (1000, 2048), (384, 5120), (96, 25600), (4096, 64), (33, 1088),
                                 (512, 1536), (48, 2560), (160, 12800), (512, 1280), (48, 3328)])
def test_quantized_matmul(M, N, K):
    from myinfer_b200 import ops
    (wq, s, b), wd = _weights(N, K, seed=N * 7 + K)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = ops.quantized_matmul(x.cuda(), wq, s, b).float().cpu()
    ref = (x.float() @ wd.T).to(torch.bfloat16).float()
    err = (y - ref).abs()
    assert (err <= ref.abs() * 2 ** -7 + 1e-3).all(), float(err.max())
