"""Prefill dequant-GEMM (tcgen05, M >= 16 tokens) vs an fp32 reference on the
dequantized weights.  The kernel sums s * (sum q x) per group plus a bias term
b * sum(x) split into bf16 hi + lo; the reference sums (q s + b) x.  Both are
fp32 accumulations in different orders, so bf16 outputs may differ by one
rounding step: tolerance |d| <= 2^-7 |y| + 1e-3 (as for the decode GEMV)."""

import numpy as np
import pytest
import torch

from oracle.quant import affine_dequantize, affine_quantize, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _weights(N, K, seed, std=0.02):
    rng = np.random.default_rng(seed)
    w = bf16_bits_to_f32(f32_to_bf16_bits((std * rng.standard_normal((N, K))).astype(np.float32)))
    q, s, b = affine_quantize(w, 64, 4)
    dev = (torch.from_numpy(q.view(np.int32)).cuda(), torch.from_numpy(s.view(np.int16)).view(torch.bfloat16).cuda(),
           torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).cuda())
    return dev, torch.from_numpy(affine_dequantize(q, s, b, 64, 4))


def _check(y, ref):
    err = (y - ref).abs()
    bad = ~(err <= ref.abs() * 2 ** -7 + 1e-3)
    assert not bad.any(), (int(bad.sum()), float(err.max()), bad.nonzero()[:5].tolist())


@pytest.mark.parametrize("M", [16, 77, 128, 300])
@pytest.mark.parametrize("N,K", [(128, 512), (1024, 1024), (384, 5120), (256, 3072), (128, 25600),
                                 (256, 3200), (128, 576), (384, 6400)])
def test_gemm_matches_reference(M, N, K):
    from myinfer_b200 import ops
    (wq, s, b), wd = _weights(N, K, seed=N * 3 + K)
    g = torch.Generator().manual_seed(M + K)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    y = ops.quantized_matmul(x.cuda(), wq, s, b).float().cpu()
    ref = (x.float() @ wd.T).to(torch.bfloat16).float()
    _check(y, ref)


def test_gemm_bias_heavy_inputs():
    """Inputs with a large common offset make the b * sum(x) term dominate and
    cancel against s * sum(q x): the hi/lo split of the group sums must hold."""
    from myinfer_b200 import ops
    (wq, s, b), wd = _weights(256, 2048, seed=11, std=0.05)
    g = torch.Generator().manual_seed(5)
    x = (torch.randn(64, 2048, generator=g) * 0.1 + 3.0).to(torch.bfloat16)
    y = ops.quantized_matmul(x.cuda(), wq, s, b).float().cpu()
    ref = (x.double() @ wd.double().T).float().to(torch.bfloat16).float()
    _check(y, ref)


def test_gemm_deterministic_and_matches_gemv_rows():
    """Bitwise repeatable; a 16-token GEMM row equals the 1-token GEMV of that
    row within one bf16 step."""
    from myinfer_b200 import ops
    (wq, s, b), _ = _weights(512, 1024, seed=2)
    x = torch.randn(40, 1024, device="cuda").to(torch.bfloat16)
    y1 = ops.quantized_matmul(x, wq, s, b)
    y2 = ops.quantized_matmul(x, wq, s, b)
    assert torch.equal(y1, y2)
    for t in (0, 17, 39):
        r = ops.quantized_matmul(x[t:t + 1], wq, s, b).float()
        d = (y1[t:t + 1].float() - r).abs()
        assert (d <= r.abs() * 2 ** -7 + 1e-3).all()


def test_gemm_status_clean():
    from myinfer_b200 import _lib
    import ctypes
    code = ctypes.c_int(-1)
    _lib.call("m5_device_status", ctypes.byref(code), 1)
    assert code.value == 0
