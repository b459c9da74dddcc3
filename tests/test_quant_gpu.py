"""Device affine quantizer (m5_affine_quantize / m5_affine_dequantize) vs the
CPU restatement of the MLX rule: bit-exact codes, scales and biases."""

import numpy as np
import pytest
import torch

from oracle.quant import affine_dequantize, affine_quantize, bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _edge_rows(rng):
    rows = []
    rows.append(np.zeros(64, np.float32))                              # all zero -> q0 == 0 branch
    rows.append(np.full(64, 0.75, np.float32))                         # constant positive
    rows.append(np.full(64, -3.5, np.float32))                         # constant negative
    r = np.zeros(64, np.float32); r[7] = 1.0; rows.append(r)           # one spike
    rows.append(np.linspace(-8.0, 1.0, 64, dtype=np.float32))         # |min| > |max|
    rows.append(np.linspace(-1.0, 8.0, 64, dtype=np.float32))         # |max| > |min|
    rows.append(np.arange(64, dtype=np.float32) % 16 + 0.5)           # half-way codes (round-half-even)
    rows.append(np.arange(64, dtype=np.float32) * 0.5)                # half steps
    rows.append((rng.standard_normal(64) * 1e-6).astype(np.float32))  # tiny range -> eps floor
    rows.append((rng.standard_normal(64) * 3e4).astype(np.float32))   # large magnitude
    rows.append(np.array([1e-30] * 32 + [-1e-30] * 32, np.float32))
    return np.stack(rows)


def _inputs(dtype, rng):
    x = np.concatenate([
        rng.standard_normal((37, 64)).astype(np.float32),
        rng.uniform(-2, 5, (16, 64)).astype(np.float32),
        _edge_rows(rng),
    ]).reshape(-1, 256)
    if dtype == "bf16":
        x = bf16_bits_to_f32(f32_to_bf16_bits(x))
    return x


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_quantize_bit_exact(bits, dtype):
    from myinfer_b200 import ops
    rng = np.random.default_rng(1234 + bits)
    x = _inputs(dtype, rng)
    xt = torch.from_numpy(x).cuda()
    if dtype == "bf16":
        xt = xt.to(torch.bfloat16)
    wq, s, b = ops.quantize(xt, 64, bits)
    rq, rs, rb_ = affine_quantize(x, 64, bits)
    assert np.array_equal(wq.cpu().numpy().view(np.uint32), rq)
    assert np.array_equal(s.cpu().view(torch.int16).numpy().view(np.uint16), rs)
    assert np.array_equal(b.cpu().view(torch.int16).numpy().view(np.uint16), rb_)


@pytest.mark.parametrize("bits", [4, 8])
def test_dequantize_exact(bits):
    from myinfer_b200 import ops
    rng = np.random.default_rng(7)
    x = bf16_bits_to_f32(f32_to_bf16_bits(rng.standard_normal((64, 512)).astype(np.float32)))
    rq, rs, rb_ = affine_quantize(x, 64, bits)
    dev = [torch.from_numpy(rq.view(np.int32)).cuda(),
           torch.from_numpy(rs.view(np.int16)).view(torch.bfloat16).cuda(),
           torch.from_numpy(rb_.view(np.int16)).view(torch.bfloat16).cuda()]
    out = ops.dequantize(*dev, 64, bits).float().cpu().numpy()
    ref = bf16_bits_to_f32(f32_to_bf16_bits(affine_dequantize(rq, rs, rb_, 64, bits)))
    assert np.array_equal(out, ref)


def test_quantize_large_matrix_matches_oracle():
    """A weight-sized matrix (the path random_weights uses) round-trips bit-exactly."""
    from myinfer_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(5)
    w = (0.02 * torch.randn(1024, 3072, generator=g, device="cuda")).to(torch.bfloat16)
    wq, s, b = ops.quantize(w, 64, 4)
    rq, rs, rb_ = affine_quantize(w.float().cpu().numpy(), 64, 4)
    assert np.array_equal(wq.cpu().numpy().view(np.uint32), rq)
    assert np.array_equal(s.cpu().view(torch.int16).numpy().view(np.uint16), rs)
    assert np.array_equal(b.cpu().view(torch.int16).numpy().view(np.uint16), rb_)
