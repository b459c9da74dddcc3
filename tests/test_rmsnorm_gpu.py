"""m5_rms_norm (mx.fast.rms_norm as mlx-lm's Qwen3 norms call it) against an
fp32 torch reference with the same rounding points: y = bf16(w * bf16(x *
rsqrt(mean(x^2) + eps))).  Rows of 16-byte-aligned width run the vectorised
kernel, others the scalar one; the sum of squares is added in a different
order than the reference's, so outputs may differ by one bf16 step."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,dim", [(16, 5120), (3, 2048), (5, 8192), (4, 1004), (2, 12288)],
                         ids=["vec5120", "vec2048", "vec8192", "scalar1004", "scalar12288"])
def test_rms_norm_matches_reference(rows, dim):
    from myinfer_b200 import ops
    g = torch.Generator().manual_seed(dim)
    x = (3 * torch.randn(rows, dim, generator=g)).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    got = ops.rms_norm(x.cuda(), w.cuda(), 1e-6).float().cpu()
    xf = x.float()
    inv = torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + 1e-6)
    ref = (w.float() * (xf * inv).to(torch.bfloat16).float()).to(torch.bfloat16).float()
    step = ref.abs().clamp_min(1e-3) * 2.0 ** -7
    assert ((got - ref).abs() <= step + 1e-6).all()
    assert (got == ref).float().mean().item() > 0.98
