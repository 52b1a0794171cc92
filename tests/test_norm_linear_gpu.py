"""RMSNorm folded into the W8 + LoRA linear (cf_rmsnorm_lora_linear_int8).

Against the reference's composition, restated by the oracle: the residual add
and RMSNorm of python/cudaforge/ops.py:164-171 / 335-382 (oracle/norm_ref,
the normalised rows rounded to the activation dtype as the reference's op
returns them), then the W8 linear (oracle/linear_ref, fp32). The folded route
rounds differently (the norm weight meets each dequantised code before the
one rounding to bf16, and the row scale is applied to the fp32 accumulator),
so the product is held to the linears' tolerance; residual_out is bit-exact.
Shapes cover the folded route (m > 128) and the decode route (m <= 128).
"""

from __future__ import annotations

import pytest
import torch

import cuda_force_b200 as cf
from oracle import linear_ref, norm_ref

pytestmark = pytest.mark.gpu

TIGHT = 5e-3


def case(m, k, n, r, dtype, device, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    res = torch.randn(m, k, generator=g).to(dtype)
    nw = (1.0 + 0.1 * torch.randn(k, generator=g)).to(dtype)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dtype)
    a = (torch.randn(k, r, generator=g) * 0.01).to(dtype)
    b = (torch.randn(r, n, generator=g) * 0.01).to(dtype)
    codes, scales = cf.quantize_int8(w.to(device))
    return x, res, nw, codes, scales, a, b


def oracle(x, res, nw, codes, scales, a, b, scale, eps, rows):
    if res is not None:
        normed, summed = norm_ref.fused_residual_rmsnorm(x[rows], res[rows], nw, eps)
    else:
        normed, summed = norm_ref.rmsnorm(x[rows], nw, eps), None
    return linear_ref.lora_linear_int8(normed, codes, scales, a, b, scale), summed


@pytest.mark.parametrize(("m", "k", "n", "r", "dtype"), [
    (512, 1024, 768, 16, torch.bfloat16),
    (1000, 2048, 1280, 64, torch.bfloat16),
    (700, 1024, 512, 8, torch.float16),
    (4096, 4096, 11008, 16, torch.bfloat16),   # benchmark config 4 prefill shape
    (32, 4096, 1024, 16, torch.bfloat16),      # decode route
])
@pytest.mark.parametrize("with_residual", [True, False])
def test_matches_the_reference_composition(m, k, n, r, dtype, with_residual, cuda_device):
    x, res, nw, codes, scales, a, b = case(m, k, n, r, dtype, cuda_device, seed=m + k + n)
    res = res if with_residual else None
    d = lambda t: t.to(cuda_device) if t is not None else None  # noqa: E731
    y, res_out = cf.rmsnorm_lora_linear_int8(d(x), d(res), d(nw), codes, scales, d(a), d(b),
                                             2.0, 1e-6)
    torch.cuda.synchronize()
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(1))[:128]
    ref, summed = oracle(x, res, nw, codes, scales, a, b, 2.0, 1e-6, rows)
    assert linear_ref.max_rel_error(y.cpu()[rows], ref) <= TIGHT
    if with_residual:
        assert torch.equal(res_out.cpu(), x + res)
        assert torch.equal(res_out.cpu()[rows], summed)
    else:
        assert res_out is None
    # and against the unfused route through this package's own kernels
    if with_residual:
        normed, _ = cf.fused_residual_rmsnorm(d(x), d(res), d(nw), 1e-6)
    else:
        normed = cf.rmsnorm(d(x), d(nw), 1e-6)
    y2 = cf.lora_linear_int8(normed, codes, scales, d(a), d(b), 2.0)
    assert linear_ref.max_rel_error(y, y2) <= TIGHT


def test_rejects_bad_shapes(cuda_device):
    x, res, nw, codes, scales, a, b = case(256, 512, 256, 16, torch.bfloat16, cuda_device, 3)
    d = lambda t: t.to(cuda_device)  # noqa: E731
    with pytest.raises(ValueError, match="norm_weight"):
        cf.rmsnorm_lora_linear_int8(d(x), d(res), d(nw[:-1]), codes, scales, d(a), d(b))
    with pytest.raises(ValueError, match="residual"):
        cf.rmsnorm_lora_linear_int8(d(x), d(res[:-1]), d(nw), codes, scales, d(a), d(b))
