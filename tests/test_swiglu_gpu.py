"""W8 gate/up projections with SwiGLU fused (cf_w8_swiglu_int8).

Oracle: the reference's transformer-block composition on the CPU
(examples/transformer_block.py:84-87): g = x @ dequantize(Wg).T and
u = x @ dequantize(Wu).T rounded to x's dtype, then silu(g) * u with
silu(v) = v / (1 + exp(-v)) (cuda/src/activations.cu:19-21) in fp32, rounded
once. Bar: max|h - ref| / max|ref| <= 1e-2, inside the path's 2e-2 tolerance: the two
products accumulate in fp32 in a different order, which can move g or u by one
ulp of the dtype before h is rounded again (measured up to ~1.5 bf16 ulps of
the largest output, 6.6e-3).
"""

from __future__ import annotations

import pytest
import torch

import cuda_force_b200 as cf
from oracle import linear_ref

pytestmark = pytest.mark.gpu


def _reference(x, gc, gs, uc, us, dtype):
    wg = linear_ref.dequantized_weight_t(gc, gs).cpu().float()
    wu = linear_ref.dequantized_weight_t(uc, us).cpu().float()
    xf = x.cpu().float()
    g = (xf @ wg).to(dtype).float()
    u = (xf @ wu).to(dtype).float()
    return (g / (1.0 + torch.exp(-g)) * u).to(dtype).float()


@pytest.mark.parametrize(("m", "k", "n", "dtype"), [
    (300, 1024, 768, torch.bfloat16),
    (129, 512, 1000, torch.float16),
    (1, 256, 136, torch.bfloat16),
    (4096, 4096, 11008, torch.bfloat16),
    (200, 320, 384, torch.bfloat16),    # K/64 not a multiple of 4: the two-accumulator kernel
    (700, 2048, 1000, torch.float16),   # N not a multiple of 64
])
def test_swiglu_matches_the_reference_composition(m, k, n, dtype, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(m + n)
    x = torch.randn(m, k, device=cuda_device, generator=g).to(dtype)
    wg = (torch.randn(n, k, device=cuda_device, generator=g) * 0.02).to(dtype)
    wu = (torch.randn(n, k, device=cuda_device, generator=g) * 0.02).to(dtype)
    gc, gs = cf.quantize_int8(wg)
    uc, us = cf.quantize_int8(wu)
    h = cf.w8_swiglu_int8(x, gc, gs, uc, us)
    assert h.shape == (m, n) and h.dtype == dtype
    rows = torch.randperm(m, generator=torch.Generator().manual_seed(0))[:256].sort().values
    ref = _reference(x[rows.to(cuda_device)], gc, gs, uc, us, dtype)
    got = h[rows.to(cuda_device)].cpu().float()
    assert (got - ref).abs().max() <= 1e-2 * ref.abs().max()


def test_leading_dims_and_errors(cuda_device):
    x = torch.randn(2, 3, 256, device=cuda_device).to(torch.bfloat16)
    w = (torch.randn(128, 256, device=cuda_device) * 0.02).to(torch.bfloat16)
    c, s = cf.quantize_int8(w)
    assert cf.w8_swiglu_int8(x, c, s, c, s).shape == (2, 3, 128)
    with pytest.raises(ValueError, match="float16 or bfloat16"):
        cf.w8_swiglu_int8(x.float(), c, s, c, s)
    with pytest.raises(ValueError, match="input features"):
        cf.w8_swiglu_int8(x[..., :128], c, s, c, s)
