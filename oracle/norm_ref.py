"""Restatement of the reference's RMSNorm and residual-add + RMSNorm.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows python/cudaforge/ops.py:164-171 (``_rmsnorm_reference``) and :188-192
(``_fused_residual_rmsnorm_reference``), the same arithmetic as
cpp/src/bindings.cpp:238-249 and :264-271:

    summed     = x + residual                       (in x's dtype)
    normalised = (f32(summed) * rsqrt(mean(f32(summed)^2) + eps) * f32(weight)).to(dtype)

evaluated on the CPU. The add is one fp32 add and one rounding to the dtype,
so ``summed`` is exact; ``normalised`` differs from a GPU kernel only by the
order of the row's sum of squares and the rsqrt, i.e. by a rounding step of
the dtype at most.
"""

from __future__ import annotations

import torch


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.detach().cpu()
    promoted = x.float()
    variance = promoted.pow(2).mean(dim=-1, keepdim=True)
    normalised = promoted * torch.rsqrt(variance + eps)
    return (normalised * weight.detach().cpu().float()).to(x.dtype)


def fused_residual_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                           eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    summed = x.detach().cpu() + residual.detach().cpu()
    return rmsnorm(summed, weight, eps), summed
