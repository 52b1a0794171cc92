"""Restatement of the reference's LoRA linear for parity checks.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows python/cudaforge/ops.py:178-185 (``_lora_linear_reference``) and
cpp/src/bindings.cpp:255-258 (``lora_linear_cpu``):

    y = x @ w + scale * ((x @ a) @ b)        w: [in, out], a: [in, r], b: [r, out]

evaluated on the CPU in float32 (or float64) from the *same* bf16/fp16 inputs
the kernel sees (upcast exactly), so the only differences left are the kernel's
accumulation order and its bf16 output rounding. The W8 variant dequantises
with the quantisation oracle first (bit-exact to the reference), i.e.
``lora_linear(x, dequantize(codes, scales).reshape(n, k).T, a, b, scale)``.
"""

from __future__ import annotations

import torch

from oracle import quant_ref


def lora_linear(x: torch.Tensor, w: torch.Tensor, a: torch.Tensor, b: torch.Tensor, scale: float,
                dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """x [M,K], w [K,N], a [K,r], b [r,N] (any float dtype, any device) -> y [M,N] on CPU."""
    x, w, a, b = (t.detach().to("cpu", dtype) for t in (x, w, a, b))
    return x @ w + scale * ((x @ a) @ b)


def dequantized_weight_t(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """codes int8 [N,K] + scales -> W^T float32 [K,N] via the quantisation oracle."""
    n, k = codes.shape
    deq = quant_ref.dequantize(codes.detach().cpu().numpy(), scales.detach().cpu().numpy())
    return torch.from_numpy(deq).reshape(n, k).t()


def lora_linear_int8(x: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, a: torch.Tensor,
                     b: torch.Tensor, scale: float,
                     dtype: torch.dtype = torch.float32) -> torch.Tensor:
    return lora_linear(x, dequantized_weight_t(codes, scales), a, b, scale, dtype)


def max_rel_error(y: torch.Tensor, ref: torch.Tensor) -> float:
    """max|y - ref| / max|ref| — the tolerance metric for the linears (bound 2e-2)."""
    y = y.detach().to("cpu", torch.float64)
    ref = ref.detach().to("cpu", torch.float64)
    denom = ref.abs().max().item()
    return (y - ref).abs().max().item() / (denom if denom > 0 else 1.0)
