"""LoRA merge + block-INT8 quantisation (cf_lora_merge_quantize_int8).

Oracle: the reference's own semantics, quantize_int8(LoRALinear.merged_weight())
(training/lora.py:95-102, python/cudaforge/ops.py:215-229), with the merged
weight computed by torch on the CPU in the module's dtype and quantised by the
numpy restatement of the reference quantiser. The kernel accumulates
lora_b @ lora_a in fp32 in its own order, so a merged value can land one ulp
of the dtype away from torch's when the fp32 sum sits on a rounding boundary;
such elements may move their code by one. The bound: at most 1e-3 of the codes
differ, by at most 1, and scales agree to 2^-7 (one bf16 ulp of the absmax).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cuda_force_b200 as cf
from oracle import quant_ref

pytestmark = pytest.mark.gpu


def _reference(w, a, b, scaling):
    merged = (w + scaling * (b @ a)).contiguous()       # CPU, module dtype
    codes, scales = quant_ref.quantize(merged.float().numpy().reshape(-1))
    return codes.reshape(w.shape), scales


@pytest.mark.parametrize(("out_f", "in_f", "rank", "dtype"), [
    (256, 512, 16, torch.bfloat16),
    (1000, 512, 8, torch.bfloat16),
    (384, 1024, 32, torch.float16),
    (4096, 4096, 16, torch.bfloat16),
    (11008, 4096, 64, torch.bfloat16),
])
def test_merge_quantize_matches_the_reference_composition(out_f, in_f, rank, dtype, cuda_device):
    g = torch.Generator().manual_seed(out_f + rank)
    w = (torch.randn(out_f, in_f, generator=g) * 0.02).to(dtype)
    a = (torch.randn(rank, in_f, generator=g) * 0.05).to(dtype)
    b = (torch.randn(out_f, rank, generator=g) * 0.05).to(dtype)
    scaling = 2.0
    codes, scales = cf.lora_merge_quantize_int8(w.to(cuda_device), a.to(cuda_device),
                                                b.to(cuda_device), scaling)
    ref_codes, ref_scales = _reference(w, a, b, scaling)
    got = codes.cpu().numpy().astype(np.int32)
    diff = np.abs(got - ref_codes.astype(np.int32))
    assert diff.max() <= 1
    assert (diff > 0).mean() <= 1e-3
    rel = np.abs(scales.cpu().numpy() - ref_scales) / ref_scales
    assert rel.max() <= 2.0 ** -7


def test_zero_adapter_is_plain_quantisation(cuda_device):
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(512, 1024, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    a = torch.zeros(16, 1024, dtype=torch.bfloat16, device=cuda_device)
    b = torch.zeros(512, 16, dtype=torch.bfloat16, device=cuda_device)
    codes, scales = cf.lora_merge_quantize_int8(w, a, b, 2.0)
    q_codes, q_scales = cf.quantize_int8(w)
    assert torch.equal(codes, q_codes)
    assert torch.equal(scales, q_scales)


def test_rejects_what_it_cannot_do(cuda_device):
    w = torch.zeros(64, 100, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError, match="multiple of 64"):
        cf.lora_merge_quantize_int8(w, torch.zeros(4, 100, dtype=torch.bfloat16, device=cuda_device),
                                    torch.zeros(64, 4, dtype=torch.bfloat16, device=cuda_device), 1.0)
    w = torch.zeros(64, 128, device=cuda_device)
    with pytest.raises(ValueError, match="float16 or bfloat16"):
        cf.lora_merge_quantize_int8(w, torch.zeros(4, 128, device=cuda_device),
                                    torch.zeros(64, 4, device=cuda_device), 1.0)
