"""The oracle, pinned against the golden fixtures generated from the reference.

CPU only. Both restatements (numpy and C) must reproduce the reference's codes,
scales and dequantised values bit for bit on every golden case.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import linear_ref, norm_ref, quant_ref
from tests.helpers import golden_cases, norm_cases, golden_hashes, regenerate, sha

CASES = golden_cases()


@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("impl", ["numpy", "c"])
def test_oracle_matches_reference_fixture(name, impl):
    case = CASES[name]
    quant = quant_ref.quantize if impl == "numpy" else quant_ref.c_quantize
    deq = quant_ref.dequantize if impl == "numpy" else quant_ref.c_dequantize
    codes, scales = quant(case["input"])
    np.testing.assert_array_equal(codes, case["codes"])
    np.testing.assert_array_equal(scales.view(np.uint32), case["scales"].view(np.uint32))
    np.testing.assert_array_equal(deq(codes, scales).view(np.uint32), case["deq"].view(np.uint32))


@pytest.mark.parametrize("name", sorted(golden_hashes()))
def test_oracle_matches_reference_hashes(name):
    entry = golden_hashes()[name]
    arr = regenerate(entry["dtype"], entry["spec"])
    assert sha(arr) == entry["input"], "regenerated input differs from the fixture's"
    codes, scales = quant_ref.quantize(arr)
    assert sha(codes) == entry["codes"]
    assert sha(scales) == entry["scales"]
    assert sha(quant_ref.dequantize(codes, scales)) == entry["deq"]


def test_scale_count_known_answers():
    # reference tests/cuda/test_quantization.cu:55-60 (0/1/64/65 -> 0/1/1/2)
    assert [quant_ref.scale_count(n) for n in (0, 1, 64, 65)] == [0, 1, 1, 2]


def test_block_max_maps_to_127_and_round_trips():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(64 * 100) * 5).astype(np.float32)
    codes, scales = quant_ref.quantize(x)
    blocks = x.reshape(-1, 64)
    idx = np.abs(blocks).argmax(axis=1)
    peak = codes.reshape(-1, 64)[np.arange(100), idx]
    assert np.all(np.abs(peak) == 127)


def test_reciprocal_shortcut_would_break_parity():
    # Documents why the kernels divide (or verify near ties): multiplying by
    # a reciprocal of 127 changes scales on a seeded input.
    rng = np.random.default_rng(1)
    x = rng.standard_normal(64 * 4096, dtype=np.float32)
    absmax = np.abs(x.reshape(-1, 64)).max(axis=1)
    exact = absmax / np.float32(127)
    recip = absmax * (np.float32(1) / np.float32(127))
    assert np.any(exact != recip)


def test_linear_oracle_definition():
    g = torch.Generator().manual_seed(0)
    x, w = torch.randn(7, 129, generator=g), torch.randn(129, 65, generator=g)
    a, b = torch.randn(129, 3, generator=g), torch.randn(3, 65, generator=g)
    y = linear_ref.lora_linear(x, w, a, b, 0.25, dtype=torch.float64)
    x, w, a, b = (t.double() for t in (x, w, a, b))
    torch.testing.assert_close(y, x @ w + 0.25 * ((x @ a) @ b), rtol=1e-12, atol=1e-12)


def test_linear_oracle_int8_uses_dequantised_weight():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(32, 128, generator=g) * 0.02
    codes, scales = quant_ref.quantize(w.numpy())
    wt = linear_ref.dequantized_weight_t(torch.from_numpy(codes).reshape(32, 128),
                                         torch.from_numpy(scales))
    assert wt.shape == (128, 32)
    assert (wt.t() - w).abs().max().item() <= scales.max() / 2 + 1e-9


@pytest.mark.parametrize("name", sorted(norm_cases()))
def test_norm_oracle_matches_reference_fixture(name):
    # Bit for bit: the fixture came from the reference's composition and its
    # compiled CPU operators (which agreed bit for bit when it was made).
    case = norm_cases()[name]
    normalised, summed = norm_ref.fused_residual_rmsnorm(case["x"], case["residual"],
                                                         case["weight"], case["eps"])
    plain = norm_ref.rmsnorm(case["x"], case["weight"], case["eps"])
    for got, key in ((normalised, "normalised"), (summed, "summed"), (plain, "plain")):
        assert torch.equal(got, case[key]), key
