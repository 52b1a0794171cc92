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


@pytest.mark.parametrize(("m", "k", "n", "r", "int8"), [
    (256, 4096, 4096, 16, False),     # benchmark config 3, 256 of its 8192 rows
    (32, 4096, 11008, 16, True),      # benchmark config 4 decode
    (256, 4096, 11008, 16, True),     # benchmark config 4 prefill, 256 of its 4096 rows
    (7, 129, 65, 3, False),           # the reference's own ragged test shape
])
def test_linear_oracle_matches_the_compiled_reference(m, k, n, r, int8):
    # oracle/linear_ref against the reference's own compiled CPU operators
    # (cpp/src/bindings.cpp:255-258 lora_linear_cpu, :320-329 dequantize_int8_cpu), on the
    # same bf16-valued inputs upcast to fp32, the dtype the reference's operator takes.
    from oracle import build_ref

    if not build_ref.load():
        pytest.skip("the reference's CPU operators are not built (oracle/_ref)")
    g = torch.Generator().manual_seed(m * 7 + k + n)
    x = torch.randn(m, k, generator=g).bfloat16()
    w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    a = (torch.randn(k, r, generator=g) * 0.01).bfloat16()
    b = (torch.randn(r, n, generator=g) * 0.01).bfloat16()
    if int8:
        codes, scales = torch.ops.cudaforge_ref.quantize_int8(w.float())
        codes = codes.reshape(n, k)
        ours = linear_ref.lora_linear_int8(x, codes, scales, a, b, 2.0)
        w_t = torch.ops.cudaforge_ref.dequantize_int8(codes, scales).reshape(n, k).t()
    else:
        ours = linear_ref.lora_linear(x, w.t(), a, b, 2.0)
        w_t = w.float().t()
    ref = torch.ops.cudaforge_ref.lora_linear(x.float(), w_t.contiguous(), a.float(),
                                              b.float(), 2.0)
    # Both are fp32 ATen compositions of the same formula; only the GEMM blocking of a
    # contiguous versus a transposed operand may differ.
    assert linear_ref.max_rel_error(ours, ref) <= 1e-6
