"""Parity of the sm_100a quantise / dequantise / fake-quant kernels.

Bit-exact against the golden fixtures (generated from the reference) and the
oracle, through both the C ABI (ctypes, raw pointers) and the dispatcher ops;
size-independent properties at the benchmark sizes; edge cases the reference tests
(tests/python/test_ops.py:164-228, tests/cuda/test_quantization.cu:55-158).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cuda_force_b200 as cf
from cuda_force_b200 import _abi
from oracle import quant_ref
from tests.helpers import (
    TORCH_TO_CF,
    golden_cases,
    golden_hashes,
    numpy_to_torch,
    ptr,
    regenerate,
    sha,
    stream_ptr,
    torch_to_numpy_input,
)

pytestmark = pytest.mark.gpu

CASES = golden_cases()


def abi_quantize(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _abi.load()
    n = x.numel()
    codes = torch.empty(n, dtype=torch.int8, device=x.device)
    scales = torch.empty(lib.cf_quant_scale_count(n), dtype=torch.float32, device=x.device)
    _abi.check(lib.cf_quantize_int8(ptr(x), TORCH_TO_CF[x.dtype], ptr(codes), ptr(scales), n,
                                    stream_ptr()), "cf_quantize_int8")
    return codes, scales


def abi_dequantize(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    lib = _abi.load()
    out = torch.empty(codes.numel(), dtype=torch.float32, device=codes.device)
    _abi.check(lib.cf_dequantize_int8(ptr(codes), ptr(scales), ptr(out), codes.numel(),
                                      stream_ptr()), "cf_dequantize_int8")
    return out


def bits(t: torch.Tensor) -> np.ndarray:
    """float32 bit patterns with every NaN mapped to one canonical pattern.

    Bit-exact comparison, except that NaN payloads are not compared: 0 * inf
    is the NaN 0xffc00000 on x86 and 0x7fffffff on the GPU, both meaning NaN.
    """
    a = t.detach().cpu().contiguous().view(torch.int32).numpy().copy()
    a[np.isnan(a.view(np.float32))] = 0x7FC00000
    return a


def golden_bits(a: np.ndarray) -> np.ndarray:
    out = a.view(np.int32).copy()
    out[np.isnan(a)] = 0x7FC00000
    return out


@pytest.mark.parametrize("name", sorted(CASES))
def test_golden_case_through_the_abi(name, cuda_device):
    case = CASES[name]
    x = numpy_to_torch(case["dtype"], case["input"]).to(cuda_device)
    codes, scales = abi_quantize(x)
    np.testing.assert_array_equal(codes.cpu().numpy(), case["codes"])
    np.testing.assert_array_equal(bits(scales), golden_bits(case["scales"]))
    deq = abi_dequantize(codes, scales)
    np.testing.assert_array_equal(bits(deq), golden_bits(case["deq"]))


@pytest.mark.parametrize("name", sorted(CASES))
def test_golden_case_through_the_dispatcher(name, cuda_device):
    case = CASES[name]
    x = numpy_to_torch(case["dtype"], case["input"]).to(cuda_device)
    codes, scales = cf.quantize_int8(x)
    assert codes.shape == x.shape and scales.dim() == 1
    np.testing.assert_array_equal(codes.cpu().numpy().reshape(-1), case["codes"])
    np.testing.assert_array_equal(bits(scales), golden_bits(case["scales"]))
    np.testing.assert_array_equal(bits(cf.dequantize_int8(codes, scales)).reshape(-1),
                                  golden_bits(case["deq"]))
    np.testing.assert_array_equal(bits(cf.quantize_dequantize(x)).reshape(-1),
                                  golden_bits(case["deq"]))


@pytest.mark.parametrize("name", sorted(golden_hashes()))
def test_large_golden_hashes(name, cuda_device):
    entry = golden_hashes()[name]
    arr = regenerate(entry["dtype"], entry["spec"])
    assert sha(arr) == entry["input"]
    x = numpy_to_torch(entry["dtype"], arr).to(cuda_device)
    codes, scales = cf.quantize_int8(x)
    assert sha(codes.cpu().numpy()) == entry["codes"]
    assert sha(scales.cpu().numpy()) == entry["scales"]
    assert sha(cf.dequantize_int8(codes, scales).cpu().numpy()) == entry["deq"]
    assert sha(cf.quantize_dequantize(x).cpu().numpy()) == entry["deq"]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("size", [1, 63, 64, 65, 127, 4096 * 3 + 1, 1 << 20, (1 << 20) + 37])
def test_matches_oracle_on_seeded_inputs(dtype, size, cuda_device):
    g = torch.Generator(device="cpu").manual_seed(size)
    x = (torch.randn(size, generator=g) * 5).to(dtype)
    codes, scales = cf.quantize_int8(x.to(cuda_device))
    ref_codes, ref_scales = quant_ref.quantize(torch_to_numpy_input(x))
    np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes)
    np.testing.assert_array_equal(scales.cpu().numpy().view(np.int32), ref_scales.view(np.int32))


@pytest.mark.parametrize("offset", [1, 2, 3, 4, 8, 17])
def test_misaligned_views_take_the_scalar_path_correctly(offset, cuda_device):
    base = torch.randn(64 * 1000 + offset + 5, device=cuda_device)
    x = base[offset:offset + 64 * 1000 + 3]
    codes_buf = torch.empty(x.numel() + offset, dtype=torch.int8, device=cuda_device)
    codes = codes_buf[offset:]
    lib = _abi.load()
    scales = torch.empty(lib.cf_quant_scale_count(x.numel()), device=cuda_device)
    _abi.check(lib.cf_quantize_int8(ptr(x), 0, ptr(codes), ptr(scales), x.numel(), stream_ptr()),
               "quantize")
    ref_codes, ref_scales = quant_ref.quantize(x.cpu().numpy())
    np.testing.assert_array_equal(codes.cpu().numpy(), ref_codes)
    np.testing.assert_array_equal(scales.cpu().numpy(), ref_scales)
    out_buf = torch.empty(x.numel() + 1, device=cuda_device)
    out = out_buf[1:]
    _abi.check(lib.cf_dequantize_int8(ptr(codes), ptr(scales), ptr(out), x.numel(), stream_ptr()),
               "dequantize")
    np.testing.assert_array_equal(out.cpu().numpy(), quant_ref.dequantize(ref_codes, ref_scales))


def test_round_trip_bound_and_range_at_config1_size(cuda_device):
    # Size-independent properties (reference test_ops.py:174-187,
    # test_quantization.cu:62-121) at benchmark config 1's size.
    g = torch.Generator(device=cuda_device).manual_seed(11)
    x = torch.randn(4096, 4096, device=cuda_device, generator=g)
    codes, scales = cf.quantize_int8(x)
    restored = cf.dequantize_int8(codes, scales)
    per_block = (x - restored).abs().reshape(-1, 64).amax(dim=1)
    assert torch.all(per_block <= scales / 2 + 1e-6)
    assert codes.min().item() >= -127 and codes.max().item() <= 127
    peak = codes.reshape(-1, 64).gather(1, x.reshape(-1, 64).abs().argmax(dim=1, keepdim=True))
    assert torch.all(peak.abs() == 127)


def test_all_zero_input_round_trips_exactly(cuda_device):
    x = torch.zeros(128, device=cuda_device)
    codes, scales = cf.quantize_int8(x)
    assert torch.all(scales > 0)
    assert torch.equal(cf.dequantize_int8(codes, scales), x)


def test_outlier_only_degrades_its_own_block(cuda_device):
    x = torch.full((256,), 0.5, device=cuda_device)
    x[0] = 1000.0
    codes, scales = cf.quantize_int8(x)
    restored = cf.dequantize_int8(codes, scales)
    assert (x[1] - restored[1]).abs() > (x[200] - restored[200]).abs()
    assert (x[200] - restored[200]).abs() < 0.01
    assert restored[0].item() == 1000.0


def test_grouped_quantisation_equals_single_calls(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(3)
    shapes = [(4096, 64), (1000, 4), (11008, 128), (65,), (2048, 512)]
    tensors = [(torch.randn(s, device=cuda_device, generator=g) * 0.02).to(torch.bfloat16)
               for s in shapes]
    grouped = cf.quantize_int8_many(tensors)
    for t, (codes, scales) in zip(tensors, grouped):
        c1, s1 = cf.quantize_int8(t)
        assert torch.equal(codes, c1) and torch.equal(scales, s1)


def test_llama_layer_bf16_matches_oracle_bit_exact(cuda_device):
    # One Llama-2-7B layer of benchmark config 2 (7 projections, N(0,0.02),
    # 0.1% outliers x20, bf16), grouped launch, checked block for block.
    g = torch.Generator(device=cuda_device).manual_seed(1234)
    shapes = [(4096, 4096)] * 4 + [(11008, 4096)] * 2 + [(4096, 11008)]
    tensors = []
    for s in shapes:
        w = torch.randn(s, device=cuda_device, generator=g) * 0.02
        mask = torch.rand(s, device=cuda_device, generator=g) < 0.001
        tensors.append(torch.where(mask, w * 20, w).to(torch.bfloat16))
    grouped = cf.quantize_int8_many(tensors)
    for t, (codes, scales) in zip(tensors, grouped):
        ref_codes, ref_scales = quant_ref.quantize(torch_to_numpy_input(t))
        np.testing.assert_array_equal(codes.cpu().numpy().reshape(-1), ref_codes)
        np.testing.assert_array_equal(scales.cpu().numpy(), ref_scales)


def test_count_above_two_to_the_31(cuda_device):
    # The reference's launchers take `int count` and overflow here.
    n = (1 << 31) + 64 * 3 + 5
    x = torch.empty(n, dtype=torch.bfloat16, device=cuda_device)
    x.normal_(generator=torch.Generator(device=cuda_device).manual_seed(9))
    codes, scales = cf.quantize_int8(x)
    assert scales.numel() == (n + 63) // 64
    rng = np.random.default_rng(0)
    blocks = np.concatenate([rng.integers(0, scales.numel(), 64), [scales.numel() - 1,
                                                                   (1 << 31) // 64]])
    for b in blocks.tolist():
        lo, hi = b * 64, min(n, b * 64 + 64)
        ref_c, ref_s = quant_ref.quantize(torch_to_numpy_input(x[lo:hi]))
        np.testing.assert_array_equal(codes[lo:hi].cpu().numpy(), ref_c)
        assert scales[b].item() == ref_s[0]
    del x, codes, scales
    torch.cuda.empty_cache()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("size", [1, 63, 64, 65, 128, 1000, 4096 * 4096])
def test_quantization_error_is_within_half_a_step(dtype, size, cuda_device):
    # reference python/cudaforge/ops.py:479-488 (quantization_error) and the bound its tests
    # hold it to (tests/python/test_ops.py:174-181, 225-229): the round trip errs by at most
    # half the largest block scale, and the helper equals a manual round trip. Here both sides
    # are also checked against the oracle's dequantised values, bit for bit.
    g = torch.Generator().manual_seed(size)
    x = (torch.randn(size, generator=g) * 5.0).to(dtype)
    xd = x.to(cuda_device)
    err = cf.quantization_error(xd)
    codes, scales = cf.quantize_int8(xd)
    manual = (xd.float() - cf.dequantize_int8(codes, scales)).abs().max()
    assert torch.equal(err, manual)
    assert err.item() <= scales.max().item() / 2 + 1e-6
    ref_codes, ref_scales = quant_ref.quantize(torch_to_numpy_input(x))
    ref = torch.from_numpy(quant_ref.dequantize(ref_codes, ref_scales))
    assert err.item() == (x.float() - ref).abs().max().item()


def test_dequantise_of_a_large_tensor_takes_the_bulk_path_bit_exact(cuda_device):
    # 2^26 elements and more run on the bulk-copy dequantiser (whole 2048-code
    # tiles), the remainder (here 4096 + 37 elements) on the register path.
    n = (1 << 26) + 4096 + 37
    g = torch.Generator(device=cuda_device).manual_seed(26)
    codes = torch.randint(-127, 128, (n,), generator=g, device=cuda_device, dtype=torch.int8)
    scales = torch.rand((n + 63) // 64, generator=g, device=cuda_device) * 0.1
    out = cf.dequantize_int8(codes, scales)
    ref = quant_ref.dequantize(codes.cpu().numpy(), scales.cpu().numpy())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
