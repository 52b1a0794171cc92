"""Residual add + RMSNorm (cf_fused_residual_rmsnorm) against the reference.

Oracle: the reference's composition (python/cudaforge/ops.py:164-171,
188-192; oracle/norm_ref.py) and the golden fixture made from it and from the
reference's compiled CPU operators (tests/golden/norm_cases.npz). Bars:
``summed`` (residual_out) bit-exact, since it is one add and one rounding;
``normalised`` within one rounding step of the dtype of the reference
(|d| <= 2^-7 |ref| for bf16, 2^-10 |ref| + 2^-24 for fp16, and the
reference's own fp32 tolerance rtol 1e-5 / atol 1e-6, tests/python/
test_ops.py:24), because the row's sum of squares is added in another order
and rsqrt is the hardware's.
"""

from __future__ import annotations

import pytest
import torch

import cuda_force_b200 as cf
from cuda_force_b200 import _abi
from oracle import norm_ref
from tests.helpers import TORCH_TO_CF, norm_cases, ptr, stream_ptr

pytestmark = pytest.mark.gpu


def assert_one_step(got: torch.Tensor, ref: torch.Tensor) -> None:
    got64 = got.detach().cpu().double()
    ref64 = ref.detach().cpu().double()
    if ref.dtype == torch.bfloat16:
        tol = ref64.abs() * 2.0**-7
    elif ref.dtype == torch.float16:
        tol = ref64.abs() * 2.0**-10 + 2.0**-24
    else:
        tol = ref64.abs() * 1e-5 + 1e-6
    bad = (got64 - ref64).abs() > tol
    assert not bad.any(), (f"{int(bad.sum())} of {bad.numel()} outside one step; worst "
                           f"{(got64 - ref64).abs().max().item():.3g}")


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    view = torch.int16 if a.element_size() == 2 else torch.int32
    return torch.equal(a.detach().cpu().view(view), b.detach().cpu().view(view))


@pytest.mark.parametrize("name", sorted(norm_cases()))
def test_norm_matches_reference_fixture(name, cuda_device):
    case = norm_cases()[name]
    x, r, w = (case[k].to(cuda_device) for k in ("x", "residual", "weight"))
    normalised, summed = cf.fused_residual_rmsnorm(x, r, w, case["eps"])
    assert bits_equal(summed, case["summed"])
    assert_one_step(normalised, case["normalised"])
    assert_one_step(cf.rmsnorm(x, w, case["eps"]), case["plain"])


@pytest.mark.parametrize(("rows", "cols", "dtype", "wdtype"), [
    (4096, 4096, torch.bfloat16, torch.bfloat16),   # 2 resident chunks per thread
    (32, 8192, torch.bfloat16, torch.float32),      # 4 resident chunks, fp32 weight
    (513, 4096, torch.float32, torch.float32),      # fp32, 4 resident chunks
    (300, 20000, torch.bfloat16, torch.bfloat16),   # long rows: second pass re-reads
    (64, 12288, torch.float32, torch.float32),      # long fp32 rows
    (77, 1000, torch.float16, torch.float16),       # 1000 % 8 != 0: element-wise form
    (3000, 96, torch.float16, torch.float32),       # short rows, many per CTA
])
def test_norm_matches_reference_composition(rows, cols, dtype, wdtype, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(rows * 7 + cols)
    x = torch.randn(rows, cols, generator=g, device=cuda_device).to(dtype)
    r = torch.randn(rows, cols, generator=g, device=cuda_device).to(dtype)
    w = (1 + 0.1 * torch.randn(cols, generator=g, device=cuda_device)).to(wdtype)
    normalised, summed = cf.fused_residual_rmsnorm(x, r, w)
    ref_norm, ref_sum = norm_ref.fused_residual_rmsnorm(x, r, w, 1e-6)
    assert bits_equal(summed, ref_sum)
    assert_one_step(normalised, ref_norm)
    assert_one_step(cf.rmsnorm(x, w), norm_ref.rmsnorm(x, w, 1e-6))


def test_norm_keeps_leading_dimensions(cuda_device):
    x = torch.randn(2, 17, 256, device=cuda_device, dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.rand(256, device=cuda_device, dtype=torch.bfloat16)
    normalised, summed = cf.fused_residual_rmsnorm(x, r, w)
    assert normalised.shape == summed.shape == x.shape
    ref_norm, ref_sum = norm_ref.fused_residual_rmsnorm(x, r, w, 1e-6)
    assert bits_equal(summed, ref_sum)
    assert_one_step(normalised, ref_norm)


def test_norm_zero_rows_give_zero(cuda_device):
    # rsqrt(0 + eps) is finite, so an all-zero row normalises to zeros (the
    # reference's behaviour; with eps = 0 it would be NaN in both).
    x = torch.zeros(5, 512, device=cuda_device, dtype=torch.bfloat16)
    normalised, summed = cf.fused_residual_rmsnorm(x, x.clone(), torch.ones(512, device=cuda_device,
                                                                           dtype=torch.bfloat16))
    assert torch.count_nonzero(normalised).item() == 0 and torch.count_nonzero(summed).item() == 0


def _abi_call(x, r, w, out, ro, rows, cols, dtype, eps=1e-6):
    lib = _abi.load()
    return lib.cf_fused_residual_rmsnorm(
        ptr(x), ptr(r) if r is not None else None, ptr(w), TORCH_TO_CF[w.dtype], ptr(out),
        ptr(ro) if ro is not None else None, rows, cols, eps, TORCH_TO_CF[dtype], stream_ptr())


def test_c_abi_in_place_and_misaligned(cuda_device):
    rows, cols = 33, 2048
    x = torch.randn(rows, cols, device=cuda_device, dtype=torch.bfloat16)
    r = torch.randn_like(x)
    w = torch.rand(cols, device=cuda_device, dtype=torch.bfloat16)
    ref_norm, ref_sum = norm_ref.fused_residual_rmsnorm(x, r, w, 1e-6)
    # in place: output over x, residual_out over residual (vector path)
    xi, ri = x.clone(), r.clone()
    assert _abi_call(xi, ri, w, xi, ri, rows, cols, torch.bfloat16) == _abi.CF_OK
    torch.cuda.synchronize()
    assert bits_equal(ri, ref_sum)
    assert_one_step(xi, ref_norm)
    # every tensor one element off a 16-byte boundary: element-wise form
    n = rows * cols
    buf = [torch.empty(n + 8, device=cuda_device, dtype=torch.bfloat16) for _ in range(4)]
    xs, rs, out, ro = (b[1:n + 1].view(rows, cols) for b in buf)
    xs.copy_(x)
    rs.copy_(r)
    assert _abi_call(xs, rs, w, out, ro, rows, cols, torch.bfloat16) == _abi.CF_OK
    torch.cuda.synchronize()
    assert bits_equal(ro, ref_sum)
    assert_one_step(out, ref_norm)
    # plain rmsnorm through the C ABI (no residual)
    out2 = torch.empty_like(x)
    assert _abi_call(x, None, w, out2, None, rows, cols, torch.bfloat16) == _abi.CF_OK
    torch.cuda.synchronize()
    assert_one_step(out2, norm_ref.rmsnorm(x, w, 1e-6))


def test_torch_op_matches_reference_schema_outputs(cuda_device):
    x = torch.randn(8, 4096, device=cuda_device)
    r = torch.randn_like(x)
    w = torch.rand(4096, device=cuda_device)
    out = torch.ops.cudaforge.fused_residual_rmsnorm(x, r, w, 1e-6)
    assert isinstance(out, list) and len(out) == 2
    ref_norm, ref_sum = norm_ref.fused_residual_rmsnorm(x, r, w, 1e-6)
    assert bits_equal(out[1], ref_sum)
    assert_one_step(out[0], ref_norm)
    assert_one_step(torch.ops.cudaforge.rmsnorm(x, w, 1e-6), norm_ref.rmsnorm(x, w, 1e-6))


@pytest.mark.parametrize(("dtype", "wdtype"), [
    (torch.float32, torch.bfloat16),
    (torch.bfloat16, torch.float16),
])
def test_norm_weight_of_another_dtype_is_widened(dtype, wdtype, cuda_device):
    # The reference composition multiplies by weight.float() whatever its dtype.
    x = torch.randn(19, 768, device=cuda_device).to(dtype)
    r = torch.randn_like(x)
    w = (1 + 0.1 * torch.randn(768, device=cuda_device)).to(wdtype)
    normalised, summed = cf.fused_residual_rmsnorm(x, r, w)
    ref_norm, ref_sum = norm_ref.fused_residual_rmsnorm(x, r, w, 1e-6)
    assert bits_equal(summed, ref_sum)
    assert_one_step(normalised, ref_norm)
    assert_one_step(cf.rmsnorm(x, w), norm_ref.rmsnorm(x, w, 1e-6))
