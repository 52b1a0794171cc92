"""Parity of the tcgen05 LoRA linears against the fp32 oracle.

Tolerance (the path's stated bf16 bar): max|y - ref| / max|ref| <= 2e-2 with fp32
accumulation, ref = the reference's formula (python/cudaforge/ops.py:178-185)
evaluated in fp32 on the CPU from the same bf16/fp16 inputs. The kernel rounds
P = scale * x A to the activation dtype before the up-projection and its output
to the activation dtype, so typical errors are ~1e-3; the tests assert the
stated bound and a tighter bound that catches a broken tile (5e-3).

Covers every storage layout of w / a / b (reference [in, out] order and the
nn.Linear transposes), ranks 16/32/64 plus padded small ranks, bf16 and fp16,
ragged M / N / K, the W8 variant, and the reference's semantic tests
(tests/python/test_ops.py:101-138: definition, zero-B, linearity in scale).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import cuda_force_b200 as cf
from cuda_force_b200 import _abi
from oracle import linear_ref

pytestmark = pytest.mark.gpu

TOL = 2e-2
TIGHT = 5e-3


def make(m, k, n, r, dtype, seed=0, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dtype)      # nn.Linear layout [out, in]
    a = (torch.randn(k, r, generator=g) * 0.01).to(dtype)
    b = (torch.randn(r, n, generator=g) * 0.01).to(dtype)
    return x, w, a, b


def as_layout(t: torch.Tensor, transposed: bool) -> torch.Tensor:
    """The same logical matrix, stored contiguous (REF) or as a transposed view (T)."""
    return t.t().contiguous().t() if transposed else t.contiguous()


@pytest.mark.parametrize("w_t", [False, True])
@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
def test_every_layout(w_t, a_t, b_t, cuda_device):
    x, w, a, b = make(256, 512, 384, 16, torch.bfloat16, seed=1)
    dev = cuda_device
    wk = as_layout(w.t().to(dev), w_t)   # logical [K, N]
    ak = as_layout(a.to(dev), a_t)
    bk = as_layout(b.to(dev), b_t)
    y = cf.lora_linear(x.to(dev), wk, ak, bk, 2.0)
    ref = linear_ref.lora_linear(x, w.t(), a, b, 2.0)
    err = linear_ref.max_rel_error(y, ref)
    assert err <= TIGHT, f"layout w_t={w_t} a_t={a_t} b_t={b_t}: {err}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rank", [16, 32, 64, 4, 8, 2])
def test_ranks_and_dtypes(dtype, rank, cuda_device):
    x, w, a, b = make(384, 1024, 512, rank, dtype, seed=rank)
    a = a * 10  # make the adapter visible next to the frozen path
    b = b * 10
    dev = cuda_device
    y = cf.lora_linear(x.to(dev), w.to(dev).t(), a.to(dev), b.to(dev), 32.0 / rank)
    ref = linear_ref.lora_linear(x, w.t(), a, b, 32.0 / rank)
    assert y.dtype == dtype
    assert linear_ref.max_rel_error(y, ref) <= TIGHT


@pytest.mark.parametrize(("m", "k", "n"), [(1, 64, 256), (33, 128, 264), (200, 200, 96),
                                           (129, 4160, 520), (1000, 256, 8)])
def test_ragged_shapes(m, k, n, cuda_device):
    x, w, a, b = make(m, k, n, 16, torch.bfloat16, seed=m)
    dev = cuda_device
    y = cf.lora_linear(x.to(dev), w.to(dev).t(), a.to(dev), b.to(dev), 2.0)
    assert y.shape == (m, n)
    assert linear_ref.max_rel_error(y, linear_ref.lora_linear(x, w.t(), a, b, 2.0)) <= TIGHT


def test_adapter_path_alone(cuda_device):
    # W = 0 isolates the adapter; linear in scale (reference test_ops.py:130-138).
    x, w, a, b = make(256, 256, 256, 16, torch.bfloat16, seed=5)
    dev = cuda_device
    w0 = torch.zeros_like(w).to(dev)
    y1 = cf.lora_linear(x.to(dev), w0.t(), a.to(dev), b.to(dev), 1.0).float()
    y2 = cf.lora_linear(x.to(dev), w0.t(), a.to(dev), b.to(dev), 2.0).float()
    ref1 = linear_ref.lora_linear(x, torch.zeros(256, 256), a, b, 1.0)
    assert linear_ref.max_rel_error(y1, ref1) <= TOL
    torch.testing.assert_close(y2, 2 * y1, rtol=2e-2, atol=1e-3)


def test_zero_b_reduces_to_the_frozen_layer(cuda_device):
    x, w, a, b = make(256, 512, 256, 16, torch.bfloat16, seed=6)
    dev = cuda_device
    y = cf.lora_linear(x.to(dev), w.to(dev).t(), a.to(dev), torch.zeros_like(b).to(dev), 2.0)
    frozen = (x.float() @ w.float().t())
    assert linear_ref.max_rel_error(y, frozen) <= TIGHT


def test_int8_weight_matches_dequantised_composition(cuda_device):
    x, w, a, b = make(256, 1024, 768, 16, torch.bfloat16, seed=7)
    dev = cuda_device
    codes, scales = cf.quantize_int8(w.to(dev))
    y = cf.lora_linear_int8(x.to(dev), codes, scales, a.to(dev), b.to(dev), 2.0)
    ref = linear_ref.lora_linear_int8(x, codes.cpu(), scales.cpu(), a, b, 2.0)
    assert linear_ref.max_rel_error(y, ref) <= TIGHT
    # and it equals the bf16 path fed with the dequantised weight, up to rounding
    wdq = cf.dequantize_int8(codes, scales).to(torch.bfloat16)
    y_bf16 = cf.lora_linear(x.to(dev), wdq.t(), a.to(dev), b.to(dev), 2.0)
    assert linear_ref.max_rel_error(y, y_bf16) <= 1e-2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize(("m", "rank", "a_t", "b_t"), [(32, 16, False, False), (300, 32, True, True),
                                                       (64, 64, False, True)])
def test_int8_variants(dtype, m, rank, a_t, b_t, cuda_device):
    x, w, a, b = make(m, 512, 1024, rank, dtype, seed=m + rank)
    dev = cuda_device
    codes, scales = cf.quantize_int8(w.to(dev))
    y = cf.lora_linear_int8(x.to(dev), codes, scales, as_layout(a.to(dev), a_t),
                            as_layout(b.to(dev), b_t), 2.0)
    ref = linear_ref.lora_linear_int8(x, codes.cpu(), scales.cpu(), a, b, 2.0)
    assert linear_ref.max_rel_error(y, ref) <= TIGHT


def test_through_the_c_abi(cuda_device):
    m, k, n, r = 256, 512, 512, 16
    x, w, a, b = (t.to(cuda_device) for t in make(m, k, n, r, torch.bfloat16, seed=8))
    lib = _abi.load()
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda_device)
    ws_bytes = lib.cf_lora_linear_workspace_bytes(m, r)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    _abi.check(lib.cf_lora_linear(p(x), p(w), _abi.CF_LAYOUT_T, p(a), _abi.CF_LAYOUT_REF, p(b),
                                  _abi.CF_LAYOUT_REF, p(y), m, k, n, r, 2.0, _abi.CF_DTYPE_BF16,
                                  p(ws), ws_bytes, s), "cf_lora_linear")
    ref = linear_ref.lora_linear(x, w.t(), a, b, 2.0)
    assert linear_ref.max_rel_error(y, ref) <= TIGHT
    assert lib.cf_device_status() == _abi.CF_OK


def sampled_rows_error(y, x, w_t, a, b, scale, rows=256, seed=0):
    g = torch.Generator().manual_seed(seed)
    idx = torch.randperm(x.shape[0], generator=g)[:rows].to(x.device)
    ref = linear_ref.lora_linear(x[idx], w_t, a, b, scale)
    return linear_ref.max_rel_error(y[idx], ref)


def test_baseline_config3_bf16_lora(cuda_device):
    # x [8192, 4096] N(0,1); W [4096, 4096] N(0, 0.02); A, B N(0, 0.01); r 16, alpha 32.
    g = torch.Generator(device=cuda_device).manual_seed(3)
    x = torch.randn(8192, 4096, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(4096, 4096, device=cuda_device, generator=g) * 0.02).to(torch.bfloat16)
    a = (torch.randn(4096, 16, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(16, 4096, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    y = cf.lora_linear(x, w.t(), a, b, 2.0)
    assert sampled_rows_error(y, x, w.t(), a, b, 2.0) <= TIGHT


@pytest.mark.parametrize("m", [32, 4096])
def test_baseline_config4_w8_lora(m, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(4)
    x = torch.randn(m, 4096, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(11008, 4096, device=cuda_device, generator=g) * 0.02).to(torch.bfloat16)
    a = (torch.randn(4096, 16, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(16, 11008, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    codes, scales = cf.quantize_int8(w)
    y = cf.lora_linear_int8(x, codes, scales, a, b, 2.0)
    w_t = linear_ref.dequantized_weight_t(codes, scales)
    assert sampled_rows_error(y, x, w_t, a, b, 2.0, rows=min(m, 256)) <= TIGHT


@pytest.mark.parametrize("rank", [16, 32, 64])
def test_w8_many_tiles_per_cta(rank, cuda_device):
    # Several 512-token tiles per CTA with rank/16 adapter k-steps each: the
    # converter warps must stay in phase with stages that carry adapter tiles.
    g = torch.Generator(device=cuda_device).manual_seed(50 + rank)
    m, k, n = 4096, 2048, 8192
    x = torch.randn(m, k, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=cuda_device, generator=g) * 0.015).to(torch.bfloat16)
    a = (torch.randn(k, rank, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(rank, n, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    codes, scales = cf.quantize_int8(w)
    y = cf.lora_linear_int8(x, codes, scales, a, b, 2.0)
    w_t = linear_ref.dequantized_weight_t(codes, scales)
    assert sampled_rows_error(y, x, w_t, a, b, 2.0, rows=1024) <= TIGHT


def _w8_case(m, k, n, rank, device, seed):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(m, k, device=device, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=device, generator=g) * 0.015).to(torch.bfloat16)
    a = (torch.randn(k, rank, device=device, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(rank, n, device=device, generator=g) * 0.01).to(torch.bfloat16)
    codes, scales = cf.quantize_int8(w)
    return x, codes, scales, a, b


@pytest.mark.parametrize("mode", ["kernel", "ce"])
@pytest.mark.parametrize(("m", "rank"), [(1536, 64), (700, 16), (5000, 32)])
@pytest.mark.parametrize("n_dest", [3, 8])
def test_multi_destination_entry_points(mode, m, rank, n_dest, cuda_device):
    # n_dest destinations on one GPU (8 = the most a call takes) stand in for
    # the ranks' copies of y; this call owns columns [col0, col0 + n) of each
    # [m, ldy] destination.
    k, n, ldy, col0 = 1024, 1024, 3072, 1024
    x, codes, scales, a, b = _w8_case(m, k, n, rank, cuda_device, seed=m + rank)
    dests = [torch.full((m, ldy), 7.0, dtype=torch.bfloat16, device=cuda_device)
             for _ in range(n_dest)]
    ptrs = (ctypes.c_void_p * n_dest)(*[t.data_ptr() for t in dests])
    lib = _abi.load()
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    if mode == "ce":
        ws_bytes = lib.cf_lora_linear_int8_allgather_ce_workspace_bytes(m, rank)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
        _abi.check(lib.cf_lora_linear_int8_allgather_ce(
            p(x), p(codes), p(scales), p(a), _abi.CF_LAYOUT_REF, p(b), _abi.CF_LAYOUT_REF, n_dest,
            ptrs, 1, ldy, col0, m, k, n, rank, 2.0, _abi.CF_DTYPE_BF16, p(ws), ws_bytes, s),
            "cf_lora_linear_int8_allgather_ce")
    else:
        ws_bytes = lib.cf_lora_linear_workspace_bytes(m, rank)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
        _abi.check(lib.cf_lora_linear_int8_allgather(
            p(x), p(codes), p(scales), p(a), _abi.CF_LAYOUT_REF, p(b), _abi.CF_LAYOUT_REF, n_dest,
            ptrs, 1, ldy, col0, m, k, n, rank, 2.0, _abi.CF_DTYPE_BF16, p(ws), ws_bytes, s),
            "cf_lora_linear_int8_allgather")
    torch.cuda.synchronize()
    assert lib.cf_device_status() == _abi.CF_OK
    y = cf.lora_linear_int8(x, codes, scales, a, b, 2.0)
    for d in dests:
        assert torch.equal(d[:, col0:col0 + n], y)
        assert (d[:, :col0] == 7.0).all() and (d[:, col0 + n:] == 7.0).all()
    w_t = linear_ref.dequantized_weight_t(codes, scales)
    assert sampled_rows_error(y, x, w_t, a, b, 2.0, rows=256) <= TIGHT


def test_copy_engine_entry_point_rejects_bad_arguments(cuda_device):
    lib = _abi.load()
    dest = torch.empty(512, 256, dtype=torch.bfloat16, device=cuda_device)
    ptrs = (ctypes.c_void_p * 1)(dest.data_ptr())
    z = ctypes.c_void_p(dest.data_ptr())
    ws = ctypes.c_void_p(dest.data_ptr())
    args = (z, z, z, z, 0, z, 0, 1, ptrs)
    tail = (256, 0, 512, 512, 128, 16, 1.0, _abi.CF_DTYPE_BF16, ws, 16, None)
    # self_dest outside [0, n_dest)
    assert lib.cf_lora_linear_int8_allgather_ce(*args, 1, *tail) == _abi.CF_ERR_INVALID_ARGUMENT
    # workspace smaller than the counters need
    assert lib.cf_lora_linear_int8_allgather_ce(*args, 0, *tail) == _abi.CF_ERR_WORKSPACE


@pytest.mark.parametrize(("m", "rank", "b_t"), [(1, 16, False), (17, 32, True), (32, 64, False),
                                                (33, 16, True), (64, 32, False), (100, 64, True),
                                                (128, 16, False)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_w8_decode_shapes(m, rank, b_t, dtype, cuda_device):
    # Token counts up to 128 take the split-K decode kernel; n = 1000 leaves a
    # ragged last feature tile and k = 1536 a K split that does not divide.
    x, w, a, b = make(m, 1536, 1000, rank, dtype, seed=300 + m + rank)
    dev = cuda_device
    codes, scales = cf.quantize_int8(w.to(dev))
    y = cf.lora_linear_int8(x.to(dev), codes, scales, a.to(dev), as_layout(b.to(dev), b_t), 2.0)
    ref = linear_ref.lora_linear_int8(x, codes.cpu(), scales.cpu(), a, b, 2.0)
    assert linear_ref.max_rel_error(y, ref) <= TIGHT
    assert _abi.load().cf_device_status() == _abi.CF_OK


# ---------------------------------------------------------------------------
# fp32 lora_linear (the reference's own CUDA dtype): three tf32 products on the
# tensor cores. Checked against an fp64 CPU composition with the reference's
# own tolerances (tests/python/test_ops.py:105-138: rtol = atol = 1e-4; the
# CUDA kernel test, tests/cuda/test_lora.cu:107, uses 1e-3).
# ---------------------------------------------------------------------------
def _f64_lora(x, w, a, b, scale):
    x, w, a, b = (t.detach().cpu().double() for t in (x, w, a, b))
    return x @ w + scale * ((x @ a) @ b)


@pytest.mark.parametrize(("batch", "k", "n", "rank"),
                         [(1, 8, 4, 2), (4, 64, 32, 8), (7, 129, 65, 3), (16, 256, 256, 16)])
def test_f32_matches_the_definition_at_the_reference_tolerance(batch, k, n, rank, cuda_device):
    g = torch.Generator().manual_seed(batch * 1000 + k)
    x = torch.randn(batch, k, generator=g)
    w = torch.randn(k, n, generator=g)
    a = torch.randn(k, rank, generator=g)
    b = torch.randn(rank, n, generator=g)
    y = cf.lora_linear(x.to(cuda_device), w.to(cuda_device), a.to(cuda_device), b.to(cuda_device),
                       0.25)
    assert y.dtype == torch.float32 and y.shape == (batch, n)
    torch.testing.assert_close(y.cpu().double(), _f64_lora(x, w, a, b, 0.25), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize(("m", "k", "n", "rank"), [(300, 1024, 768, 16), (1024, 4096, 1024, 64),
                                                   (129, 512, 4100, 32)])
@pytest.mark.parametrize("w_t", [False, True])
@pytest.mark.parametrize("ab_t", [False, True])
def test_f32_shapes_and_layouts(m, k, n, rank, w_t, ab_t, cuda_device):
    g = torch.Generator().manual_seed(m + k + n + rank)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(k, n, generator=g) * 0.05
    a = torch.randn(k, rank, generator=g) * 0.05
    b = torch.randn(rank, n, generator=g) * 0.05
    dev = cuda_device
    y = cf.lora_linear(x.to(dev), as_layout(w.to(dev), w_t), as_layout(a.to(dev), ab_t),
                       as_layout(b.to(dev), ab_t), 2.0)
    ref = _f64_lora(x, w, a, b, 2.0)
    # K up to 4096: measured against the output's scale (fp32 accumulation
    # alone moves elements by ~1e-5 of it).
    assert (y.cpu().double() - ref).abs().max() <= 1e-4 * ref.abs().max()


def test_f32_zero_b_reduces_to_the_frozen_layer(cuda_device):
    # The reference's shapes and tolerance (tests/python/test_ops.py:117-126).
    g = torch.Generator().manual_seed(11)
    x, w = torch.randn(4, 32, generator=g), torch.randn(32, 16, generator=g)
    a, b = torch.randn(32, 4, generator=g), torch.zeros(4, 16)
    y = cf.lora_linear(x.to(cuda_device), w.to(cuda_device), a.to(cuda_device), b.to(cuda_device),
                       1.0)
    torch.testing.assert_close(y.cpu().double(), x.double() @ w.double(), rtol=1e-5, atol=1e-5)
    # and at K = 320, against the output's scale
    x, w = torch.randn(64, 320, generator=g), torch.randn(320, 160, generator=g)
    a, b = torch.randn(320, 4, generator=g), torch.zeros(4, 160)
    y = cf.lora_linear(x.to(cuda_device), w.to(cuda_device), a.to(cuda_device), b.to(cuda_device),
                       1.0).cpu().double()
    ref = x.double() @ w.double()
    assert (y - ref).abs().max() <= 1e-5 * ref.abs().max()


def test_f32_through_the_c_abi(cuda_device):
    m, k, n, r = 256, 512, 384, 32
    g = torch.Generator().manual_seed(12)
    x, w = torch.randn(m, k, generator=g), torch.randn(k, n, generator=g) * 0.05
    a, b = torch.randn(k, r, generator=g) * 0.05, torch.randn(r, n, generator=g) * 0.05
    xd, wd, ad, bd = (t.to(cuda_device) for t in (x, w, a, b))
    lib = _abi.load()
    y = torch.empty(m, n, dtype=torch.float32, device=cuda_device)
    ws_bytes = lib.cf_lora_linear_workspace_bytes(m, r)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    _abi.check(lib.cf_lora_linear(p(xd), p(wd), _abi.CF_LAYOUT_REF, p(ad), _abi.CF_LAYOUT_REF,
                                  p(bd), _abi.CF_LAYOUT_REF, p(y), m, k, n, r, 0.5,
                                  _abi.CF_DTYPE_F32, p(ws), ws_bytes, s), "cf_lora_linear")
    torch.testing.assert_close(y.cpu().double(), _f64_lora(x, w, a, b, 0.5), rtol=1e-4, atol=1e-4)
    assert lib.cf_device_status() == _abi.CF_OK


@pytest.mark.parametrize(("m", "k", "n"), [(7, 129, 65), (256, 1024, 512), (1000, 2048, 3000)])
@pytest.mark.parametrize("b_t", [False, True])
def test_matmul_f32(m, k, n, b_t, cuda_device):
    g = torch.Generator().manual_seed(m + k + n)
    a, b = torch.randn(m, k, generator=g), torch.randn(k, n, generator=g)
    ref = a.double() @ b.double()
    bd = as_layout(b.to(cuda_device), b_t)
    precise = cf.matmul_f32(a.to(cuda_device), bd).cpu().double()
    assert (precise - ref).abs().max() <= 2e-5 * ref.abs().max()
    tf32 = cf.matmul_f32(a.to(cuda_device), bd, precise=False).cpu().double()
    # one tf32 product: operands rounded to 10 explicit mantissa bits
    assert (tf32 - ref).abs().max() <= 5e-3 * ref.abs().max()
    assert (tf32 - ref).abs().max() > (precise - ref).abs().max()


@pytest.mark.parametrize("mode", ["kernel", "ce"])
def test_config5_per_rank_shape_into_eight_destinations(mode, cuda_device):
    # Benchmark config 5 at 8 GPUs, one rank's share: K 8192, rank 64, 28672 / 8 = 3584 output
    # features at column offset 3 * 3584 of y [M, 28672], pushed into 8 copies of y (on one GPU
    # here, standing in for the 8 ranks' symmetric buffers). Every copy must hold exactly the
    # single-destination product in this rank's columns and nothing outside them.
    m, k, n, rank, n_dest, ldy = 2048, 8192, 3584, 64, 8, 28672
    col0 = 3 * n
    x, codes, scales, a, b = _w8_case(m, k, n, rank, cuda_device, seed=55)
    dests = [torch.full((m, ldy), 7.0, dtype=torch.bfloat16, device=cuda_device)
             for _ in range(n_dest)]
    ptrs = (ctypes.c_void_p * n_dest)(*[t.data_ptr() for t in dests])
    lib = _abi.load()
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    if mode == "ce":
        fn, ws_bytes = (lib.cf_lora_linear_int8_allgather_ce,
                        lib.cf_lora_linear_int8_allgather_ce_workspace_bytes(m, rank))
    else:
        fn, ws_bytes = lib.cf_lora_linear_int8_allgather, lib.cf_lora_linear_workspace_bytes(m, rank)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
    _abi.check(fn(p(x), p(codes), p(scales), p(a), _abi.CF_LAYOUT_REF, p(b), _abi.CF_LAYOUT_REF,
                  n_dest, ptrs, 3, ldy, col0, m, k, n, rank, 2.0, _abi.CF_DTYPE_BF16, p(ws),
                  ws_bytes, s), mode)
    torch.cuda.synchronize()
    assert lib.cf_device_status() == _abi.CF_OK
    y = cf.lora_linear_int8(x, codes, scales, a, b, 2.0)
    for d in dests:
        assert torch.equal(d[:, col0:col0 + n], y)
        assert (d[:, :col0] == 7.0).all() and (d[:, col0 + n:] == 7.0).all()
    w_t = linear_ref.dequantized_weight_t(codes, scales)
    assert sampled_rows_error(y, x, w_t, a, b, 2.0, rows=128) <= TIGHT
