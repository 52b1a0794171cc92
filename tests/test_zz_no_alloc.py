"""The allocation-free LoRA entry point (cf_lora_linear_noalloc).

It exists for callers that cannot allocate device memory for the workspace
(hosts whose HBM is reserved by another allocator, foreign-language hosts
without a CUDA allocator, loops that must not pay cudaMalloc's device
synchronisation). Its workspace is a 4 MiB array inside the library.

Checked through the C ABI against cf_lora_linear (caller-provided workspace)
on two calls in a row with different inputs, so a stale workspace from the
first call would show up in the second. This file is collected last so a run
that stops at the first failure has run every other test; it passes alone in a
fresh process too (its first call does the per-device set-up).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from cuda_force_b200 import _abi
from oracle import linear_ref

pytestmark = pytest.mark.gpu

TIGHT = 5e-3


def p(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


CF_DTYPE = {torch.bfloat16: _abi.CF_DTYPE_BF16, torch.float32: _abi.CF_DTYPE_F32}


def inputs(m, k, n, r, seed, device, dtype=torch.bfloat16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype).to(device)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dtype).to(device)
    a = (torch.randn(k, r, generator=g) * 0.05).to(dtype).to(device)
    b = (torch.randn(r, n, generator=g) * 0.05).to(dtype).to(device)
    return x, w, a, b


def with_workspace(lib, x, w, a, b, m, k, n, r, stream):
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    ws_bytes = lib.cf_lora_linear_workspace_bytes(m, r)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    _abi.check(lib.cf_lora_linear(p(x), p(w), _abi.CF_LAYOUT_T, p(a), _abi.CF_LAYOUT_REF, p(b),
                                  _abi.CF_LAYOUT_REF, p(y), m, k, n, r, 2.0, CF_DTYPE[x.dtype],
                                  p(ws), ws_bytes, stream), "cf_lora_linear")
    return y


def no_alloc(lib, x, w, a, b, m, k, n, r, stream):
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    _abi.check(lib.cf_lora_linear_noalloc(p(x), p(w), _abi.CF_LAYOUT_T, p(a), _abi.CF_LAYOUT_REF,
                                          p(b), _abi.CF_LAYOUT_REF, p(y), m, k, n, r, 2.0,
                                          CF_DTYPE[x.dtype], stream), "cf_lora_linear_noalloc")
    return y


def test_no_alloc_matches_the_workspace_entry_point_on_two_calls(cuda_device):
    lib = _abi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, (m, k, n, r, seed) in enumerate([(512, 1024, 768, 16, 11), (300, 512, 1024, 64, 12)]):
        x, w, a, b = inputs(m, k, n, r, seed, cuda_device)
        y_ref = with_workspace(lib, x, w, a, b, m, k, n, r, stream)
        y = no_alloc(lib, x, w, a, b, m, k, n, r, stream)
        torch.cuda.synchronize()
        err = linear_ref.max_rel_error(y, y_ref)
        assert err <= TIGHT, f"call {call}: max relative error {err} against cf_lora_linear"
        oracle_err = linear_ref.max_rel_error(y, linear_ref.lora_linear(x, w.t(), a, b, 2.0))
        assert oracle_err <= TIGHT
    assert lib.cf_device_status() == _abi.CF_OK


def test_no_alloc_fp32_matches_the_workspace_entry_point_on_two_calls(cuda_device):
    # fp32 calls keep the down-projection in fp32: 4 bytes per workspace element.
    lib = _abi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, (m, k, n, r, seed) in enumerate([(384, 512, 256, 16, 21), (257, 256, 512, 32, 22)]):
        x, w, a, b = inputs(m, k, n, r, seed, cuda_device, torch.float32)
        y_ref = with_workspace(lib, x, w, a, b, m, k, n, r, stream)
        y = no_alloc(lib, x, w, a, b, m, k, n, r, stream)
        torch.cuda.synchronize()
        err = linear_ref.max_rel_error(y, y_ref)
        assert err <= 1e-5, f"call {call}: max relative error {err} against cf_lora_linear"
    assert lib.cf_device_status() == _abi.CF_OK


@pytest.mark.parametrize(("dtype", "m"), [(torch.bfloat16, 131072), (torch.float32, 65536)])
def test_no_alloc_at_its_limit(dtype, m, cuda_device):
    # The largest call that fits the 4 MiB array at rank 16: m * 16 * (2 or 4) bytes = 4 MiB.
    lib = _abi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    k, n, r = 128, 256, 16
    x, w, a, b = inputs(m, k, n, r, 31, cuda_device, dtype)
    y_ref = with_workspace(lib, x, w, a, b, m, k, n, r, stream)
    y = no_alloc(lib, x, w, a, b, m, k, n, r, stream)
    torch.cuda.synchronize()
    tol = TIGHT if dtype == torch.bfloat16 else 1e-5
    assert linear_ref.max_rel_error(y, y_ref) <= tol
    assert lib.cf_device_status() == _abi.CF_OK


@pytest.mark.parametrize(("dtype", "m"), [(_abi.CF_DTYPE_BF16, 131073), (_abi.CF_DTYPE_F32, 65537)])
def test_no_alloc_rejects_a_workspace_beyond_its_limit(dtype, m, cuda_device):
    lib = _abi.load()
    f = ctypes.c_void_p(0x1000)
    # one row past the limit at rank 16: refused before any launch.
    st = lib.cf_lora_linear_noalloc(f, f, _abi.CF_LAYOUT_T, f, _abi.CF_LAYOUT_REF, f,
                                    _abi.CF_LAYOUT_REF, f, m, 64, 64, 16, 1.0, dtype, None)
    assert st == _abi.CF_ERR_WORKSPACE
