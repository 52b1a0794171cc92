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


def inputs(m, k, n, r, seed, device):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(device)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16).to(device)
    a = (torch.randn(k, r, generator=g) * 0.05).to(torch.bfloat16).to(device)
    b = (torch.randn(r, n, generator=g) * 0.05).to(torch.bfloat16).to(device)
    return x, w, a, b


def with_workspace(lib, x, w, a, b, m, k, n, r, stream):
    y = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    ws_bytes = lib.cf_lora_linear_workspace_bytes(m, r)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    _abi.check(lib.cf_lora_linear(p(x), p(w), _abi.CF_LAYOUT_T, p(a), _abi.CF_LAYOUT_REF, p(b),
                                  _abi.CF_LAYOUT_REF, p(y), m, k, n, r, 2.0, _abi.CF_DTYPE_BF16,
                                  p(ws), ws_bytes, stream), "cf_lora_linear")
    return y


def no_alloc(lib, x, w, a, b, m, k, n, r, stream):
    y = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    _abi.check(lib.cf_lora_linear_noalloc(p(x), p(w), _abi.CF_LAYOUT_T, p(a), _abi.CF_LAYOUT_REF,
                                          p(b), _abi.CF_LAYOUT_REF, p(y), m, k, n, r, 2.0,
                                          _abi.CF_DTYPE_BF16, stream), "cf_lora_linear_noalloc")
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


def test_no_alloc_rejects_a_workspace_beyond_its_limit(cuda_device):
    lib = _abi.load()
    f = ctypes.c_void_p(0x1000)
    # 131073 rows x rank 16 x 2 bytes > 4 MiB: refused before any launch.
    st = lib.cf_lora_linear_noalloc(f, f, _abi.CF_LAYOUT_T, f, _abi.CF_LAYOUT_REF, f,
                                    _abi.CF_LAYOUT_REF, f, 131073, 64, 64, 16, 1.0,
                                    _abi.CF_DTYPE_BF16, None)
    assert st == _abi.CF_ERR_WORKSPACE
