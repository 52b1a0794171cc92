"""The bounded-wait error path, made to run out on purpose without a fault.

Every barrier wait in the kernels is bounded; on expiry a kernel ORs
CF_ERR_DEVICE_TIMEOUT into the device error word and returns, so the context
stays usable (the non-sticky class of the reference's CudaError::is_sticky,
cuda/include/cudaforge/cuda_error.cuh:15-41). ``cf_debug_expire_wait`` waits
on a barrier that nothing arrives on with that same bounded wait; the test
checks that the host reads the status once, that reading clears it, and that
the next normal call runs and is bit-exact.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import cuda_force_b200 as cf
from cuda_force_b200 import _abi
from oracle import quant_ref

pytestmark = pytest.mark.gpu


def test_an_expired_wait_is_reported_and_the_context_stays_usable(cuda_device):
    lib = _abi.load()
    assert lib.cf_device_status() == _abi.CF_OK  # nothing pending from earlier tests
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _abi.check(lib.cf_debug_expire_wait(50_000_000, stream), "cf_debug_expire_wait")  # 50 ms
    torch.cuda.synchronize()
    assert lib.cf_device_status() == _abi.CF_ERR_DEVICE_TIMEOUT
    assert lib.cf_device_status() == _abi.CF_OK  # read and cleared
    x = torch.randn(1 << 20, generator=torch.Generator().manual_seed(4))
    codes, scales = cf.quantize_int8(x.to(cuda_device))
    ref_codes, ref_scales = quant_ref.quantize(x.numpy())
    assert np.array_equal(codes.cpu().numpy(), ref_codes)
    assert np.array_equal(scales.cpu().numpy(), ref_scales)
    assert lib.cf_device_status() == _abi.CF_OK


def test_expire_wait_rejects_limits_outside_its_range(cuda_device):
    lib = _abi.load()
    assert lib.cf_debug_expire_wait(10, None) == _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_debug_expire_wait(3_000_000_000, None) == _abi.CF_ERR_INVALID_ARGUMENT
