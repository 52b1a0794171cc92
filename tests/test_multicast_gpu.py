"""The multicast-store epilogue of the column-sharded W8 linear on one GPU.

``cf_lora_linear_int8_allgather_mc`` writes this rank's columns once, with
multimem stores, to the NVLink multicast address of y; the switch delivers
each store to every GPU bound to the multicast object. Here the object has
one member, this GPU (built with the CUDA driver's multicast API), so the
test sees the multimem path land in the one bound copy: the columns must
equal the plain single-destination product bit for bit, and nothing outside
them may change. On several GPUs the same kernel runs under
``bench.py --gpus N`` (config 5, every rank's slice checked against the
oracle).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

import cuda_force_b200 as cf
from cuda_force_b200 import _abi

pytestmark = pytest.mark.gpu


def _ok(result):
    err = result[0] if isinstance(result, tuple) else result
    assert int(err) == 0, f"CUDA driver call failed: {err}"
    return result[1] if isinstance(result, tuple) and len(result) == 2 else result


class _Mapped:
    """One device's memory bound to a one-member multicast object, mapped twice:
    the plain (unicast) view and the multicast view."""

    def __init__(self, nbytes: int, ordinal: int):
        from cuda.bindings import driver as cu

        self.cu = cu
        torch.cuda.init()
        self.dev = _ok(cu.cuDeviceGet(ordinal))
        attr = cu.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED
        self.supported = bool(_ok(cu.cuDeviceGetAttribute(attr, self.dev)))
        self.parts = []
        if not self.supported:
            return
        fd = cu.CUmemAllocationHandleType.CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR
        mprop = cu.CUmulticastObjectProp()
        mprop.numDevices = 1
        mprop.handleTypes = fd
        mprop.size = nbytes
        gran = _ok(cu.cuMulticastGetGranularity(
            mprop, cu.CUmulticastGranularity_flags.CU_MULTICAST_GRANULARITY_RECOMMENDED))
        aprop = cu.CUmemAllocationProp()
        aprop.type = cu.CUmemAllocationType.CU_MEM_ALLOCATION_TYPE_PINNED
        aprop.location.type = cu.CUmemLocationType.CU_MEM_LOCATION_TYPE_DEVICE
        aprop.location.id = ordinal
        aprop.requestedHandleTypes = fd
        agran = _ok(cu.cuMemGetAllocationGranularity(
            aprop, cu.CUmemAllocationGranularity_flags.CU_MEM_ALLOC_GRANULARITY_RECOMMENDED))
        g = max(int(gran), int(agran))
        self.size = (nbytes + g - 1) // g * g
        mprop.size = self.size
        self.mc = _ok(cu.cuMulticastCreate(mprop))
        self.parts.append(("mc", self.mc))
        _ok(cu.cuMulticastAddDevice(self.mc, self.dev))
        self.phys = _ok(cu.cuMemCreate(self.size, aprop, 0))
        self.parts.append(("phys", self.phys))
        _ok(cu.cuMulticastBindMem(self.mc, 0, self.phys, 0, self.size, 0))
        self.parts.append(("bind", None))
        access = cu.CUmemAccessDesc()
        access.location.type = cu.CUmemLocationType.CU_MEM_LOCATION_TYPE_DEVICE
        access.location.id = ordinal
        access.flags = cu.CUmemAccess_flags.CU_MEM_ACCESS_FLAGS_PROT_READWRITE
        self.uc_va = _ok(cu.cuMemAddressReserve(self.size, g, 0, 0))
        self.parts.append(("va", self.uc_va))
        _ok(cu.cuMemMap(self.uc_va, self.size, 0, self.phys, 0))
        self.parts.append(("map", self.uc_va))
        _ok(cu.cuMemSetAccess(self.uc_va, self.size, [access], 1))
        self.mc_va = _ok(cu.cuMemAddressReserve(self.size, g, 0, 0))
        self.parts.append(("va", self.mc_va))
        _ok(cu.cuMemMap(self.mc_va, self.size, 0, self.mc, 0))
        self.parts.append(("map", self.mc_va))
        _ok(cu.cuMemSetAccess(self.mc_va, self.size, [access], 1))

    def close(self) -> None:
        cu = self.cu
        torch.cuda.synchronize()
        for kind, obj in reversed(self.parts):
            if kind == "map":
                cu.cuMemUnmap(obj, self.size)
            elif kind == "va":
                cu.cuMemAddressFree(obj, self.size)
            elif kind == "bind":
                cu.cuMulticastUnbind(self.mc, self.dev, 0, self.size)
            elif kind in ("phys", "mc"):
                cu.cuMemRelease(obj)
        self.parts = []


class _View:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


def test_multicast_epilogue_matches_the_plain_product(cuda_device):
    m, k, n, rank, ldy, col0 = 1536, 2048, 1024, 64, 3072, 1024
    g = torch.Generator(device=cuda_device).manual_seed(77)
    x = torch.randn(m, k, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=cuda_device, generator=g) * 0.015).to(torch.bfloat16)
    a = (torch.randn(k, rank, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(rank, n, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    codes, scales = cf.quantize_int8(w)
    mapped = _Mapped(m * ldy * 2, cuda_device.index or 0)
    try:
        if not mapped.supported:
            pytest.skip("this GPU reports no multicast support")
        y = torch.as_tensor(_View(int(mapped.uc_va), (m, ldy), "<i2"), device=cuda_device)
        y = y.view(torch.bfloat16)
        y.fill_(7.0)
        lib = _abi.load()
        ws_bytes = lib.cf_lora_linear_workspace_bytes(m, rank)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for call in range(2):
            _abi.check(lib.cf_lora_linear_int8_allgather_mc(
                p(x), p(codes), p(scales), p(a), _abi.CF_LAYOUT_REF, p(b), _abi.CF_LAYOUT_REF,
                ctypes.c_void_p(int(mapped.uc_va)), ctypes.c_void_p(int(mapped.mc_va)), ldy, col0,
                m, k, n, rank, 2.0, _abi.CF_DTYPE_BF16, p(ws), ws_bytes, s),
                "cf_lora_linear_int8_allgather_mc")
            torch.cuda.synchronize()
            assert lib.cf_device_status() == _abi.CF_OK
            ref = cf.lora_linear_int8(x, codes, scales, a, b, 2.0)
            assert torch.equal(y[:, col0:col0 + n], ref), f"call {call}"
            assert (y[:, :col0] == 7.0).all() and (y[:, col0 + n:] == 7.0).all()
            x = x.flip(0).contiguous()  # a different product for the second call
        del y
    finally:
        mapped.close()


def test_multicast_entry_point_rejects_bad_arguments(cuda_device):
    lib = _abi.load()
    z = ctypes.c_void_p(0x10000)
    args = (z, z, z, z, 0, z, 0)
    tail = (512, 512, 128, 16, 1.0, _abi.CF_DTYPE_BF16, z, 1 << 20, None)
    assert lib.cf_lora_linear_int8_allgather_mc(*args, None, z, 256, 0, *tail) == \
        _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_lora_linear_int8_allgather_mc(*args, z, ctypes.c_void_p(0x10008), 256, 0,
                                                *tail) == _abi.CF_ERR_MISALIGNED
    assert lib.cf_lora_linear_int8_allgather_mc(*args, z, z, 256, 200, *tail) == \
        _abi.CF_ERR_INVALID_ARGUMENT
