"""The multicast-store epilogue of the column-sharded W8 linear.

``cf_lora_linear_int8_allgather_mc`` writes this rank's columns once, with
multimem stores, to the NVLink multicast address of y; the switch delivers
each store to every GPU bound to the multicast object. A multicast object
needs at least two member GPUs, so the end-to-end test needs two visible GPUs
(it skips with one): one process binds a buffer on each GPU to one object
(the CUDA driver's multicast API), runs the kernel on GPU 0 only, and reads
both copies. The columns must equal the plain single-destination product bit
for bit on both GPUs, and nothing outside them may change. No kernel waits on
another GPU. Under ``bench.py --gpus N`` the same kernel runs on every rank
(config 5, every rank's slice checked against the oracle).
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
    """One buffer per GPU, all bound to one multicast object; each mapped
    (unicast) on its own GPU, and the multicast view mapped for all of them."""

    def __init__(self, nbytes: int, ordinals: list[int]):
        from cuda.bindings import driver as cu

        self.cu = cu
        for o in ordinals:
            torch.zeros(1, device=torch.device("cuda", o))  # primary contexts
        self.devs = [_ok(cu.cuDeviceGet(o)) for o in ordinals]
        attr = cu.CUdevice_attribute.CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED
        self.supported = all(bool(_ok(cu.cuDeviceGetAttribute(attr, d))) for d in self.devs)
        self.parts = []
        self.uc_va = []
        if not self.supported:
            return
        fd = cu.CUmemAllocationHandleType.CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR
        mprop = cu.CUmulticastObjectProp()
        mprop.numDevices = len(ordinals)
        mprop.handleTypes = fd
        mprop.size = nbytes
        g = int(_ok(cu.cuMulticastGetGranularity(
            mprop, cu.CUmulticastGranularity_flags.CU_MULTICAST_GRANULARITY_RECOMMENDED)))
        access, aprops = [], []
        for o in ordinals:
            a = cu.CUmemAccessDesc()
            a.location.type = cu.CUmemLocationType.CU_MEM_LOCATION_TYPE_DEVICE
            a.location.id = o
            a.flags = cu.CUmemAccess_flags.CU_MEM_ACCESS_FLAGS_PROT_READWRITE
            access.append(a)
            ap = cu.CUmemAllocationProp()
            ap.type = cu.CUmemAllocationType.CU_MEM_ALLOCATION_TYPE_PINNED
            ap.location.type = cu.CUmemLocationType.CU_MEM_LOCATION_TYPE_DEVICE
            ap.location.id = o
            ap.requestedHandleTypes = fd
            aprops.append(ap)
            g = max(g, int(_ok(cu.cuMemGetAllocationGranularity(
                ap, cu.CUmemAllocationGranularity_flags.CU_MEM_ALLOC_GRANULARITY_RECOMMENDED))))
        self.size = (nbytes + g - 1) // g * g
        mprop.size = self.size
        self.mc = _ok(cu.cuMulticastCreate(mprop))
        self.parts.append(("mc", self.mc))
        for d in self.devs:
            _ok(cu.cuMulticastAddDevice(self.mc, d))
        for i, (d, ap) in enumerate(zip(self.devs, aprops)):
            phys = _ok(cu.cuMemCreate(self.size, ap, 0))
            self.parts.append(("phys", phys))
            _ok(cu.cuMulticastBindMem(self.mc, 0, phys, 0, self.size, 0))
            self.parts.append(("bind", d))
            va = _ok(cu.cuMemAddressReserve(self.size, g, 0, 0))
            self.parts.append(("va", va))
            _ok(cu.cuMemMap(va, self.size, 0, phys, 0))
            self.parts.append(("map", va))
            _ok(cu.cuMemSetAccess(va, self.size, [access[i]], 1))
            self.uc_va.append(va)
        self.mc_va = _ok(cu.cuMemAddressReserve(self.size, g, 0, 0))
        self.parts.append(("va", self.mc_va))
        _ok(cu.cuMemMap(self.mc_va, self.size, 0, self.mc, 0))
        self.parts.append(("map", self.mc_va))
        _ok(cu.cuMemSetAccess(self.mc_va, self.size, access, len(access)))

    def close(self) -> None:
        cu = self.cu
        for d in range(torch.cuda.device_count()):
            torch.cuda.synchronize(d)
        for kind, obj in reversed(self.parts):
            if kind == "map":
                cu.cuMemUnmap(obj, self.size)
            elif kind == "va":
                cu.cuMemAddressFree(obj, self.size)
            elif kind == "bind":
                cu.cuMulticastUnbind(self.mc, obj, 0, self.size)
            elif kind in ("phys", "mc"):
                cu.cuMemRelease(obj)
        self.parts = []


class _View:
    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3}


def test_multicast_epilogue_matches_the_plain_product(cuda_device):
    if torch.cuda.device_count() < 2:
        pytest.skip("a multicast object needs two GPUs; one is visible")
    m, k, n, rank, ldy, col0 = 1536, 2048, 1024, 64, 3072, 1024
    g = torch.Generator(device=cuda_device).manual_seed(77)
    x = torch.randn(m, k, device=cuda_device, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, device=cuda_device, generator=g) * 0.015).to(torch.bfloat16)
    a = (torch.randn(k, rank, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    b = (torch.randn(rank, n, device=cuda_device, generator=g) * 0.01).to(torch.bfloat16)
    codes, scales = cf.quantize_int8(w)
    other = torch.device("cuda", 1)
    mapped = _Mapped(m * ldy * 2, [0, 1])
    try:
        if not mapped.supported:
            pytest.skip("these GPUs report no multicast support")
        y0 = torch.as_tensor(_View(int(mapped.uc_va[0]), (m, ldy), "<i2"), device=cuda_device)
        y1 = torch.as_tensor(_View(int(mapped.uc_va[1]), (m, ldy), "<i2"), device=other)
        y0, y1 = y0.view(torch.bfloat16), y1.view(torch.bfloat16)
        y0.fill_(7.0)
        y1.fill_(7.0)
        torch.cuda.synchronize(other)
        lib = _abi.load()
        ws_bytes = lib.cf_lora_linear_workspace_bytes(m, rank)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=cuda_device)
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        s = ctypes.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
        for call in range(2):
            _abi.check(lib.cf_lora_linear_int8_allgather_mc(
                p(x), p(codes), p(scales), p(a), _abi.CF_LAYOUT_REF, p(b), _abi.CF_LAYOUT_REF,
                ctypes.c_void_p(int(mapped.uc_va[0])), ctypes.c_void_p(int(mapped.mc_va)), ldy,
                col0, m, k, n, rank, 2.0, _abi.CF_DTYPE_BF16, p(ws), ws_bytes, s),
                "cf_lora_linear_int8_allgather_mc")
            torch.cuda.synchronize(cuda_device)
            assert lib.cf_device_status() == _abi.CF_OK
            ref = cf.lora_linear_int8(x, codes, scales, a, b, 2.0)
            for y in (y0, y1.to(cuda_device)):
                assert torch.equal(y[:, col0:col0 + n], ref), f"call {call}"
                assert (y[:, :col0] == 7.0).all() and (y[:, col0 + n:] == 7.0).all()
            x = x.flip(0).contiguous()  # a different product for the second call
        del y0, y1
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
